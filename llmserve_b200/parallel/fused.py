"""Row-parallel projection fused with its reduction, residual add and the following RMSNorm.

Per rank, the sm_100a GEMM writes fp32 split-K partials of ``x_r @ W_r^T``.  Then one kernel
finishes the layer:

* TP = 1: sum the split-K partials, add the residual, RMSNorm -> (normed bf16, residual bf16).
* TP > 1 with ``FusedComm`` (``llmserve_b200.parallel.comm``): partials land in a peer-mapped
  buffer and the finishing kernel reduces every rank's partials over NVLink for its share of the
  rows, applies residual + RMSNorm and pushes the finished rows to every peer.
* TP > 1 without ``FusedComm`` (baseline): split-K reduce to bf16, NCCL all-reduce, add+RMSNorm.

This replaces ``dist.all_reduce`` (``llmserve/layers/linear.py:234-235``) plus the separate
``add_rms_forward`` of the reference.
"""
import os
import torch

from llmserve_b200.ops import gemm, norm as norm_ops
from llmserve_b200.ops._ext import C
from llmserve_b200.parallel import state as tp

# the reduction epilogue reads every split; 4 costs the GEMM almost nothing (B200 sweep)
ROW_PARALLEL_MAX_SPLITS = int(os.environ.get("LLMSERVE_ROW_SPLITS", "64"))


def row_parallel_add_norm(x, weight, residual, norm_weight, eps, fused=None):
    x = x.contiguous()
    T, K = x.shape
    N = weight.shape[0]
    world = tp.get_tp_size()
    if fused is not None and world > 1 and fused.can_handle(T, N):
        return fused.row_parallel_add_norm(x, weight, residual, norm_weight, eps)
    if gemm.use_cluster(T, weight):
        partials = gemm.linear_reduced(x, weight, plane=True)
    else:
        splits = min(gemm.splits_for(T, weight), ROW_PARALLEL_MAX_SPLITS)
        partials = gemm.linear_partials(x, weight, splits)
    if world == 1:
        out = torch.empty(T, N, dtype=x.dtype, device=x.device)
        res_out = torch.empty_like(residual)
        C().splitk_reduce_add_rmsnorm(out, res_out, partials, residual.contiguous(), norm_weight, eps)
        return out, res_out
    y = torch.empty(T, N, dtype=x.dtype, device=x.device)
    C().splitk_reduce(y, partials)
    tp.all_reduce(y)
    return norm_ops.add_rms_norm(y, residual, norm_weight, eps)
