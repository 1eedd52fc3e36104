"""Paged attention over a KV pool laid out ``[num_blocks, kv_heads, block_size, head_dim]``.

One layout serves every path: a 64-key tile of one head is a contiguous 16 KiB run, so the
prefill kernel streams it with bulk copies, and a whole block of a layer is one contiguous
region for the prefill->decode KV push.

* ``decode_attention``  -- one query token per sequence (``flash_attn_with_kvcache`` in the
  reference, ``llmserve/layers/attention.py:130-132``).  Persistent sm_100a kernel: one CTA per
  SM pair slot, a producer warp streams K/V pages with 2-D tensor copies (128B swizzle) through a
  3-stage ring, four warps run the GQA math with the query heads of one KV head packed together; chunks of
  long contexts are merged (log-sum-exp) by the CTA that finishes last, so one launch per layer.
  The earlier cp.async split-KV kernel remains for block sizes the tensor copy cannot tile.
* ``prefill_attention`` -- varlen causal attention of a query chunk against the paged keys of
  its sequence (``flash_attn_varlen_func(..., block_table)`` in the reference, ``:121-126``):
  covers plain prefill, chunked prefill, prefix-cache hits and the packed EAGLE3 verify.
  Query ``j`` of a chunk of ``q_len`` against ``k_len`` keys sees keys ``< k_len - q_len + j + 1``.
* ``tree_attention``    -- EAGLE3 tree verify: prefix keys from the pool (all visible) plus the
  tree nodes' own keys under an ancestor mask (``attention.py:77-109`` of the reference).  On the
  tcgen05 kernel (``tree_sm100.cu``) the (node, head) rows of one KV head share a 128-row MMA tile
  and the prefix is split over the SMs; the CUDA-core kernel takes the shapes it does not.
"""
import math
import os

import torch

from llmserve_b200.ops._ext import C, status
from llmserve_b200.ops.gemm import NUM_SMS


def _gather_pages(cache: torch.Tensor, block_table: torch.Tensor, length: int) -> torch.Tensor:
    """[num_blocks, nkv, bs, hd] -> [length, nkv, hd] for one sequence."""
    bs = cache.shape[2]
    nblk = -(-length // bs)
    pages = cache[block_table[:nblk].long()]
    return pages.permute(0, 2, 1, 3).reshape(nblk * bs, cache.shape[1], cache.shape[3])[:length]


def _attend(q, k, v, scale, mask=None):
    """q [Lq, nh, hd], k/v [Lk, nkv, hd] -> [Lq, nh, hd] (fp32 math)."""
    group = q.shape[1] // k.shape[1]
    qf = q.float().transpose(0, 1)
    kf = k.float().repeat_interleave(group, dim=1).transpose(0, 1)
    vf = v.float().repeat_interleave(group, dim=1).transpose(0, 1)
    s = torch.matmul(qf, kf.transpose(1, 2)) * scale
    if mask is not None:
        s = s.masked_fill(~mask.unsqueeze(0), float("-inf"))
    p = torch.softmax(s, dim=-1)
    return torch.matmul(p, vf).transpose(0, 1).to(q.dtype)


def decode_attention_ref(q, k_cache, v_cache, block_tables, context_lens, scale):
    out = torch.empty_like(q)
    for b in range(q.shape[0]):
        n = int(context_lens[b])
        k = _gather_pages(k_cache, block_tables[b], n)
        v = _gather_pages(v_cache, block_tables[b], n)
        out[b] = _attend(q[b:b + 1], k, v, scale)[0]
    return out


def prefill_attention_ref(q, k_cache, v_cache, cu_seqlens_q, seqlens_k, block_tables, scale):
    out = torch.empty_like(q)
    cu_q = cu_seqlens_q.tolist()
    for i in range(len(cu_q) - 1):
        qs, qe = cu_q[i], cu_q[i + 1]
        lq, lk = qe - qs, int(seqlens_k[i])
        k = _gather_pages(k_cache, block_tables[i], lk)
        v = _gather_pages(v_cache, block_tables[i], lk)
        qpos = torch.arange(lk - lq, lk).unsqueeze(1)
        mask = torch.arange(lk).unsqueeze(0) <= qpos
        out[qs:qe] = _attend(q[qs:qe], k, v, scale, mask.to(q.device))
    return out


def tree_attention_ref(q, k_cache, v_cache, block_table, prefix_len, tree_k, tree_v, tree_mask, scale):
    pk = _gather_pages(k_cache, block_table, prefix_len)
    pv = _gather_pages(v_cache, block_table, prefix_len)
    k = torch.cat([pk, tree_k.to(pk.dtype)], 0)
    v = torch.cat([pv, tree_v.to(pv.dtype)], 0)
    mask = torch.cat([torch.ones(q.shape[0], prefix_len, dtype=torch.bool, device=q.device),
                      tree_mask.to(q.device, torch.bool)], dim=1)
    return _attend(q, k, v, scale, mask)


DECODE_PARTITION = 128   # key granularity of a split (the kernel widens splits for large batches)


def decode_partition(batch: int, kv_heads: int) -> int:
    """Keys per split: short splits (more CTAs) for small batches, long pipelined splits once the
    (sequence, kv head) pairs alone fill the GPU."""
    pairs = batch * kv_heads
    return 128 if pairs < 148 else 256 if pairs < 296 else 512


class DecodeWorkspace:
    """Scratch for split-KV partial results, sized once for the largest batch so decode kernels
    can be captured in CUDA graphs (the kernel itself allocates nothing)."""

    def __init__(self, max_batch: int, num_heads: int, head_dim: int, max_context: int, device):
        self.max_batch = max_batch
        self.max_splits = max(1, -(-max_context // 128))
        self.partial_out = torch.empty(max_batch * num_heads * self.max_splits * head_dim,
                                       dtype=torch.float32, device=device)
        self.partial_ml = torch.empty(max_batch * num_heads * self.max_splits * 2,
                                      dtype=torch.float32, device=device)
        # per (sequence, kv head) split-completion counters; the merging CTA resets its counter
        self.counters = torch.zeros(max_batch * num_heads, dtype=torch.int32, device=device)


_DECODE_TMA = os.environ.get("LLMSERVE_DECODE_TMA", "1") != "0"
_TMA_PARTITION = int(os.environ.get("LLMSERVE_DECODE_TMA_PARTITION", "0"))


def tma_partition(batch: int, kv_heads: int) -> int:
    """Keys per work item of the persistent TMA decode kernel: enough items to keep every SM's ring
    busy and to even out the round-robin tail, without paying a partial merge on every chunk."""
    if _TMA_PARTITION:
        return _TMA_PARTITION
    pairs = batch * kv_heads
    return 128 if pairs < NUM_SMS // 2 else 256 if pairs < NUM_SMS else 512


def decode_attention(q, k_cache, v_cache, block_tables, context_lens, scale, workspace=None):
    if not q.is_cuda:
        return decode_attention_ref(q, k_cache, v_cache, block_tables, context_lens, scale)
    B, nh, hd = q.shape
    cap = block_tables.shape[1] * k_cache.shape[2]
    if workspace is None or workspace.max_batch < B or workspace.max_splits * 128 < cap:
        workspace = DecodeWorkspace(B, nh, hd, cap, q.device)
    out = torch.empty_like(q)
    if _DECODE_TMA and C().decode_tma_supported(k_cache.shape[2], hd):
        C().decode_attention_tma(out, q.contiguous(), k_cache, v_cache, block_tables, context_lens, float(scale),
                                 workspace.partial_out, workspace.partial_ml, workspace.counters,
                                 workspace.max_splits, tma_partition(B, k_cache.shape[1]), 1, status(q.device))
        return out
    part = decode_partition(B, k_cache.shape[1])
    C().decode_attention(out, q.contiguous(), k_cache, v_cache, block_tables, context_lens, float(scale),
                         workspace.partial_out, workspace.partial_ml, workspace.counters,
                         -(-workspace.max_splits * 128 // part), part, 0, status(q.device))
    return out


def verify_fits_decode_kernel(nq: int, num_heads: int, num_kv_heads: int, block_size: int, head_dim: int) -> bool:
    """Whether a packed verify chunk of ``nq`` queries per sequence runs on the TMA decode kernel:
    every (query, head) row of a KV head in one 16-row MMA tile."""
    return (_DECODE_TMA and nq >= 1 and nq * (num_heads // num_kv_heads) <= 16
            and C().decode_tma_supported(block_size, head_dim))


def verify_attention(q, k_cache, v_cache, block_tables, seqlens_k, scale, nq: int, workspace=None):
    """Causal attention of ``nq`` consecutive new tokens per sequence (an EAGLE3 verify chunk,
    ``q [B * nq, nh, hd]``, sequence b's tokens at positions ``seqlens_k[b] - nq ..``) against the
    paged pool, on the TMA decode kernel: the (query, head) rows of one KV head share an MMA tile,
    so every K/V byte is read once per KV head instead of once per query head."""
    T, nh, hd = q.shape
    B = T // nq
    if not q.is_cuda:
        cu = torch.arange(0, (B + 1) * nq, nq, dtype=torch.int32)
        return prefill_attention_ref(q, k_cache, v_cache, cu, seqlens_k, block_tables, scale)
    cap = block_tables.shape[1] * k_cache.shape[2]
    if workspace is None or workspace.max_batch < T or workspace.max_splits * 128 < cap:
        workspace = DecodeWorkspace(T, nh, hd, cap, q.device)
    out = torch.empty_like(q)
    C().decode_attention_tma(out, q.contiguous(), k_cache, v_cache, block_tables, seqlens_k, float(scale),
                             workspace.partial_out, workspace.partial_ml, workspace.counters,
                             workspace.max_splits, tma_partition(B, k_cache.shape[1]), int(nq), status(q.device))
    return out


# From this many query rows in the longest sequence of a step, prefill runs on the tcgen05 kernel
# (128-row query tiles); shorter chunks (verify, small chunked-prefill pieces) on the mma.sync one.
PREFILL_TC_MIN_Q = int(os.environ.get("LLMSERVE_PREFILL_TC_MIN_Q", "65"))


def prefill_attention(q, k_cache, v_cache, cu_seqlens_q, seqlens_k, block_tables, scale, max_seqlen_q: int,
                      kernel: str = "auto"):
    """Varlen causal attention of packed query rows against the paged pool.  ``kernel``: "auto"
    (by ``max_seqlen_q``), "tc" (tcgen05 / TMEM / TMA, ``ops/csrc/prefill_sm100.cu``) or "mma"
    (mma.sync tiles, ``ops/csrc/attention.cu``)."""
    if not q.is_cuda:
        return prefill_attention_ref(q, k_cache, v_cache, cu_seqlens_q, seqlens_k, block_tables, scale)
    out = torch.empty_like(q)
    q = q.contiguous()
    bs, hd = k_cache.shape[2], k_cache.shape[3]
    use_tc = kernel == "tc" or (kernel == "auto" and max_seqlen_q >= PREFILL_TC_MIN_Q)
    if use_tc and C().prefill_tc_supported(bs, hd):
        C().prefill_attention_tc(out, q, k_cache, v_cache, cu_seqlens_q, seqlens_k, block_tables, float(scale),
                                 int(max_seqlen_q), status(q.device))
    else:
        C().prefill_attention(out, q, k_cache, v_cache, cu_seqlens_q, seqlens_k, block_tables,
                              float(scale), int(max_seqlen_q), status(q.device))
    return out


# tree verify on the tcgen05 kernel (LLMSERVE_TREE_TC=0: the CUDA-core kernel)
TREE_TC = os.environ.get("LLMSERVE_TREE_TC", "1") != "0"


def tree_attention(q, k_cache, v_cache, block_table, prefix_len, tree_k, tree_v, tree_mask, scale,
                   mask_bits=None):
    """``tree_mask [n_q, n_tree]`` bool; on CUDA the kernel takes one int32 ancestor bitmask per
    query row (``mask_bits``, at most 32 tree nodes)."""
    if not q.is_cuda:
        return tree_attention_ref(q, k_cache, v_cache, block_table, prefix_len, tree_k, tree_v,
                                  tree_mask, scale)
    if mask_bits is None:
        n = tree_mask.shape[1]
        w = 1 << torch.arange(n, dtype=torch.int64, device=q.device)
        mask_bits = (tree_mask.to(q.device).long() * w).sum(1).to(torch.int32)
    out = torch.empty_like(q)
    n_tree = tree_k.shape[0]
    if TREE_TC and C().tree_tc_supported(q.shape[0], q.shape[1], k_cache.shape[1], n_tree, k_cache.shape[2],
                                         q.shape[2]):
        C().tree_attention_tc(out, q.contiguous(), k_cache, v_cache, block_table.to(torch.int32).contiguous(),
                              int(prefix_len), tree_k.contiguous(), tree_v.contiguous(), mask_bits.to(torch.int32),
                              float(scale), status(q.device))
        return out
    C().tree_attention(out, q.contiguous(), k_cache, v_cache, block_table.to(torch.int32), int(prefix_len),
                       tree_k.contiguous(), tree_v.contiguous(), mask_bits, float(scale), status(q.device))
    return out


def default_scale(head_dim: int) -> float:
    return 1.0 / math.sqrt(head_dim)
