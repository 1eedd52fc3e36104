"""Paged-KV data movement outside attention.

* ``store_kvcache``   -- scatter K/V rows into the pool by flat slot (``slot < 0`` skips);
  the reference's Triton kernel (``llmserve/layers/attention.py:21-57``).  The hot path fuses this
  store into the QK-norm/RoPE kernel; this standalone op serves tests and utilities.
* ``commit_tree_kv``  -- copy the accepted EAGLE3 tree nodes' K/V of every layer into their
  paged slots in one launch (``llmserve/speculative/tree_kv.py:13-76``).
* ``push_blocks``     -- copy whole paged blocks (every layer, K and V) from one pool into another,
  on another GPU over NVLink by peer stores (prefill/decode disaggregation).
* ``embedding``       -- row gather from a replicated embedding table.
"""
import torch

from llmserve_b200.ops._ext import C, status
from llmserve_b200.ops.rope import store_kv_ref


def store_kvcache(k, v, k_cache, v_cache, slot_mapping):
    if not k.is_cuda:
        return store_kv_ref(k, v, k_cache, v_cache, slot_mapping)
    C().store_kvcache(k.contiguous(), v.contiguous(), k_cache, v_cache, slot_mapping.to(torch.int32),
                      status(k.device))


def commit_tree_kv_ref(tree_k, tree_v, k_cache, v_cache, node_indices, slot_mapping):
    """tree_k/v [L, n, nkv, hd]; k/v_cache [L, nblocks, nkv, bs, hd]."""
    bs = k_cache.shape[3]
    for node, slot in zip(node_indices.tolist(), slot_mapping.tolist()):
        blk, off = slot // bs, slot % bs
        k_cache[:, blk, :, off] = tree_k[:, node]
        v_cache[:, blk, :, off] = tree_v[:, node]


def commit_tree_kv(tree_k, tree_v, k_cache, v_cache, node_indices, slot_mapping):
    if tree_k.ndim != 4 or tree_k.shape != tree_v.shape:
        raise ValueError("tree K/V must be [layers, nodes, kv_heads, head_dim]")
    if k_cache.ndim != 5 or k_cache.shape != v_cache.shape:
        raise ValueError("target K/V cache must be [layers, blocks, kv_heads, block_size, head_dim]")
    if (tree_k.shape[0] != k_cache.shape[0] or tree_k.shape[2] != k_cache.shape[2]
            or tree_k.shape[3] != k_cache.shape[4]):
        raise ValueError("tree KV and target cache layer/head shapes must match")
    if node_indices.ndim != 1 or node_indices.numel() != slot_mapping.numel():
        raise ValueError("selected nodes and slots must have matching one-dimensional shapes")
    if not tree_k.is_cuda:
        return commit_tree_kv_ref(tree_k, tree_v, k_cache, v_cache, node_indices, slot_mapping)
    C().commit_tree_kv(tree_k.contiguous(), tree_v.contiguous(), k_cache, v_cache,
                       node_indices.to(torch.int32), slot_mapping.to(torch.int32), status(tree_k.device))


def embedding(ids: torch.Tensor, table: torch.Tensor) -> torch.Tensor:
    if not ids.is_cuda:
        return torch.nn.functional.embedding(ids, table)
    out = torch.empty(ids.shape[0], table.shape[1], dtype=table.dtype, device=table.device)
    C().embedding(out, ids.contiguous(), table, status(table.device))
    return out


def push_blocks(src_k, src_v, dst_k, dst_v, src_ids, dst_ids):
    """Copy blocks ``src_ids`` of the pools ``src_k/src_v [L, Bs, kvh, bs, hd]`` into blocks
    ``dst_ids`` of ``dst_k/dst_v [L, Bd, kvh, bs, hd]``.  On CUDA the copy is one kernel on the
    source GPU's current stream whose stores go straight to the destination GPU (peer access is
    enabled on first use); the caller orders the destination's readers after it (an event)."""
    if len(src_ids) != len(dst_ids):
        raise ValueError("source and destination block lists differ in length")
    if not len(src_ids):
        return
    if not src_k.is_cuda:
        si = torch.as_tensor(src_ids, dtype=torch.long)
        di = torch.as_tensor(dst_ids, dtype=torch.long)
        dst_k[:, di] = src_k[:, si].to(dst_k.device)
        dst_v[:, di] = src_v[:, si].to(dst_v.device)
        return
    dev = src_k.device
    si = torch.as_tensor(src_ids, dtype=torch.int32).to(dev, non_blocking=True)
    di = torch.as_tensor(dst_ids, dtype=torch.int32).to(dev, non_blocking=True)
    C().kv_push(src_k, src_v, dst_k, dst_v, si, di, status(dev))
