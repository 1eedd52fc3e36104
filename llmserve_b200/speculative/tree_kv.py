"""Commit of the accepted tree path's K/V into the paged target cache.

Parity with ``TreeKVCacheManager`` of the reference (``llmserve/speculative/tree_kv.py:79-154``):
during a tree verify every target attention layer keeps the K/V of all tree nodes in
``tree_k`` / ``tree_v`` (``[nodes, kv_heads, head_dim]``, not written to the pool); after
acceptance :meth:`TreeKVCacheManager.commit` checks the captures, copies the selected nodes of
every layer into their slots with one kernel (``ops.kv.commit_tree_kv``: grid over layers x
nodes, 16-byte vector copies) and clears the captures whether or not the commit succeeded, so a
failed step never leaves stale tree K/V behind.
"""
from collections.abc import Sequence

import torch

from llmserve_b200.ops import kv as kv_ops


class TreeKVCacheManager:
    """Owns the per-layer tree captures of one target model between verify and commit.

    ``attention_layers`` are objects with ``tree_k`` / ``tree_v`` attributes; ``k_cache`` /
    ``v_cache`` are the target pools ``[layers, blocks, kv_heads, block_size, head_dim]``."""

    def __init__(self, attention_layers: Sequence, *, k_cache: torch.Tensor | None = None,
                 v_cache: torch.Tensor | None = None):
        if not attention_layers:
            raise ValueError("a tree K/V manager needs at least one attention layer")
        self.attention_layers = list(attention_layers)
        self.k_cache, self.v_cache = k_cache, v_cache

    def clear(self):
        for layer in self.attention_layers:
            layer.tree_k = layer.tree_k.new_empty(0)
            layer.tree_v = layer.tree_v.new_empty(0)

    def _check(self, node_indices: list[int], slot_mapping: torch.Tensor) -> int:
        if slot_mapping.ndim != 1 or slot_mapping.numel() != len(node_indices):
            raise ValueError("tree K/V slot count must match the number of selected nodes")
        shape = None
        for layer in self.attention_layers:
            if layer.tree_k.numel() == 0 or layer.tree_v.numel() == 0:
                raise ValueError("every target layer must capture tree K/V before a commit")
            if layer.tree_k.shape != layer.tree_v.shape:
                raise ValueError("tree K and V captures must have the same shape")
            if shape is not None and layer.tree_k.shape != shape:
                raise ValueError("all target layers must capture tree K/V of the same shape")
            shape = layer.tree_k.shape
        nodes = shape[0]
        if not node_indices or any(not isinstance(i, int) or not 0 <= i < nodes for i in node_indices):
            raise ValueError(f"tree K/V node index out of range 0..{nodes - 1}: {node_indices}")
        return nodes

    def commit(self, node_indices: list[int], slot_mapping: torch.Tensor):
        """Write nodes ``node_indices`` of every layer's capture to ``slot_mapping`` (one slot per node)."""
        try:
            self._check(node_indices, slot_mapping)
            if self.k_cache is None or self.v_cache is None:
                raise ValueError("a tree K/V commit needs the target K/V pools")
            tree_k = torch.stack([layer.tree_k for layer in self.attention_layers])
            tree_v = torch.stack([layer.tree_v for layer in self.attention_layers])
            nodes = torch.tensor(node_indices, dtype=torch.int32, device=tree_k.device)
            kv_ops.commit_tree_kv(tree_k, tree_v, self.k_cache, self.v_cache, nodes, slot_mapping)
        finally:
            self.clear()
