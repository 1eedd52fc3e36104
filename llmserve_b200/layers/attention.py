"""Attention layer over the paged KV pool (``llmserve/layers/attention.py:60-133`` of the reference).

The QK RMSNorm, RoPE and the K/V store into the pool run as one kernel; then prefill (varlen
paged) or decode (split-KV) attention reads the pool.  In tree-verify mode the nodes' K/V are not
stored: they are captured in ``tree_k``/``tree_v`` and attended with the ancestor mask, and the
accepted path is committed afterwards by ``ops.kv.commit_tree_kv``.
"""
import torch
from torch import nn

from llmserve_b200.ops import attention as attn_ops
from llmserve_b200.ops import rope as rope_ops
from llmserve_b200.utils.context import get_context


class Attention(nn.Module):

    def __init__(self, num_heads: int, head_dim: int, scale: float, num_kv_heads: int):
        super().__init__()
        self.num_heads, self.head_dim, self.scale, self.num_kv_heads = num_heads, head_dim, scale, num_kv_heads
        self.k_cache = self.v_cache = torch.tensor([])
        self.tree_k = self.tree_v = torch.tensor([])

    def forward(self, qkv: torch.Tensor, positions: torch.Tensor, cos_sin: torch.Tensor,
                q_norm_w: torch.Tensor | None, k_norm_w: torch.Tensor | None, eps: float) -> torch.Tensor:
        ctx = get_context()
        T = positions.shape[0]
        if ctx.tree_attention_mask is not None:
            q, k, v = rope_ops.qkv_norm_rope_store(qkv, positions, cos_sin, q_norm_w, k_norm_w, eps,
                                                   None, None, None, self.num_heads, self.num_kv_heads,
                                                   self.head_dim)
            self.tree_k, self.tree_v = k.contiguous(), v.contiguous()
            o = attn_ops.tree_attention(q, self.k_cache, self.v_cache, ctx.tree_block_table,
                                        ctx.tree_prefix_len, self.tree_k, self.tree_v,
                                        ctx.tree_attention_mask, self.scale, ctx.tree_mask_bits)
            return o.reshape(T, -1)
        q, _, _ = rope_ops.qkv_norm_rope_store(qkv, positions, cos_sin, q_norm_w, k_norm_w, eps,
                                               self.k_cache, self.v_cache, ctx.slot_mapping,
                                               self.num_heads, self.num_kv_heads, self.head_dim)
        if ctx.is_prefill and ctx.uniform_q and q.is_cuda and attn_ops.verify_fits_decode_kernel(
                ctx.uniform_q, self.num_heads, self.num_kv_heads, self.k_cache.shape[2], self.head_dim):
            o = attn_ops.verify_attention(q, self.k_cache, self.v_cache, ctx.block_tables, ctx.seqlens_k, self.scale,
                                          ctx.uniform_q, ctx.decode_workspace)
        elif ctx.is_prefill:
            o = attn_ops.prefill_attention(q, self.k_cache, self.v_cache, ctx.cu_seqlens_q, ctx.seqlens_k,
                                           ctx.block_tables, self.scale, ctx.max_seqlen_q)
        else:
            o = attn_ops.decode_attention(q, self.k_cache, self.v_cache, ctx.block_tables, ctx.context_lens,
                                          self.scale, ctx.decode_workspace)
        return o.reshape(T, -1)
