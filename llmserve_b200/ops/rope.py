"""Rotary embedding (neox halves) with optional per-head QK RMSNorm, fused with the paged
K/V store.

Reference math: ``llmserve/layers/rotary_embedding.py`` (cos/sin cache of
``max_position x head_dim/2``, rotation in fp32, result rounded to the activation dtype) and
``llmserve/models/qwen3.py:83-96`` (q_norm/k_norm per head before RoPE).  On CUDA one kernel
reads the packed ``qkv`` row once, writes the rotated query to ``q_out`` and the rotated key /
raw value straight into the paged cache at ``slot_mapping`` (slot < 0 skips the store), which
replaces the separate norm, rope and ``store_kvcache`` launches of the reference.  Without a
bound cache (tree verify) a sibling kernel returns rotated q and k instead.
"""
import torch

from llmserve_b200.ops._ext import C, status
from llmserve_b200.ops.norm import rms_norm_ref


def build_cos_sin_cache(head_dim: int, max_position: int, base: float, device=None) -> torch.Tensor:
    inv_freq = 1.0 / (base ** (torch.arange(0, head_dim, 2, dtype=torch.float) / head_dim))
    t = torch.arange(max_position, dtype=torch.float)
    freqs = torch.outer(t, inv_freq)
    return torch.cat([freqs.cos(), freqs.sin()], dim=-1).to(device)  # [P, head_dim] fp32


def apply_rope_ref(x: torch.Tensor, positions: torch.Tensor, cos_sin: torch.Tensor) -> torch.Tensor:
    cs = cos_sin[positions]
    cos, sin = cs.chunk(2, dim=-1)
    cos, sin = cos.unsqueeze(1), sin.unsqueeze(1)
    x1, x2 = x.float().chunk(2, dim=-1)
    return torch.cat([x1 * cos - x2 * sin, x2 * cos + x1 * sin], dim=-1).to(x.dtype)


def store_kv_ref(k, v, k_cache, v_cache, slot_mapping):
    """k/v: [T, nkv, hd]; caches: [num_blocks, nkv, block_size, hd]."""
    bs = k_cache.shape[2]
    slots = slot_mapping.long()
    keep = slots >= 0
    if not bool(keep.any()):
        return
    slots = slots[keep]
    blk, off = slots // bs, slots % bs
    k_cache[blk, :, off] = k[keep].to(k_cache.dtype)
    v_cache[blk, :, off] = v[keep].to(v_cache.dtype)


def _opt(w, device):
    return w if w is not None else torch.empty(0, device=device)


def qkv_norm_rope_store(qkv, positions, cos_sin, q_norm_w, k_norm_w, eps,
                        k_cache, v_cache, slot_mapping, num_heads, num_kv_heads, head_dim):
    """Split ``qkv [T, (nh+2nkv)*hd]``; return rotated ``(q, k, v)``.  With a bound cache the CUDA
    path stores k/v into it and returns ``(q, None, None)``.  On CUDA ``qkv`` may also be the fp32
    split-K partials ``[S, T, W]`` of the QKV projection, reduced inside the kernel."""
    if qkv.dtype == torch.float32 and qkv.dim() == 3 and qkv.is_cuda:
        if k_cache is None or not k_cache.numel():
            qkv = qkv.sum(0).to(torch.bfloat16)
            return qkv_norm_rope_store(qkv, positions, cos_sin, q_norm_w, k_norm_w, eps, k_cache, v_cache,
                                       slot_mapping, num_heads, num_kv_heads, head_dim)
        T = qkv.shape[1]
        q = torch.empty(T, num_heads, head_dim, dtype=torch.bfloat16, device=qkv.device)
        C().qkv_rope(q, q, qkv, positions, cos_sin, _opt(q_norm_w, qkv.device), _opt(k_norm_w, qkv.device), eps,
                     k_cache, v_cache, slot_mapping, num_heads, num_kv_heads, head_dim, True, status(qkv.device))
        return q, None, None
    T = qkv.shape[0]
    qs, ks = num_heads * head_dim, num_kv_heads * head_dim
    if qkv.is_cuda:
        qkv = qkv.contiguous()
        q = torch.empty(T, num_heads, head_dim, dtype=qkv.dtype, device=qkv.device)
        if k_cache is not None and k_cache.numel():
            C().qkv_rope(q, q, qkv, positions, cos_sin, _opt(q_norm_w, qkv.device),
                         _opt(k_norm_w, qkv.device), eps, k_cache, v_cache, slot_mapping,
                         num_heads, num_kv_heads, head_dim, True, status(qkv.device))
            return q, None, None
        k = torch.empty(T, num_kv_heads, head_dim, dtype=qkv.dtype, device=qkv.device)
        e = _opt(None, qkv.device)
        C().qkv_rope(q, k, qkv, positions, cos_sin, _opt(q_norm_w, qkv.device), _opt(k_norm_w, qkv.device),
                     eps, e, e, e, num_heads, num_kv_heads, head_dim, False, status(qkv.device))
        v = qkv[:, qs + ks:].reshape(T, num_kv_heads, head_dim)
        return q, k, v
    q = qkv[:, :qs].reshape(T, num_heads, head_dim)
    k = qkv[:, qs:qs + ks].reshape(T, num_kv_heads, head_dim)
    v = qkv[:, qs + ks:].reshape(T, num_kv_heads, head_dim)
    if q_norm_w is not None:
        q = rms_norm_ref(q, q_norm_w, eps)
        k = rms_norm_ref(k, k_norm_w, eps)
    q = apply_rope_ref(q, positions, cos_sin)
    k = apply_rope_ref(k, positions, cos_sin)
    if k_cache is not None and k_cache.numel():
        store_kv_ref(k, v, k_cache, v_cache, slot_mapping)
    return q, k, v
