"""RMSNorm and fused residual-add + RMSNorm.

Math parity with ``llmserve/layers/layernorm.py:16-40`` of the reference: statistics in fp32,
the normalised value is rounded to the activation dtype *before* the weight multiply, and the
fused variant returns ``residual = (x + residual)`` rounded to the activation dtype.
"""
import torch

from llmserve_b200.ops._ext import C


def rms_norm_ref(x: torch.Tensor, weight: torch.Tensor, eps: float) -> torch.Tensor:
    xf = x.float()
    inv = torch.rsqrt(xf.pow(2).mean(dim=-1, keepdim=True) + eps)
    return (xf * inv).to(x.dtype) * weight


def add_rms_norm_ref(x, residual, weight, eps):
    s = x.float() + residual.float()
    new_residual = s.to(x.dtype)
    inv = torch.rsqrt(s.pow(2).mean(dim=-1, keepdim=True) + eps)
    return (s * inv).to(x.dtype) * weight, new_residual


def rms_norm(x: torch.Tensor, weight: torch.Tensor, eps: float) -> torch.Tensor:
    if not x.is_cuda:
        return rms_norm_ref(x, weight, eps)
    x2 = x.reshape(-1, x.shape[-1]).contiguous()
    out = torch.empty_like(x2)
    C().rms_norm(out, x2, weight, eps)
    return out.view_as(x)


def add_rms_norm(x: torch.Tensor, residual: torch.Tensor, weight: torch.Tensor, eps: float):
    """Returns ``(rmsnorm(x + residual) * w, x + residual)``."""
    if not x.is_cuda:
        return add_rms_norm_ref(x, residual, weight, eps)
    out = torch.empty_like(x)
    res_out = torch.empty_like(residual)
    C().add_rms_norm(out, res_out, x.contiguous(), residual.contiguous(), weight, eps)
    return out, res_out
