"""SiLU-gated multiply: ``silu(x[:, :I]) * x[:, I:]`` (``llmserve/layers/activation.py:8-11``)."""
import torch
import torch.nn.functional as F

from llmserve_b200.ops._ext import C


def silu_and_mul_ref(x: torch.Tensor) -> torch.Tensor:
    g, u = x.chunk(2, -1)
    return (F.silu(g.float()) * u.float()).to(x.dtype)


def silu_and_mul(x: torch.Tensor) -> torch.Tensor:
    if not x.is_cuda:
        return silu_and_mul_ref(x)
    out = torch.empty(x.shape[0], x.shape[1] // 2, dtype=x.dtype, device=x.device)
    C().silu_and_mul(out, x.contiguous())
    return out
