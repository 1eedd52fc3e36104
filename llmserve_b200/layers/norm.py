import torch
from torch import nn

from llmserve_b200.ops import norm as norm_ops


class RMSNorm(nn.Module):
    """RMSNorm module; ``forward(x, residual)`` is the fused residual-add form
    (``llmserve/layers/layernorm.py`` of the reference)."""

    def __init__(self, hidden_size: int, eps: float = 1e-6):
        super().__init__()
        self.eps = eps
        self.weight = nn.Parameter(torch.ones(hidden_size), requires_grad=False)

    def forward(self, x, residual=None):
        if residual is None:
            return norm_ops.rms_norm(x, self.weight, self.eps)
        return norm_ops.add_rms_norm(x, residual, self.weight, self.eps)
