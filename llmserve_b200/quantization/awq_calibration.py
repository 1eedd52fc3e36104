"""Activation-aware weight quantisation (AWQ, Lin et al. 2023) to AutoAWQ GEMM W4A16.

Offline, not on a serving path.  Behaviour parity with
``llmserve/quantization/awq_calibration.py`` of the reference (API names and semantics kept:
``quantize_awq_weight`` :35-62, ``fake_quantize_awq_weight`` :65-83, ``search_awq_scale``
:122-190, ``search_awq_clip`` :193-265, ``apply_awq_clip`` :268-282, ``fold_rmsnorm_scale``
:285-302, ``fold_linear_scale`` :305-323).

Method (from the AWQ paper):

* group quantiser -- asymmetric 4-bit round-to-nearest per (output row, group of ``group_size``
  input channels): ``s = max(hi - lo, 1e-5) / 15``, ``z = clamp(-round(lo / s), 0, 15)``,
  ``q = clamp(round(w / s) + z, 0, 15)``, ``w' = (q - z) s``;
* scale search -- per input channel ``s(a) = mean|x|^a / (w_mean^(1-a) + 1e-4)`` (``duo`` form;
  plain ``mean|x|^a`` otherwise), normalised by ``sqrt(max(s) min(s))``, for ``a = i / n_grid``;
  the candidate with the smallest output MSE of ``x W^T`` against ``x (Q(W s) / s)^T`` over all
  linears that share the input wins (``a = 0``'s identity is the starting point);
  ``w_mean`` is the mean over output rows of ``|w|`` normalised by its group's max;
* clip search -- per (output row, group), symmetric clipping at ``max|w| (1 - i / n_grid)``,
  ``i = 1 .. max_shrink n_grid``; the threshold with the smallest mean over tokens of the squared
  error of that group's partial dot product wins (no clipping is the starting point).

Differences from the reference (same method, B200-side choices): every error is evaluated in
fp32 whatever the weights' dtype; the scale search scores all linears of a group with one matmul
of their stacked rows; the clip search contracts the inputs once per candidate with the error
``W - Q(clip(W))`` instead of twice (reference and candidate); both searches subsample tokens at
evenly spaced rows.
"""
from collections.abc import Sequence
from dataclasses import dataclass

import torch
from torch import nn

from llmserve_b200.quantization.awq import pack_awq_int4

QMAX = 15


@dataclass(frozen=True)
class PackedAWQWeight:
    qweight: torch.Tensor   # int32 [in, out / 8]
    qzeros: torch.Tensor    # int32 [in / group, out / 8]
    scales: torch.Tensor    # [in / group, out], the weight's dtype


def _check_grouped(weight: torch.Tensor, group_size: int, what: str):
    if weight.ndim != 2:
        raise ValueError(f"{what} expects a two-dimensional weight tensor")
    if not weight.is_floating_point():
        raise ValueError(f"{what} expects a floating-point weight tensor")
    if group_size <= 0 or weight.shape[1] % group_size:
        raise ValueError("input size must be divisible by a positive group_size")


def _group_params(grouped: torch.Tensor):
    """(scale, zero) of each group along the last dim of an fp32 tensor."""
    lo = grouped.amin(dim=-1, keepdim=True)
    hi = grouped.amax(dim=-1, keepdim=True)
    scale = (hi - lo).clamp(min=1e-5) / QMAX
    zero = torch.round(-lo / scale).clamp(0, QMAX)
    return scale, zero


def _codes(grouped: torch.Tensor, scale: torch.Tensor, zero: torch.Tensor) -> torch.Tensor:
    return (torch.round(grouped / scale) + zero).clamp(0, QMAX)


def _fake_quant_fp32(w: torch.Tensor, group_size: int) -> torch.Tensor:
    """Quantise-dequantise in fp32, any leading shape; groups along the last dim."""
    g = w.reshape(*w.shape[:-1], w.shape[-1] // group_size, group_size)
    scale, zero = _group_params(g)
    return ((_codes(g, scale, zero) - zero) * scale).reshape(w.shape)


def quantize_awq_weight(weight: torch.Tensor, group_size: int = 128) -> PackedAWQWeight:
    """Quantise an ``[out_features, in_features]`` weight into AutoAWQ GEMM tensors."""
    _check_grouped(weight, group_size, "AWQ quantization")
    out_f, in_f = weight.shape
    if out_f % 8:
        raise ValueError("output size must be divisible by 8")
    g = weight.float().reshape(out_f, in_f // group_size, group_size)
    scale, zero = _group_params(g)
    codes = _codes(g, scale, zero).to(torch.int32).reshape(out_f, in_f)
    return PackedAWQWeight(qweight=pack_awq_int4(codes.t().contiguous()),
                           qzeros=pack_awq_int4(zero.squeeze(-1).to(torch.int32).t().contiguous()),
                           scales=scale.squeeze(-1).t().contiguous().to(weight.dtype))


def fake_quantize_awq_weight(weight: torch.Tensor, group_size: int = 128) -> torch.Tensor:
    """The dequantised value of ``weight`` under the group quantiser, in ``weight``'s dtype."""
    _check_grouped(weight, group_size, "AWQ fake quantization")
    return _fake_quant_fp32(weight.float(), group_size).to(weight.dtype)


def _even_rows(x: torch.Tensor, limit: int) -> torch.Tensor:
    flat = x.reshape(-1, x.shape[-1])
    if flat.shape[0] <= limit:
        return flat
    idx = torch.linspace(0, flat.shape[0] - 1, limit, device=flat.device).round().long()
    return flat.index_select(0, idx)


def _group_normalised_mean(w: torch.Tensor, group_size: int) -> torch.Tensor:
    """Mean over output rows of |w| divided by the max |w| of its (row, group)."""
    g = w.float().abs().reshape(w.shape[0], -1, group_size)
    g = g / (g.amax(dim=-1, keepdim=True) + 1e-6)
    return g.reshape(w.shape).mean(dim=0)


@torch.no_grad()
def search_awq_scale(inputs: torch.Tensor, weights: Sequence[torch.Tensor], *, group_size: int = 128,
                     n_grid: int = 20, duo_scaling: bool = True, max_tokens: int = 512) -> torch.Tensor:
    """Per-input-channel AWQ scale for the linears in ``weights`` (all reading ``inputs``)."""
    if inputs.ndim < 2 or not inputs.is_floating_point():
        raise ValueError("inputs must be a floating tensor with a channel dimension")
    if not weights:
        raise ValueError("at least one weight tensor is required")
    if n_grid <= 0 or max_tokens <= 0:
        raise ValueError("n_grid and max_tokens must be positive")
    c = inputs.shape[-1]
    for w in weights:
        if w.ndim != 2 or w.shape[1] != c:
            raise ValueError("all weights must share the input channel dimension")
        if w.device != inputs.device or w.dtype != inputs.dtype:
            raise ValueError("inputs and weights must share device and dtype")
    if c % group_size:
        raise ValueError("input size must be divisible by group_size")

    x = _even_rows(inputs, max_tokens).float()
    w_all = torch.cat([w.float() for w in weights], dim=0)          # one matmul for every linear
    ref = x @ w_all.t()
    x_mean = x.abs().mean(dim=0).clamp(min=1e-4)
    w_mean = torch.stack([_group_normalised_mean(w, group_size) * w.shape[0] for w in weights]).sum(0)
    w_mean = (w_mean / w_all.shape[0]).clamp(min=1e-4)

    def error(scales: torch.Tensor) -> float:
        s = scales.to(inputs.dtype).float()      # the scale is stored in the model's dtype
        wq = _fake_quant_fp32((w_all * s).to(inputs.dtype).float(), group_size) / s
        return float((ref - x @ wq.t()).pow(2).mean())

    ones = torch.ones(c, dtype=torch.float32, device=inputs.device)
    best, best_err = ones, error(ones)
    for i in range(n_grid):
        a = i / n_grid
        s = x_mean.pow(a) / (w_mean.pow(1 - a) + 1e-4) if duo_scaling else x_mean.pow(a)
        s = s.clamp(min=1e-4)
        s = s / torch.sqrt(s.max() * s.min())
        s = torch.where(torch.isfinite(s), s, ones)
        e = error(s)
        if e < best_err:
            best, best_err = s.clone(), e
    return best.to(inputs.dtype)


@torch.no_grad()
def search_awq_clip(weight: torch.Tensor, inputs: torch.Tensor, *, group_size: int = 128, n_grid: int = 20,
                    max_shrink: float = 0.5, max_tokens: int = 512, output_chunk_size: int = 256) -> torch.Tensor:
    """Per (output row, group) clipping threshold ``[out, in / group, 1]`` in ``weight``'s dtype."""
    if weight.ndim != 2 or inputs.ndim < 2:
        raise ValueError("weight and inputs must have channel dimensions")
    if not weight.is_floating_point() or not inputs.is_floating_point():
        raise ValueError("weight and inputs must be floating tensors")
    if weight.shape[1] != inputs.shape[-1]:
        raise ValueError("weight and input channel dimensions must match")
    if weight.device != inputs.device or weight.dtype != inputs.dtype:
        raise ValueError("weight and inputs must share device and dtype")
    if group_size <= 0 or weight.shape[1] % group_size:
        raise ValueError("input size must be divisible by a positive group_size")
    if n_grid <= 0 or max_tokens <= 0 or output_chunk_size <= 0:
        raise ValueError("search sizes must be positive")
    if not 0 <= max_shrink < 1:
        raise ValueError("max_shrink must be in [0, 1)")

    groups = weight.shape[1] // group_size
    x = _even_rows(inputs, max_tokens).float().reshape(-1, groups, group_size)        # [t, g, i]
    steps = max(1, int(max_shrink * n_grid))
    shrink = torch.tensor([1.0] + [1 - i / n_grid for i in range(1, steps + 1)], device=weight.device)
    out = []
    for chunk in weight.split(output_chunk_size, dim=0):
        w = chunk.float().reshape(-1, groups, group_size)                             # [o, g, i]
        wmax = w.abs().amax(dim=-1, keepdim=True)                                      # [o, g, 1]
        best = best_err = None
        for k in range(shrink.numel()):
            lim = wmax * shrink[k]
            # candidates are quantised in the weight's dtype, as the exported model would see them
            cand = torch.maximum(torch.minimum(w, lim), -lim).to(weight.dtype).float()
            diff = w - _fake_quant_fp32(cand, group_size)
            err = torch.einsum("tgi,ogi->otg", x, diff).pow(2).mean(dim=1)            # [o, g]
            if best is None:
                best, best_err = torch.zeros_like(err, dtype=torch.long), err
                continue
            better = err < best_err       # first strictly better candidate in grid order wins
            best = torch.where(better, torch.full_like(best, k), best)
            best_err = torch.where(better, err, best_err)
        out.append(wmax * shrink[best].unsqueeze(-1))
    return torch.cat(out, dim=0).to(weight.dtype)


@torch.no_grad()
def apply_awq_clip(weight: torch.Tensor, max_values: torch.Tensor, *, group_size: int = 128) -> None:
    """Clamp ``weight`` in place to ``[-max, max]`` per (output row, group)."""
    if weight.ndim != 2 or weight.shape[1] % group_size:
        raise ValueError("weight input size must be divisible by group_size")
    want = (weight.shape[0], weight.shape[1] // group_size, 1)
    if tuple(max_values.shape) != want:
        raise ValueError(f"clip values must have shape {want}")
    lim = max_values.to(device=weight.device, dtype=weight.dtype)
    g = weight.view(weight.shape[0], -1, group_size)
    g.copy_(torch.maximum(torch.minimum(g, lim), -lim))


def _scale_inputs_of(linears: Sequence[nn.Module], scales: torch.Tensor, what: str):
    for lin in linears:
        if lin.weight.shape[1] != scales.numel():
            raise ValueError(f"{what} input size and scale size must match")
        lin.weight.mul_(scales.to(device=lin.weight.device, dtype=lin.weight.dtype).view(1, -1))


@torch.no_grad()
def fold_rmsnorm_scale(norm: nn.Module, linears: Sequence[nn.Module], scales: torch.Tensor) -> None:
    """``norm`` output / s, following linears' input columns * s: the network is unchanged."""
    if not hasattr(norm, "weight") or norm.weight.numel() != scales.numel():
        raise ValueError("RMSNorm weight and scale sizes must match")
    for p in (norm.weight, getattr(norm, "bias", None)):
        if p is not None:
            p.div_(scales.to(device=p.device, dtype=p.dtype))
    _scale_inputs_of(linears, scales, "linear")


@torch.no_grad()
def fold_linear_scale(previous: nn.Module, following: Sequence[nn.Module], scales: torch.Tensor) -> None:
    """``previous`` output rows / s, following linears' input columns * s."""
    if previous.weight.shape[0] != scales.numel():
        raise ValueError("previous linear output size and scale size must match")
    s = scales.to(device=previous.weight.device, dtype=previous.weight.dtype)
    previous.weight.div_(s.view(-1, 1))
    if getattr(previous, "bias", None) is not None:
        previous.bias.div_(s)
    _scale_inputs_of(following, scales, "following linear")
