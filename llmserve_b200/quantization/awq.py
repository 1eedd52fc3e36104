"""AutoAWQ GEMM (W4A16, group 128, zero point) checkpoint format and runtime dispatch.

Format parity with ``llmserve/layers/quantization/awq.py`` of the reference:

* ``qweight`` int32 ``[K, N/8]``: eight 4-bit codes per word; the code of logical column ``8j+i``
  sits at nibble ``AWQ_PACK_ORDER.index(i)`` (AutoAWQ's interleave 0,2,4,6,1,3,5,7; the inverse
  permutation used to unpack is 0,4,1,5,2,6,3,7 -- ``awq.py:8``);
* ``qzeros`` int32 ``[K/128, N/8]`` with the same nibble order;
* ``scales`` bf16 ``[K/128, N]``;  ``w[k, n] = (q[k, n] - z[k/128, n]) * s[k/128, n]``.

The only accepted configuration is quant_method=awq, backend=autoawq, version=gemm, bits=4,
group_size=128, zero_point=True with bf16 activations (``AWQRuntimeConfig.from_hf_config``).
Unlike the reference, tensor parallelism is supported: column-parallel layers slice the packed
output dimension (every shard is a multiple of 8 columns) and row-parallel layers slice K in
whole groups.
"""
from collections.abc import Mapping
from dataclasses import dataclass

import torch
from torch import nn

AWQ_PACK_ORDER = (0, 2, 4, 6, 1, 3, 5, 7)
AWQ_REVERSE_ORDER = (0, 4, 1, 5, 2, 6, 3, 7)


@dataclass(frozen=True)
class AWQRuntimeConfig:
    bits: int
    group_size: int
    zero_point: bool
    version: str
    backend: str
    activation_dtype: torch.dtype
    quant_method: str = "awq"
    execution_backend: str = "reference"

    @property
    def pack_factor(self) -> int:
        return 32 // self.bits

    @classmethod
    def from_hf_config(cls, hf_config) -> "AWQRuntimeConfig":
        raw = getattr(hf_config, "quantization_config", None)
        if not isinstance(raw, Mapping):
            raise ValueError("quantization_config must be an AWQ mapping")
        got = {
            "quant_method": str(raw.get("quant_method", "")).lower(),
            "backend": str(raw.get("backend", "")).lower(),
            "bits": raw.get("bits"),
            "group_size": raw.get("group_size"),
            "version": str(raw.get("version", "")).lower(),
            "zero_point": raw.get("zero_point"),
        }
        want = {"quant_method": "awq", "backend": "autoawq", "bits": 4, "group_size": 128,
                "version": "gemm", "zero_point": True}
        for key, value in want.items():
            if got[key] != value:
                raise ValueError(f"unsupported AWQ {key}: expected {value!r}, got {got[key]!r}")
        dtype = getattr(hf_config, "dtype", None)
        if dtype != torch.bfloat16:
            raise ValueError(f"unsupported AWQ dtype: expected torch.bfloat16, got {dtype!r}")
        return cls(bits=4, group_size=128, zero_point=True, version="gemm", backend="autoawq",
                   activation_dtype=dtype, quant_method="awq")


def pack_awq_int4(codes: torch.Tensor) -> torch.Tensor:
    """Pack int codes ``[R, C]`` (0..15, C % 8 == 0) into AutoAWQ words ``[R, C/8]``."""
    if codes.ndim != 2 or codes.shape[1] % 8:
        raise ValueError("codes must be [R, C] with C divisible by 8")
    c = codes.to(torch.int64).view(codes.shape[0], -1, 8)
    word = torch.zeros(c.shape[:2], dtype=torch.int64, device=codes.device)
    for slot, logical in enumerate(AWQ_PACK_ORDER):
        word |= (c[:, :, logical] & 0xF) << (4 * slot)
    word = torch.where(word >= 2**31, word - 2**32, word)
    return word.to(torch.int32)


def unpack_awq_int4(packed: torch.Tensor) -> torch.Tensor:
    """Inverse of :func:`pack_awq_int4`: ``[R, C/8]`` int32 -> ``[R, C]`` codes in logical order."""
    if packed.ndim != 2 or packed.dtype != torch.int32:
        raise ValueError("packed AWQ tensor must be a two-dimensional int32 tensor")
    shifts = torch.arange(0, 32, 4, dtype=torch.int32, device=packed.device)
    nibbles = (packed.unsqueeze(-1) >> shifts) & 0xF
    order = torch.tensor(AWQ_REVERSE_ORDER, dtype=torch.long, device=packed.device)
    return nibbles[:, :, order].reshape(packed.shape[0], -1)


def validate_awq_tensors(qweight, qzeros, scales, group_size: int):
    if qweight.ndim != 2 or qweight.dtype != torch.int32:
        raise ValueError("qweight must be a two-dimensional int32 tensor")
    if qzeros.ndim != 2 or qzeros.dtype != torch.int32:
        raise ValueError("qzeros must be a two-dimensional int32 tensor")
    if scales.ndim != 2 or not scales.is_floating_point():
        raise ValueError("scales must be a two-dimensional floating tensor")
    if group_size <= 0:
        raise ValueError("group_size must be positive")
    k = qweight.shape[0]
    if k % group_size:
        raise ValueError("qweight input size must be divisible by group_size")
    groups, n = k // group_size, qweight.shape[1] * 8
    if tuple(qzeros.shape) != (groups, qweight.shape[1]):
        raise ValueError("qzeros shape must be [input_size / group_size, output_size / 8]")
    if tuple(scales.shape) != (groups, n):
        raise ValueError("scales shape must be [input_size / group_size, output_size]")
    if len({qweight.device, qzeros.device, scales.device}) != 1:
        raise ValueError("qweight, qzeros, and scales must share one device")


def dequantize_awq_gemm(qweight, qzeros, scales, *, group_size: int) -> torch.Tensor:
    """Dense ``[K, N]`` weight in the scales' dtype."""
    validate_awq_tensors(qweight, qzeros, scales, group_size)
    q = unpack_awq_int4(qweight)
    z = unpack_awq_int4(qzeros).repeat_interleave(group_size, dim=0)
    s = scales.repeat_interleave(group_size, dim=0)
    return (q.to(scales.dtype) - z.to(scales.dtype)) * s


def awq_reference_linear(inputs, qweight, qzeros, scales, *, group_size: int) -> torch.Tensor:
    """Reference W4A16 linear: dequantize then matmul (oracle for the CUDA kernel)."""
    if not inputs.is_floating_point():
        raise ValueError("AWQ activations must use a floating dtype")
    if inputs.dtype != scales.dtype:
        raise ValueError("AWQ activation dtype must match checkpoint scales dtype")
    if inputs.device != qweight.device:
        raise ValueError("AWQ activations and weights must share one device")
    if inputs.shape[-1] != qweight.shape[0]:
        raise ValueError("AWQ activation K must match qweight input size")
    weight = dequantize_awq_gemm(qweight, qzeros, scales, group_size=group_size)
    return torch.matmul(inputs.float(), weight.float()).to(inputs.dtype)


class AWQLinearMethod:
    """Creates the packed parameters of a linear layer and runs it.

    ``process_weights_after_loading`` converts the AutoAWQ tensors into the layout the sm_100a
    W4A16 kernel streams (``llmserve_b200/ops/awq.py``) when the layer lives on CUDA.
    """

    def __init__(self, config: AWQRuntimeConfig):
        self.config = config

    def create_weights(self, layer: nn.Module, input_size: int, output_size: int):
        g, pf = self.config.group_size, self.config.pack_factor
        if input_size % g:
            raise ValueError("AWQ input size must be divisible by group_size")
        if output_size % pf:
            raise ValueError("AWQ output size must be divisible by pack_factor")
        layer.qweight = nn.Parameter(torch.empty(input_size, output_size // pf, dtype=torch.int32),
                                     requires_grad=False)
        layer.qzeros = nn.Parameter(torch.empty(input_size // g, output_size // pf, dtype=torch.int32),
                                    requires_grad=False)
        layer.scales = nn.Parameter(torch.empty(input_size // g, output_size,
                                                dtype=self.config.activation_dtype), requires_grad=False)
        for p in (layer.qweight, layer.qzeros):
            p.output_dim, p.input_dim, p.packed_dim, p.pack_factor = 1, 0, 1, pf
        layer.scales.output_dim, layer.scales.input_dim = 1, 0

    def process_weights_after_loading(self, layer: nn.Module):
        if self.config.execution_backend != "cuda" or layer.qweight.device.type != "cuda":
            return
        from llmserve_b200.ops import awq as awq_ops
        layer.awq_packed = awq_ops.prepare_awq_weights(layer.qweight.data, layer.qzeros.data,
                                                       layer.scales.data, self.config.group_size)

    def apply(self, layer: nn.Module, x: torch.Tensor) -> torch.Tensor:
        packed = getattr(layer, "awq_packed", None)
        if packed is not None:
            from llmserve_b200.ops import awq as awq_ops
            return awq_ops.awq_linear(x, packed)
        if x.is_cuda and self.config.execution_backend == "cuda":
            raise RuntimeError("AWQ CUDA weights must be processed after checkpoint loading")
        return awq_reference_linear(x, layer.qweight, layer.qzeros, layer.scales,
                                    group_size=self.config.group_size)
