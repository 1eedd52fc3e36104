"""Megatron-style 1-D tensor-parallel linear layers.

Loader semantics follow ``llmserve/layers/linear.py`` of the reference (column-parallel slices the
output dimension, merged/QKV layers place each checkpoint shard at its offset, row-parallel slices
the input dimension; AWQ tensors are sliced along their packed dimension).  The forward passes run
the sm_100a GEMM (``llmserve_b200.ops.gemm``) or the W4A16 kernel.  ``RowParallelLinear`` exposes
``forward_add_norm``, which fuses split-K reduction, the TP all-reduce, the residual add and the
following RMSNorm on the CUDA path.
"""
import os
import torch
from torch import nn

from llmserve_b200.ops import gemm, norm as norm_ops
from llmserve_b200.parallel import state as tp
from llmserve_b200.quantization.awq import AWQLinearMethod, AWQRuntimeConfig


def divide(a: int, b: int) -> int:
    if a % b:
        raise ValueError(f"{a} is not divisible by {b}")
    return a // b


class LinearBase(nn.Module):

    def __init__(self, input_size: int, output_size: int, bias: bool = False, tp_dim: int | None = None,
                 quant_config: AWQRuntimeConfig | None = None):
        super().__init__()
        self.tp_dim = tp_dim
        self.tp_rank = tp.get_tp_rank()
        self.tp_size = tp.get_tp_size()
        self.input_size, self.output_size = input_size, output_size
        self.quant_method = AWQLinearMethod(quant_config) if quant_config else None
        if self.quant_method is None:
            self.weight = nn.Parameter(torch.empty(output_size, input_size), requires_grad=False)
            self.weight.weight_loader = self.weight_loader
        else:
            if bias:
                raise ValueError("AWQ Linear bias is not supported")
            self.quant_method.create_weights(self, input_size, output_size)
            for p in (self.qweight, self.qzeros, self.scales):
                p.weight_loader = self.weight_loader
        if bias:
            self.bias = nn.Parameter(torch.empty(output_size), requires_grad=False)
            self.bias.weight_loader = self.weight_loader
        else:
            self.register_parameter("bias", None)

    packed_weight = None

    @property
    def gemm_weight(self):
        """The operand handed to the GEMM: the AWQ tiles of a quantised layer, the packed tile
        image once ``pack_for_gemm`` ran, else the row-major weight."""
        awq = getattr(self, "awq_packed", None)
        if awq is not None:
            return awq
        return self.packed_weight if self.packed_weight is not None else self.weight

    @property
    def fused_gemm_ok(self) -> bool:
        """Whether the split-K partial paths (QKV reducer, fused add+RMSNorm) apply: a dense
        weight, or AWQ weights repacked for the W4A16 kernel; no bias."""
        return self.bias is None and (self.quant_method is None or getattr(self, "awq_packed", None) is not None)

    def pack_for_gemm(self):
        """After loading: re-store the dense CUDA weight as ``gemm.PackedWeight`` (tile-contiguous,
        pre-swizzled) and release the row-major copy.  The tile image is kept as a buffer so
        memory accounting still sees it."""
        if (os.environ.get("LLMSERVE_PACK_WEIGHTS", "1") == "0" or self.quant_method is not None
                or not self.weight.is_cuda or self.packed_weight is not None):
            return
        pw = gemm.pack_weight(self.weight.data)
        self.register_buffer("weight_tiles", pw.data, persistent=False)
        self.packed_weight = pw
        self.weight.data = torch.empty(0, dtype=self.weight.dtype, device=self.weight.device)

    def apply_linear(self, x: torch.Tensor, bias=True) -> torch.Tensor:
        if self.quant_method is not None:
            return self.quant_method.apply(self, x)
        return gemm.linear(x, self.gemm_weight, self.bias if bias else None)

    @staticmethod
    def _pack_factor(param, dim: int) -> int:
        return getattr(param, "pack_factor", 1) if getattr(param, "packed_dim", None) == dim else 1

    def forward(self, x):  # pragma: no cover - abstract
        raise NotImplementedError


class ReplicatedLinear(LinearBase):

    def __init__(self, input_size, output_size, bias=False, quant_config=None):
        super().__init__(input_size, output_size, bias, quant_config=quant_config)

    def weight_loader(self, param, loaded):
        param.data.copy_(loaded)

    def forward(self, x):
        return self.apply_linear(x)


class ColumnParallelLinear(LinearBase):

    def __init__(self, input_size, output_size, bias=False, quant_config=None):
        super().__init__(input_size, divide(output_size, tp.get_tp_size()), bias, 0, quant_config)

    def weight_loader(self, param, loaded):
        dim = getattr(param, "output_dim", self.tp_dim)
        size = param.data.size(dim)
        param.data.copy_(loaded.narrow(dim, self.tp_rank * size, size))

    def forward(self, x):
        return self.apply_linear(x)


class MergedColumnParallelLinear(ColumnParallelLinear):
    """gate_proj and up_proj stored side by side: [gate shard | up shard] on each rank.

    With ``LLMSERVE_SILU_EPILOGUE=1`` the dense CUDA weight is permuted after loading
    (``interleave_for_silu``) so the GEMM applies SiLU-mul in its epilogue and ``forward_silu``
    returns ``silu(gate) * up`` directly.  It is off by default: on the Qwen3-8B decode step the
    epilogue forces one K split for gate_up (192 CTAs on 148 SMs) and measured about 1% slower
    than split-K GEMM + separate SiLU-mul kernel."""

    interleaved = False

    def interleave_for_silu(self):
        if os.environ.get("LLMSERVE_SILU_EPILOGUE", "0") == "1" \
                and self.quant_method is None and self.weight.is_cuda and len(self.output_sizes) == 2 \
                and self.output_sizes[0] == self.output_sizes[1] and (self.output_sizes[0] // self.tp_size) % 64 == 0:
            self.weight.data = gemm.interleave_gate_up(self.weight.data)
            self.interleaved = True

    def forward_silu(self, x):
        if self.interleaved:
            return gemm.linear_silu(x, self.gemm_weight)
        from llmserve_b200.ops import activation
        return activation.silu_and_mul(self.forward(x))

    def __init__(self, input_size, output_sizes: list[int], bias=False, quant_config=None):
        if quant_config is not None and any(s % quant_config.pack_factor for s in output_sizes):
            raise ValueError("each AWQ output shard must be divisible by pack_factor")
        self.output_sizes = output_sizes
        super().__init__(input_size, sum(output_sizes), bias, quant_config)
        for p in self.parameters(recurse=False):
            p.expected_shard_ids = tuple(range(len(output_sizes)))

    def weight_loader(self, param, loaded, shard_id: int):
        dim = getattr(param, "output_dim", self.tp_dim)
        pf = self._pack_factor(param, dim)
        offset = sum(self.output_sizes[:shard_id]) // self.tp_size // pf
        size = self.output_sizes[shard_id] // self.tp_size // pf
        param.data.narrow(dim, offset, size).copy_(loaded.chunk(self.tp_size, dim)[self.tp_rank])


class QKVParallelLinear(ColumnParallelLinear):
    """q, k and v projections stored as [q heads | k heads | v heads] of this rank."""

    def forward_partials(self, x):
        """On CUDA with split K: the fp32 partials ``[S, T, W]`` (the QK-norm/RoPE kernel reduces
        them); otherwise the projection output."""
        if x.is_cuda and self.fused_gemm_ok:
            x2 = x.reshape(-1, x.shape[-1])
            w = self.gemm_weight
            if gemm.use_cluster(x2.shape[0], w):
                return gemm.linear_reduced(x2.contiguous(), w, plane=True)
            splits = gemm.splits_for(x2.shape[0], w)
            if splits > 1:
                return gemm.linear_partials(x2.contiguous(), w, splits)
        return self.forward(x)

    def __init__(self, hidden_size, head_size, total_num_heads, total_num_kv_heads=None, bias=False,
                 quant_config=None):
        world = tp.get_tp_size()
        total_num_kv_heads = total_num_kv_heads or total_num_heads
        self.head_size = head_size
        self.num_heads = divide(total_num_heads, world)
        self.num_kv_heads = divide(total_num_kv_heads, world)
        if quant_config is not None:
            for s in (total_num_heads * head_size, total_num_kv_heads * head_size):
                if s % quant_config.pack_factor:
                    raise ValueError("each AWQ output shard must be divisible by pack_factor")
        super().__init__(hidden_size, (total_num_heads + 2 * total_num_kv_heads) * head_size, bias,
                         quant_config)
        for p in self.parameters(recurse=False):
            p.expected_shard_ids = ("q", "k", "v")

    def weight_loader(self, param, loaded, shard_id: str):
        if shard_id not in ("q", "k", "v"):
            raise ValueError(shard_id)
        dim = getattr(param, "output_dim", self.tp_dim)
        pf = self._pack_factor(param, dim)
        q, kv = self.num_heads * self.head_size, self.num_kv_heads * self.head_size
        offset, size = {"q": (0, q), "k": (q, kv), "v": (q + kv, kv)}[shard_id]
        param.data.narrow(dim, offset // pf, size // pf).copy_(loaded.chunk(self.tp_size, dim)[self.tp_rank])


class RowParallelLinear(LinearBase):

    def __init__(self, input_size, output_size, bias=False, quant_config=None):
        super().__init__(divide(input_size, tp.get_tp_size()), output_size, bias, 1, quant_config)

    def weight_loader(self, param, loaded):
        if param.data.ndim == 1:
            param.data.copy_(loaded)
            return
        dim = getattr(param, "input_dim", self.tp_dim)
        size = param.data.size(dim)
        param.data.copy_(loaded.narrow(dim, self.tp_rank * size, size))

    def forward(self, x):
        y = self.apply_linear(x, bias=self.tp_rank == 0)
        return tp.all_reduce(y)

    def forward_add_norm(self, x: torch.Tensor, residual: torch.Tensor, norm_weight: torch.Tensor, eps: float):
        """``(rmsnorm(allreduce(x @ W^T) + residual) * w, allreduce(..) + residual)``."""
        if x.is_cuda and self.fused_gemm_ok:
            from llmserve_b200.parallel import fused as fused_ops
            return fused_ops.row_parallel_add_norm(x, self.gemm_weight, residual, norm_weight, eps,
                                                   tp.get_fused_comm())
        y = self.forward(x)
        return norm_ops.add_rms_norm(y, residual, norm_weight, eps)
