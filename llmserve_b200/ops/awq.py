"""W4A16 linear for AutoAWQ GEMM checkpoints (4-bit, group 128, zero point) on sm_100a.

Load time (``prepare_awq_weights``, the counterpart of the reference's qweight repack and qzeros
reorder kernels, ``llmserve/quantization/csrc/awq_w4a16.cu:81-118``): the AutoAWQ tensors
``qweight [K, N/8]``, ``qzeros [K/128, N/8]`` and ``scales [K/128, N]`` are rewritten into

* ``qtiles`` int32 ``[ceil(N/128), K/64, 128, 8]``: for every 128-feature x 64-K tile, each
  feature's 64 codes as 8 words; word ``c`` holds K elements ``8c..8c+7`` with element ``2i`` in
  bits ``4i..4i+3`` and element ``2i+1`` in bits ``16+4i..``, so ``(word >> 4i) & 0x000F000F``
  selects one bf16 pair of codes;
* ``sztiles`` int32 ``[ceil(N/128), K/128, 128, 2]``: per feature and group, the bf16 pairs
  ``(s, s)`` and ``(128 + z, 128 + z)``.

Run time (``awq_linear``): the tcgen05 kernel copies 4 KiB code tiles + 1 KiB scale tiles per
step, dequantises to a bf16 operand tile in shared memory (``(128+q) - (128+z)`` is exact in
bf16, times ``s`` rounds once) and accumulates in TMEM; split-K partials are summed by the
reduction kernel.  Replaces the reference's ``awq_w4a16_kernel`` (``mma.sync``) and its Triton
GEMV/GEMM (``awq_triton.py``).
"""
import os
from dataclasses import dataclass

import torch

from llmserve_b200.ops._ext import C, status
from llmserve_b200.quantization.awq import unpack_awq_int4, validate_awq_tensors

TILE_N = 128
TILE_K = 64
NUM_SMS = 148
_SHIFTS = (0, 16, 4, 20, 8, 24, 12, 28)   # bit position of K element j (0..7) inside a word


@dataclass
class AWQPacked:
    qtiles: torch.Tensor
    sztiles: torch.Tensor
    n: int
    k: int

    @property
    def shape(self):
        return (self.n, self.k)


def _wrap_int32(v: torch.Tensor) -> torch.Tensor:
    return torch.where(v >= 2**31, v - 2**32, v).to(torch.int32)


def prepare_awq_weights(qweight: torch.Tensor, qzeros: torch.Tensor, scales: torch.Tensor,
                        group_size: int) -> AWQPacked:
    validate_awq_tensors(qweight, qzeros, scales, group_size)
    if group_size != 128:
        raise ValueError("the W4A16 kernel supports group_size 128 only")
    K, N = qweight.shape[0], qweight.shape[1] * 8
    G = K // group_size
    mt = -(-N // TILE_N)
    npad = mt * TILE_N
    dev = qweight.device
    codes = torch.zeros(npad, K, dtype=torch.int64, device=dev)
    codes[:N] = unpack_awq_int4(qweight).t().to(torch.int64)
    tiles = codes.view(mt, TILE_N, K // TILE_K, 8, 8).permute(0, 2, 1, 3, 4)     # [mt, kt, 128, word, j]
    shifts = torch.tensor(_SHIFTS, dtype=torch.int64, device=dev)
    words = (tiles << shifts).sum(-1)
    qtiles = _wrap_int32(words).contiguous()

    zeros = torch.zeros(npad, G, dtype=torch.int64, device=dev)
    zeros[:N] = unpack_awq_int4(qzeros).t().to(torch.int64)
    sc = torch.zeros(npad, G, dtype=torch.bfloat16, device=dev)
    sc[:N] = scales.t().to(torch.bfloat16)
    s_bits = sc.view(torch.int16).to(torch.int64) & 0xFFFF
    z_bits = 0x4300 | zeros
    sz = torch.stack([s_bits | (s_bits << 16), z_bits | (z_bits << 16)], -1)     # [npad, G, 2]
    sztiles = _wrap_int32(sz.view(mt, TILE_N, G, 2).permute(0, 2, 1, 3)).contiguous()
    return AWQPacked(qtiles, sztiles, N, K)


# CTAs per SM of the W4A16 kernel: 2 (two operand buffers, default) or 3 (LLMSERVE_AWQ_WBUF=1:
# one operand buffer and a shorter ring, for more CTAs in flight)
AWQ_CTAS_PER_SM = 3 if os.environ.get("LLMSERVE_AWQ_WBUF", "2") == "1" else 2
# decode-sized W4A16 products reduce their K splits in a thread-block cluster (LLMSERVE_AWQ_CLUSTER=0:
# fp32 partial planes + the reduction kernel)
AWQ_CLUSTER = os.environ.get("LLMSERVE_AWQ_CLUSTER", "1") != "0"


def choose_awq_splits(T: int, n: int, k: int) -> int:
    """Split K so the grid fills the CTA slots of every SM about once; >= 8 K steps per split."""
    bn = 16 if T <= 16 else 32 if T <= 32 else 64 if T <= 64 else 128 if T <= 128 else 256
    tiles = (-(-n // TILE_N)) * (-(-T // bn))
    k_tiles = k // TILE_K
    slots = AWQ_CTAS_PER_SM * NUM_SMS
    if tiles >= slots:
        return 1
    return max(1, min(slots // tiles, k_tiles // 8, 16))


def awq_linear(x: torch.Tensor, packed: AWQPacked) -> torch.Tensor:
    x2 = x.reshape(-1, x.shape[-1]).contiguous()
    T = x2.shape[0]
    out = torch.empty(T, packed.n, dtype=x.dtype, device=x.device)
    if T == 0:
        return out.view(*x.shape[:-1], packed.n)
    splits = choose_awq_splits(T, packed.n, packed.k)
    empty32 = torch.empty(0, dtype=torch.float32, device=x.device)
    if AWQ_CLUSTER and splits > 1 and T <= 128:
        # the K splits of a tile reduce in a thread-block cluster: bf16 out, no partial planes
        C().awq_gemm_reduced(out, x2, packed.qtiles, packed.sztiles, packed.n, min(splits, 8), status(x.device))
        return out.view(*x.shape[:-1], packed.n)
    if splits == 1:
        C().awq_gemm(out, x2, packed.qtiles, packed.sztiles, packed.n, empty32, 1, status(x.device))
    else:
        partials = torch.empty(splits, T, packed.n, dtype=torch.float32, device=x.device)
        C().awq_gemm(torch.empty(0, dtype=x.dtype, device=x.device), x2, packed.qtiles, packed.sztiles, packed.n,
                     partials, splits, status(x.device))
        C().splitk_reduce(out, partials)
    return out.view(*x.shape[:-1], packed.n)


def dequantize_packed(packed: AWQPacked) -> torch.Tensor:
    """Dense ``[N, K]`` bf16 weight rebuilt from the packed tiles (CPU oracle of the kernel's
    dequantisation, used by the tests)."""
    mt, kt = packed.qtiles.shape[0], packed.qtiles.shape[1]
    w = packed.qtiles.to(torch.int64) & 0xFFFFFFFF
    shifts = torch.tensor(_SHIFTS, dtype=torch.int64, device=w.device)
    codes = (w.unsqueeze(-1) >> shifts) & 0xF                                    # [mt, kt, 128, 8, 8]
    codes = codes.permute(0, 2, 1, 3, 4).reshape(mt * TILE_N, kt * TILE_K)
    sz = packed.sztiles.to(torch.int64) & 0xFFFFFFFF                             # [mt, G, 128, 2]
    s_bits = (sz[..., 0] & 0xFFFF).permute(0, 2, 1).reshape(mt * TILE_N, -1)
    s_bits = torch.where(s_bits >= 2**15, s_bits - 2**16, s_bits).to(torch.int16)
    scale = s_bits.view(torch.bfloat16)
    zero = ((sz[..., 1] & 0xFFFF) - 0x4300).permute(0, 2, 1).reshape(mt * TILE_N, -1)
    scale = scale.repeat_interleave(128, dim=1)[:, : packed.k]
    zero = zero.repeat_interleave(128, dim=1)[:, : packed.k]
    deq = ((codes - zero).to(torch.bfloat16) * scale)
    return deq[: packed.n].contiguous()
