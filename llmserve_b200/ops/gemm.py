"""Dense bf16 linear layers on the sm_100a tensor cores (tcgen05 + TMEM, operands by TMA).

``y[T, N] = x[T, K] @ w[N, K]^T``.  The kernel computes the transposed product: weight rows are
the UMMA M dimension (128 per tile) and tokens are the N dimension (16..256), so a decode batch
of a few dozen tokens still fills a 128-row tensor-core tile and the weight stream -- which sets
decode speed -- is read exactly once.  When there are fewer output tiles than SMs, K is split
across CTAs; the fp32 partials are then reduced by a kernel that also applies the layer's
post-op (plain store, residual add + RMSNorm, or the tensor-parallel all-reduce in
``llmserve_b200.parallel.fused``).  The reference runs these through cuBLAS
(``F.linear`` in ``llmserve/layers/linear.py:57``).
"""
import functools
import os

import torch
import torch.nn.functional as F

from llmserve_b200.ops._ext import C, status

NUM_SMS = 148
TILE_M = 128          # weight rows per CTA
TILE_K = 64           # K elements per pipeline stage (128 B rows -> 128B swizzle)
MAX_TILE_T = 256      # tokens per CTA (UMMA N limit)


SMALL_T = 64          # up to here the 4-stage ring is used, two CTAs per SM


def choose_splits(T: int, N: int, K: int) -> int:
    """Split K so the grid fills the CTA slots about once (weights are streamed once either way).

    Decode-sized token tiles (T <= 64) run two CTAs per SM (296 slots) with >= 8 K tiles each;
    larger tiles run one CTA per SM.  (Chosen from a per-shape sweep on B200.)"""
    tiles = (-(-N // TILE_M)) * (-(-T // MAX_TILE_T))
    k_tiles = -(-K // TILE_K)
    slots, min_kt = (2 * NUM_SMS, 8) if T <= SMALL_T else (int(NUM_SMS * 1.25), 4)
    splits = 1
    while tiles * splits * 2 <= slots and k_tiles // (splits * 2) >= min_kt:
        splits *= 2
    return splits


def _stages(T: int) -> int:
    return 4 if T <= SMALL_T else 0


def stages_for_tokens(T: int) -> int:
    """Pipeline depth the tile GEMM uses for T tokens (4: shallow ring, two CTAs per SM; 0: deepest)."""
    return _stages(T)


class PackedWeight:
    """A weight ``[N, K]`` stored as 128 x 64 tiles in tile order ``(row tile, k tile)``, each tile
    the exact 16 KiB image the GEMM keeps in shared memory (128-byte rows, 16-byte chunks XOR-
    swizzled by row).  A K-range of one row tile is then one contiguous run of HBM, which the
    decode GEMM streams with sequential DRAM pages instead of 128-byte pieces of 128 rows.
    Rows are zero-padded to a multiple of 256 (the 2-SM tile) and K to a multiple of 64."""

    def __init__(self, data: torch.Tensor, n: int, k: int):
        self.data, self.n, self.k = data, n, k

    @property
    def shape(self):
        return (self.n, self.k)

    @property
    def device(self):
        return self.data.device

    @property
    def dtype(self):
        return self.data.dtype

    def unpack(self) -> torch.Tensor:
        return unpack_weight(self)


def _swizzle_index(device):
    r = torch.arange(TILE_M, device=device).view(TILE_M, 1)
    p = torch.arange(8, device=device).view(1, 8)
    return p ^ (r & 7)           # physical chunk p of row r holds logical chunk p ^ (r & 7)


def pack_weight(w: torch.Tensor) -> PackedWeight:
    N, K = w.shape
    Np, Kp = -(-N // 256) * 256, -(-K // TILE_K) * TILE_K
    if (Np, Kp) != (N, K):
        wp = torch.zeros(Np, Kp, dtype=w.dtype, device=w.device)
        wp[:N, :K] = w
    else:
        wp = w
    mt, kt = Np // TILE_M, Kp // TILE_K
    tiles = wp.view(mt, TILE_M, kt, 8, 8).permute(0, 2, 1, 3, 4)          # [mt, kt, 128, chunk, 8]
    idx = _swizzle_index(w.device).view(1, 1, TILE_M, 8, 1).expand(mt, kt, TILE_M, 8, 8)
    packed = torch.gather(tiles, 3, idx).contiguous().view(-1, TILE_K)
    return PackedWeight(packed, N, K)


def unpack_weight(pw: PackedWeight) -> torch.Tensor:
    Np, Kp = -(-pw.n // 256) * 256, -(-pw.k // TILE_K) * TILE_K
    mt, kt = Np // TILE_M, Kp // TILE_K
    tiles = pw.data.view(mt, kt, TILE_M, 8, 8)
    idx = _swizzle_index(pw.device).view(1, 1, TILE_M, 8, 1).expand(mt, kt, TILE_M, 8, 8)
    logical = torch.gather(tiles, 3, idx)                                  # XOR swizzle is its own inverse
    return logical.permute(0, 2, 1, 3, 4).reshape(Np, Kp)[: pw.n, : pw.k].contiguous()


def linear_ref(x: torch.Tensor, w, bias: torch.Tensor | None = None) -> torch.Tensor:
    if isinstance(w, PackedWeight):
        w = w.unpack()
    return F.linear(x, w, bias)


@functools.lru_cache(maxsize=None)
def _num_sms_cached(index: int) -> int:
    return torch.cuda.get_device_properties(index).multi_processor_count


def _num_sms(device) -> int:
    return _num_sms_cached(device.index if device.index is not None else torch.cuda.current_device())


def splits_for(T: int, w) -> int:
    """Partial planes of a [T, K] x W^T product: the K split count.  AWQ splits are rounded down
    to a power of two, at most 8."""
    from llmserve_b200.ops import awq as awq_ops
    if isinstance(w, awq_ops.AWQPacked):
        s = min(awq_ops.choose_awq_splits(T, w.n, w.k), 8)
        return 1 << (s.bit_length() - 1)
    return choose_splits(T, w.shape[0], w.shape[1])


def _gemm(out, x, w, partials, splits, T):
    from llmserve_b200.ops import awq as awq_ops
    if isinstance(w, awq_ops.AWQPacked):
        C().awq_gemm(out, x, w.qtiles, w.sztiles, w.n, partials, splits, status(x.device))
        return
    if isinstance(w, PackedWeight):
        C().gemm_bf16_packed(out, x, w.data, w.n, partials, splits, status(x.device), _stages(T))
    else:
        C().gemm_bf16(out, x, w, partials, splits, status(x.device), _stages(T))


_EMPTY = {}


def _empty(device, dtype):
    key = (device, dtype)
    if key not in _EMPTY:
        _EMPTY[key] = torch.empty(0, device=device, dtype=dtype)
    return _EMPTY[key]


# ---- K splits reduced on chip (thread-block cluster + distributed shared memory) -------------
# With the cluster reduction a K split costs no HBM traffic for partial planes and no reduction
# kernel, so K is split for parallelism alone.  The split count (a power of two, at least two K
# tiles per CTA) minimises waves x (K tiles per CTA + a fixed per-CTA cost), where a wave is every
# CTA slot of the GPU (two per SM with the shallow ring of decode-sized T).  Fitted to a per-shape
# sweep of the Qwen3-8B projections at TP 1/2/8 inside CUDA graphs on B200, where it beat the
# split-K-planes + reduction kernel path on every projection but the 192-tile gate_up (a tie).
CLUSTER_SPLITK = os.environ.get("LLMSERVE_CLUSTER_SPLITK", "1") != "0"
CLUSTER_MAX_SPLITS = 16
CLUSTER_FIXED_KTILES = float(os.environ.get("LLMSERVE_SPLIT_FIXED_KTILES", "8"))
CLUSTER_MAX_T = int(os.environ.get("LLMSERVE_CLUSTER_MAX_T", "511"))   # from 512 tokens the persistent 2-SM kernel takes over
# split counts considered: powers of two (default), or every count up to 16 (LLMSERVE_CLUSTER_ANY_SPLITS=1).
# The latter fills the CTA slots more evenly on paper (48 qkv tiles x 6 = 288 of 296 slots) but measured
# slower on a B200 (Qwen3-8B decode step at C = 64: 5.85-5.90 ms against 4.48-4.53 ms), so it stays off.
CLUSTER_ANY_SPLITS = os.environ.get("LLMSERVE_CLUSTER_ANY_SPLITS", "0") == "1"


@functools.lru_cache(maxsize=None)
def cluster_splits(T: int, N: int, K: int, num_sms: int = NUM_SMS) -> int:
    tiles = (-(-N // TILE_M)) * (-(-T // MAX_TILE_T))
    k_tiles = -(-K // TILE_K)
    slots = num_sms * (2 if T <= SMALL_T else 1)
    best, best_cost = 1, float("inf")
    candidates = range(1, CLUSTER_MAX_SPLITS + 1) if CLUSTER_ANY_SPLITS else \
        [1 << i for i in range(CLUSTER_MAX_SPLITS.bit_length()) if (1 << i) <= CLUSTER_MAX_SPLITS]
    for s in candidates:
        per = -(-k_tiles // s)
        if s > 1 and (per < 2 or (s - 1) * per >= k_tiles):   # >= 2 K tiles each, no empty split
            continue
        cost = (-(-tiles * s // slots)) * (per + CLUSTER_FIXED_KTILES)
        if cost < best_cost - 1e-9:
            best, best_cost = s, cost
    return best


def _dense(w) -> bool:
    from llmserve_b200.ops import awq as awq_ops
    return not isinstance(w, awq_ops.AWQPacked)


def use_cluster(T: int, w) -> bool:
    return CLUSTER_SPLITK and 0 < T <= CLUSTER_MAX_T and _dense(w) and w.device.type == "cuda"


def _operand(w):
    """(tensor, logical rows, packed) for the C entry points."""
    if isinstance(w, PackedWeight):
        return w.data, w.n, True
    return w, w.shape[0], False


def linear_reduced(x2: torch.Tensor, w, out: torch.Tensor | None = None, plane: bool = False):
    """``x2 @ w^T`` with K split over a cluster: bf16 ``[T, N]``, or (``plane``) one fp32 plane
    ``[1, T, N]`` -- the layout the split-K consumers (QK-norm/RoPE, add+RMSNorm) read."""
    T, _ = x2.shape
    data, n, packed = _operand(w)
    splits = cluster_splits(T, n, x2.shape[1], _num_sms(x2.device))
    if plane:
        res = torch.empty(1, T, n, dtype=torch.float32, device=x2.device)
        C().gemm_bf16_reduced(_empty(x2.device, x2.dtype), x2, data, n, packed, res, splits, status(x2.device),
                              _stages(T))
        return res
    res = out if out is not None else torch.empty(T, n, dtype=x2.dtype, device=x2.device)
    C().gemm_bf16_reduced(res, x2, data, n, packed, _empty(x2.device, torch.float32), splits, status(x2.device),
                          _stages(T))
    return res


def linear(x: torch.Tensor, w: torch.Tensor, bias: torch.Tensor | None = None) -> torch.Tensor:
    if not x.is_cuda:
        return linear_ref(x, w, bias)
    x2 = x.reshape(-1, x.shape[-1]).contiguous()
    T, K = x2.shape
    N = w.shape[0]
    out = torch.empty(T, N, dtype=x.dtype, device=x.device)
    if T == 0:
        return out.view(*x.shape[:-1], N)
    if use_cluster(T, w):
        linear_reduced(x2, w, out)
        if bias is not None:
            out += bias
        return out.view(*x.shape[:-1], N)
    splits = splits_for(T, w)
    if splits == 1:
        _gemm(out, x2, w, _empty(x.device, torch.float32), 1, T)
    else:
        partials = torch.empty(splits, T, N, dtype=torch.float32, device=x.device)
        _gemm(_empty(x.device, x.dtype), x2, w, partials, splits, T)
        C().splitk_reduce(out, partials)
    if bias is not None:
        out += bias
    return out.view(*x.shape[:-1], N)


def linear_partials(x: torch.Tensor, w: torch.Tensor, splits: int, partials: torch.Tensor | None = None):
    """fp32 partial planes ``[splits, T, N]`` (not reduced) whose sum is ``x @ w^T``; ``splits``
    comes from :func:`splits_for`."""
    T, K = x.shape
    N = w.shape[0]
    if partials is None:
        partials = torch.empty(splits, T, N, dtype=torch.float32, device=x.device)
    _gemm(_empty(x.device, x.dtype), x.contiguous(), w, partials, splits, T)
    return partials


def interleave_gate_up(w: torch.Tensor) -> torch.Tensor:
    """[gate (I rows) ; up (I rows)] -> rows interleaved per 64: g0..g63, u0..u63, g64.., so every
    128-row tile of the GEMM holds matching gate and up rows (I % 64 == 0)."""
    I = w.shape[0] // 2
    g, u = w[:I].view(I // 64, 64, -1), w[I:].view(I // 64, 64, -1)
    return torch.stack([g, u], dim=1).reshape(2 * I, -1).contiguous()


SILU_EPILOGUE_MAX_T = 128     # above this the projection runs on the 2-SM kernel and SiLU-mul separately


def linear_silu(x: torch.Tensor, w_interleaved: torch.Tensor, max_splits: int = 8) -> torch.Tensor:
    """``silu(x @ gate^T) * (x @ up^T)`` for an interleaved gate/up weight, fused in the GEMM
    epilogue (or in the split-K reduction when K is split)."""
    x2 = x.reshape(-1, x.shape[-1]).contiguous()
    T, K = x2.shape
    N = w_interleaved.shape[0]
    out = torch.empty(T, N // 2, dtype=x.dtype, device=x.device)
    if T == 0:
        return out
    if T > SILU_EPILOGUE_MAX_T:
        # prefill-sized: the 2-SM GEMM writes the interleaved projection, then one SiLU-mul pass
        y = linear(x2, w_interleaved)
        C().silu_and_mul_interleaved(out, y)
        return out
    if use_cluster(T, w_interleaved) and max_splits > 1:
        data, n, packed = _operand(w_interleaved)
        C().gemm_bf16_silu_reduced(out, x2, data, n, packed, cluster_splits(T, n, K, _num_sms(x2.device)),
                                   status(x.device), _stages(T))
        return out
    splits = min(choose_splits(T, N, K), max_splits)
    if splits == 1 and isinstance(w_interleaved, PackedWeight):
        C().gemm_bf16_silu_packed(out, x2, w_interleaved.data, w_interleaved.n, status(x.device), _stages(T))
    elif splits == 1:
        C().gemm_bf16_silu(out, x2, w_interleaved, status(x.device), _stages(T))
    else:
        partials = linear_partials(x2, w_interleaved, splits)
        C().splitk_silu(out, partials)
    return out
