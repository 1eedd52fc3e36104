"""The C entry point ``lsb_decode_attention_noalloc``.

Some callers of this library cannot allocate GPU memory (a host framework that owns all device
allocations, or a plugin handed only pointers and a stream), so they cannot pass the workspace
that ``decode_attention`` takes.  ``lsb_decode_attention_noalloc`` keeps that scratch in a static
device array instead.  These tests call it through its exported C symbol, several times in a row
(the array keeps the previous call's contents), and compare each result with an fp32 PyTorch
gather-and-softmax of the same inputs and with the existing ``decode_attention`` entry point.
The file name sorts last so that a run stopping at the first failure has run everything else.
"""
import ctypes
import math

import pytest
import torch

pytestmark = pytest.mark.gpu

TOL = 1e-2     # relative Frobenius error against fp32, as the other attention kernel tests


def _lib():
    import llmserve_b200._C as ext  # torch is imported first, so libc10 resolves
    lib = ctypes.CDLL(ext.__file__)
    fn = lib.lsb_decode_attention_noalloc
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_void_p] * 4 + [ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p] + [ctypes.c_int] * 6 + \
        [ctypes.c_float, ctypes.c_void_p]
    lib.lsb_noalloc_last_error.restype = ctypes.c_char_p
    return lib, fn


def _case(B, nh, nkv, hd, bs, lens, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    width = max(1, max(-(-L // bs) for L in lens))
    nblk = B * width + 2
    kc = torch.randn(nblk, nkv, bs, hd, device="cuda", generator=g).bfloat16()
    vc = torch.randn(nblk, nkv, bs, hd, device="cuda", generator=g).bfloat16()
    tables = torch.randperm(nblk, device="cuda", generator=g)[: B * width].view(B, width).int().contiguous()
    ctx = torch.tensor(lens, dtype=torch.int32, device="cuda")
    q = torch.randn(B, nh, hd, device="cuda", generator=g).bfloat16()
    return q, kc, vc, tables, ctx


def _fp32_oracle(q, kc, vc, tables, lens, scale):
    """Softmax attention in fp32 over the gathered pages (contexts clamped to the table row, as the
    entry point documents)."""
    from llmserve_b200.ops import attention
    cap = tables.shape[1] * kc.shape[2]
    ctx = torch.tensor([min(L, cap) for L in lens], dtype=torch.int32)
    return attention.decode_attention_ref(q.float().cpu(), kc.float().cpu(), vc.float().cpu(), tables.cpu(), ctx,
                                          scale)


def _rel(a, b):
    a, b = a.float().cpu(), b.float().cpu()
    return ((a - b).norm() / (b.norm() + 1e-12)).item()


def _call(fn, out, q, kc, vc, tables, ctx, scale):
    B, nh, hd = q.shape
    stream = torch.cuda.current_stream().cuda_stream
    return fn(out.data_ptr(), q.data_ptr(), kc.data_ptr(), vc.data_ptr(), tables.data_ptr(), tables.shape[1],
              ctx.data_ptr(), B, nh, kc.shape[1], hd, kc.shape[0], kc.shape[2], scale, stream)


def _run(lib, fn, q, kc, vc, tables, ctx, scale):
    out = torch.full_like(q, float("nan"))
    rc = _call(fn, out, q, kc, vc, tables, ctx, scale)
    assert rc == 0, lib.lsb_noalloc_last_error().decode()
    torch.cuda.synchronize()
    return out


@pytest.mark.parametrize("B,nh,nkv,hd,bs,lens", [
    (7, 32, 8, 128, 256, [1, 5, 64, 300, 513, 1200, 2047]),     # multi-split contexts, short splits
    (64, 32, 8, 128, 256, [384 + 17 * i for i in range(64)]),   # decode-batch shape, long splits
    (3, 4, 2, 64, 16, [33, 200, 129]),
    (4, 8, 2, 128, 64, [0, 70, 0, 1]),                          # empty contexts write zeros
])
def test_no_alloc_decode_matches_fp32_and_existing_entry_point(B, nh, nkv, hd, bs, lens):
    from llmserve_b200.ops import attention
    lib, fn = _lib()
    q, kc, vc, tables, ctx = _case(B, nh, nkv, hd, bs, lens, seed=B)
    scale = 1.0 / math.sqrt(hd)
    oracle = _fp32_oracle(q, kc, vc, tables, lens, scale)
    existing = attention.decode_attention(q, kc, vc, tables, ctx, scale)
    for _ in range(2):
        out = _run(lib, fn, q, kc, vc, tables, ctx, scale)
        assert torch.isfinite(out.float()).all()
        assert _rel(out, oracle) < TOL
        assert _rel(out, existing) < TOL
        for b, L in enumerate(lens):
            if L == 0:
                assert out[b].abs().sum().item() == 0.0


def test_no_alloc_decode_smaller_batch_after_larger_one():
    """The scratch keeps the larger call's partials and counters; the smaller call must not see them."""
    lib, fn = _lib()
    big = _case(48, 32, 8, 128, 256, [1500 + 7 * i for i in range(48)], seed=3)
    small = _case(5, 32, 8, 128, 256, [900, 1, 2500, 256, 257], seed=4)
    scale = 1.0 / math.sqrt(128)
    for q, kc, vc, tables, ctx in (big, small, big, small):
        out = _run(lib, fn, q, kc, vc, tables, ctx, scale)
        assert _rel(out, _fp32_oracle(q, kc, vc, tables, ctx.tolist(), scale)) < TOL


def test_no_alloc_decode_clamps_long_context_and_skips_bad_blocks():
    """A context past the block-table row attends to the row only, and an out-of-range block id
    reads zeros; neither disturbs a correct call that follows."""
    lib, fn = _lib()
    q, kc, vc, tables, ctx = _case(6, 16, 4, 128, 64, [100, 64, 190, 5, 128, 129], seed=5)
    scale = 1.0 / math.sqrt(128)
    good = _fp32_oracle(q, kc, vc, tables, ctx.tolist(), scale)
    long_ctx = ctx.clone()
    long_ctx[2] = 1 << 30                        # far past the 3 x 64 keys of its row
    out = _run(lib, fn, q, kc, vc, tables, long_ctx, scale)
    assert _rel(out, _fp32_oracle(q, kc, vc, tables, long_ctx.tolist(), scale)) < TOL
    bad = tables.clone()
    bad[0, 1] = kc.shape[0] + 5
    bad[4, 0] = -1
    out = _run(lib, fn, q, kc, vc, bad, ctx, scale)
    assert torch.isfinite(out.float()).all()
    for b in (1, 2, 3, 5):                       # rows whose blocks are all valid
        assert _rel(out[b], good[b]) < TOL
    assert _rel(_run(lib, fn, q, kc, vc, tables, ctx, scale), good) < TOL


def test_no_alloc_decode_rejects_oversized_request():
    lib, fn = _lib()
    q, kc, vc, tables, ctx = _case(2, 8, 2, 128, 256, [10, 20], seed=1)
    huge = torch.zeros(2, 1 << 16, dtype=torch.int32, device="cuda")   # 16M keys per sequence
    out = torch.zeros_like(q)
    rc = _call(fn, out, q, kc, vc, huge, ctx, 0.1)
    assert rc == -2
    assert b"LSB_NOALLOC_SCRATCH_BYTES" in lib.lsb_noalloc_last_error()
    assert out.abs().sum().item() == 0.0
