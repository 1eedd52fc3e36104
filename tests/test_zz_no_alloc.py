"""The C entry point ``lsb_decode_attention_noalloc`` against the existing decode entry point.

Some callers of this library cannot allocate GPU memory (a host framework that owns all device
allocations, or a plugin handed only pointers and a stream), so they cannot pass the workspace
that ``decode_attention`` takes.  ``lsb_decode_attention_noalloc`` keeps that scratch in a static
device array instead.  This test calls it through its exported C symbol, twice in a row (the
array keeps the previous call's contents), and compares each result with ``decode_attention``.
The file name sorts last so that a run stopping at the first failure has run everything else.
"""
import ctypes
import math

import pytest
import torch

pytestmark = pytest.mark.gpu


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
    width = max(-(-L // bs) for L in lens)
    nblk = B * width + 2
    kc = torch.randn(nblk, nkv, bs, hd, device="cuda", generator=g).bfloat16()
    vc = torch.randn(nblk, nkv, bs, hd, device="cuda", generator=g).bfloat16()
    tables = torch.randperm(nblk, device="cuda", generator=g)[: B * width].view(B, width).int().contiguous()
    ctx = torch.tensor(lens, dtype=torch.int32, device="cuda")
    q = torch.randn(B, nh, hd, device="cuda", generator=g).bfloat16()
    return q, kc, vc, tables, ctx


def _call(fn, out, q, kc, vc, tables, ctx, scale):
    B, nh, hd = q.shape
    stream = torch.cuda.current_stream().cuda_stream
    return fn(out.data_ptr(), q.data_ptr(), kc.data_ptr(), vc.data_ptr(), tables.data_ptr(), tables.shape[1],
              ctx.data_ptr(), B, nh, kc.shape[1], hd, kc.shape[0], kc.shape[2], scale, stream)


@pytest.mark.parametrize("B,nh,nkv,hd,bs,lens", [
    (7, 32, 8, 128, 256, [1, 5, 64, 300, 513, 1200, 2047]),     # multi-split contexts, short splits
    (64, 32, 8, 128, 256, [384 + 17 * i for i in range(64)]),   # decode-batch shape, long splits
    (3, 4, 2, 64, 16, [33, 200, 129]),
])
def test_no_alloc_decode_matches_existing_entry_point(B, nh, nkv, hd, bs, lens):
    from llmserve_b200.ops import attention
    lib, fn = _lib()
    q, kc, vc, tables, ctx = _case(B, nh, nkv, hd, bs, lens, seed=B)
    scale = 1.0 / math.sqrt(hd)
    ref = attention.decode_attention(q, kc, vc, tables, ctx, scale)
    for _ in range(2):
        out = torch.full_like(q, float("nan"))
        rc = _call(fn, out, q, kc, vc, tables, ctx, scale)
        assert rc == 0, lib.lsb_noalloc_last_error().decode()
        torch.cuda.synchronize()
        err = ((out.float() - ref.float()).norm() / ref.float().norm()).item()
        assert err < 1e-2, err


def test_no_alloc_decode_rejects_oversized_request():
    lib, fn = _lib()
    q, kc, vc, tables, ctx = _case(2, 8, 2, 128, 256, [10, 20], seed=1)
    huge = torch.zeros(2, 1 << 16, dtype=torch.int32, device="cuda")   # 16M keys per sequence
    out = torch.zeros_like(q)
    rc = _call(fn, out, q, kc, vc, huge, ctx, 0.1)
    assert rc == -2
    assert b"LSB_NOALLOC_SCRATCH_BYTES" in lib.lsb_noalloc_last_error()
    assert out.abs().sum().item() == 0.0
