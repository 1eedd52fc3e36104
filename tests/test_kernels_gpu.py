"""sm_100a kernels against fp32 PyTorch references of the same ops (small shapes)."""
import math

import pytest
import torch

pytestmark = pytest.mark.gpu

from llmserve_b200.ops import activation, attention, gemm, kv, norm, rope, sampling  # noqa: E402
from llmserve_b200.ops._ext import C, check_status, status  # noqa: E402

DEV = "cuda"


def rel_err(a, b):
    a, b = a.float(), b.float()
    return ((a - b).norm() / (b.norm() + 1e-12)).item()


@pytest.fixture(autouse=True)
def _status():
    C()
    yield
    check_status(torch.device(DEV))


@pytest.mark.parametrize("T", [1, 7, 16, 33, 64, 100, 256, 300])
@pytest.mark.parametrize("N,K", [(128, 64), (384, 256), (1000, 512), (256, 4096)])
def test_gemm_matches_fp32(T, N, K):
    g = torch.Generator(device=DEV).manual_seed(T * 7 + N + K)
    x = torch.randn(T, K, device=DEV, generator=g).bfloat16()
    w = (torch.randn(N, K, device=DEV, generator=g) * 0.05).bfloat16()
    ref = x.float() @ w.float().t()
    out = gemm.linear(x, w)
    torch.cuda.synchronize()
    assert rel_err(out, ref) < 1e-2


@pytest.mark.parametrize("T,N,K", [(512, 256, 64), (777, 1000, 520), (1024, 6144, 4096), (2304, 4104, 1024),
                                   (4096, 24576, 256)])
def test_pair_gemm_matches_fp32(T, N, K):
    """Prefill-sized token counts run the persistent 2-SM (cta_group::2) kernel: ragged T and N,
    K not a multiple of the 64-wide stage, several tiles per cluster."""
    g = torch.Generator(device=DEV).manual_seed(T + N + K)
    x = torch.randn(T, K, device=DEV, generator=g).bfloat16()
    w = (torch.randn(N, K, device=DEV, generator=g) * 0.05).bfloat16()
    ref = x.float() @ w.float().t()
    out = gemm.linear(x, w)
    parts = gemm.linear_partials(x, w, 1)         # fp32 output variant
    torch.cuda.synchronize()
    assert rel_err(out, ref) < 1e-2
    assert rel_err(parts[0], ref) < 1e-4
    assert torch.isfinite(parts).all()


@pytest.mark.parametrize("T", [1, 17, 64, 300, 1024])
@pytest.mark.parametrize("N,K", [(4096, 4096), (1000, 520), (6144, 1024)])
def test_packed_gemm_matches_fp32(T, N, K):
    """Tile-packed weights (decode kernel for small T, 2-SM kernel for large T, split-K partials)."""
    g = torch.Generator(device=DEV).manual_seed(T + N + K + 1)
    x = torch.randn(T, K, device=DEV, generator=g).bfloat16()
    w = (torch.randn(N, K, device=DEV, generator=g) * 0.05).bfloat16()
    pw = gemm.pack_weight(w)
    assert torch.equal(pw.unpack(), w)
    ref = x.float() @ w.float().t()
    out = gemm.linear(x, pw)
    parts = gemm.linear_partials(x, pw, 2 if K >= 1024 else 1)
    torch.cuda.synchronize()
    assert rel_err(out, ref) < 1e-2
    assert rel_err(parts.sum(0), ref) < 1e-4


@pytest.mark.parametrize("splits", [2, 4, 8])
def test_gemm_split_k_partials_sum(splits):
    x = torch.randn(48, 2048, device=DEV).bfloat16()
    w = (torch.randn(512, 2048, device=DEV) * 0.05).bfloat16()
    parts = gemm.linear_partials(x, w, splits)
    ref = x.float() @ w.float().t()
    assert rel_err(parts.sum(0), ref) < 1e-3


@pytest.mark.parametrize("H", [256, 4096, 8192])
def test_rms_norm_and_add(H):
    x = torch.randn(37, H, device=DEV).bfloat16()
    r = torch.randn(37, H, device=DEV).bfloat16()
    w = (1 + 0.1 * torch.randn(H, device=DEV)).bfloat16()
    assert rel_err(norm.rms_norm(x, w, 1e-6), norm.rms_norm_ref(x.cpu(), w.cpu(), 1e-6).to(DEV)) < 5e-3
    o, res = norm.add_rms_norm(x, r, w, 1e-6)
    ro, rres = norm.add_rms_norm_ref(x.cpu(), r.cpu(), w.cpu(), 1e-6)
    assert rel_err(o, ro.to(DEV)) < 5e-3
    assert rel_err(res, rres.to(DEV)) < 5e-3


@pytest.mark.parametrize("N", [512, 4096, 8192])
def test_splitk_reduce_add_rmsnorm(N):
    parts = torch.randn(4, 9, N, device=DEV)
    r = torch.randn(9, N, device=DEV).bfloat16()
    w = torch.ones(N, device=DEV).bfloat16()
    out = torch.empty(9, N, device=DEV, dtype=torch.bfloat16)
    res = torch.empty_like(out)
    C().splitk_reduce_add_rmsnorm(out, res, parts, r, w, 1e-6)
    ro, rres = norm.add_rms_norm_ref(parts.sum(0).bfloat16().cpu(), r.cpu(), w.cpu(), 1e-6)
    assert rel_err(out, ro.to(DEV)) < 5e-3 and rel_err(res, rres.to(DEV)) < 5e-3


def test_silu_and_mul():
    x = torch.randn(13, 2 * 1024, device=DEV).bfloat16()
    assert rel_err(activation.silu_and_mul(x), activation.silu_and_mul_ref(x.cpu()).to(DEV)) < 5e-3


def test_embedding():
    table = torch.randn(1000, 256, device=DEV).bfloat16()
    ids = torch.randint(0, 1000, (17,), device=DEV)
    assert torch.equal(kv.embedding(ids, table), table[ids])


@pytest.mark.parametrize("hd", [64, 128])
@pytest.mark.parametrize("qknorm", [True, False])
def test_qkv_norm_rope_store(hd, qknorm):
    T, nh, nkv, bs, nblk = 21, 8, 2, 16, 8
    qkv = torch.randn(T, (nh + 2 * nkv) * hd, device=DEV).bfloat16()
    pos = torch.randint(0, 500, (T,), device=DEV)
    cs = rope.build_cos_sin_cache(hd, 1024, 1e6).to(DEV)
    qw = (1 + 0.1 * torch.randn(hd, device=DEV)).bfloat16() if qknorm else None
    kw = (1 + 0.1 * torch.randn(hd, device=DEV)).bfloat16() if qknorm else None
    kc = torch.zeros(nblk, nkv, bs, hd, device=DEV, dtype=torch.bfloat16)
    vc = torch.zeros_like(kc)
    slots = torch.randperm(nblk * bs, device=DEV)[:T].int()
    slots[3] = -1
    q, _, _ = rope.qkv_norm_rope_store(qkv, pos, cs, qw, kw, 1e-6, kc, vc, slots, nh, nkv, hd)
    kc_ref, vc_ref = torch.zeros_like(kc).cpu(), torch.zeros_like(vc).cpu()
    q_ref, k_ref, v_ref = rope.qkv_norm_rope_store(qkv.cpu(), pos.cpu(), cs.cpu(), None if qw is None else qw.cpu(),
                                                   None if kw is None else kw.cpu(), 1e-6, kc_ref, vc_ref,
                                                   slots.cpu(), nh, nkv, hd)
    assert rel_err(q, q_ref.to(DEV)) < 5e-3
    assert rel_err(kc, kc_ref.to(DEV)) < 5e-3
    assert torch.equal(vc.cpu(), vc_ref)
    qn, kn, vn = rope.qkv_norm_rope_store(qkv, pos, cs, qw, kw, 1e-6, None, None, None, nh, nkv, hd)
    assert rel_err(qn, q_ref.to(DEV)) < 5e-3 and rel_err(kn, k_ref.to(DEV)) < 5e-3


def _pool(nblk, nkv, bs, hd, seed=0):
    g = torch.Generator(device=DEV).manual_seed(seed)
    kc = torch.randn(nblk, nkv, bs, hd, device=DEV, generator=g).bfloat16()
    vc = torch.randn(nblk, nkv, bs, hd, device=DEV, generator=g).bfloat16()
    return kc, vc


@pytest.mark.parametrize("bs", [16, 32, 64, 256])
@pytest.mark.parametrize("hd,nh,nkv", [(128, 32, 8), (64, 4, 2), (128, 4, 1)])
def test_decode_attention(bs, hd, nh, nkv):
    lens = [1, 5, 64, 65, 300, 513, 1200]
    B = len(lens)
    maxblk = max(-(-L // bs) for L in lens)
    nblk = B * maxblk + 3
    kc, vc = _pool(nblk, nkv, bs, hd)
    perm = torch.randperm(nblk)[: B * maxblk].view(B, maxblk).int().to(DEV)
    ctx = torch.tensor(lens, dtype=torch.int32, device=DEV)
    q = torch.randn(B, nh, hd, device=DEV).bfloat16()
    scale = 1 / math.sqrt(hd)
    out = attention.decode_attention(q, kc, vc, perm, ctx, scale)
    ref = attention.decode_attention_ref(q.cpu().float(), kc.cpu().float(), vc.cpu().float(), perm.cpu(), ctx.cpu(), scale)
    assert rel_err(out, ref.to(DEV)) < 1e-2


@pytest.mark.parametrize("B,partition", [(3, 128), (40, 128), (80, 256), (80, 512)])
def test_decode_attention_tma_poisoned_pool(B, partition):
    """Persistent TMA decode kernel: pool slots past each context hold NaN (the kernel must mask
    K and zero V there), many chunks per context, repeated launches (self-resetting counters)
    and agreement with the cp.async split-KV kernel."""
    hd, nh, nkv, bs = 128, 32, 8, 256
    g = torch.Generator(device=DEV).manual_seed(B)
    lens = torch.randint(1, 1500, (B,), generator=g, device=DEV).tolist()
    maxblk = max(-(-L // bs) for L in lens)
    nblk = B * maxblk + 2
    kc = torch.full((nblk, nkv, bs, hd), float("nan"), device=DEV).bfloat16()
    vc = torch.full_like(kc, float("nan"))
    perm = torch.randperm(nblk, generator=g, device=DEV)[: B * maxblk].view(B, maxblk).int()
    for b, L in enumerate(lens):
        for j in range(-(-L // bs)):
            n = min(bs, L - j * bs)
            blk = int(perm[b, j])
            kc[blk, :, :n] = torch.randn(nkv, n, hd, device=DEV, generator=g).bfloat16()
            vc[blk, :, :n] = torch.randn(nkv, n, hd, device=DEV, generator=g).bfloat16()
    ctx = torch.tensor(lens, dtype=torch.int32, device=DEV)
    q = torch.randn(B, nh, hd, device=DEV, generator=g).bfloat16()
    scale = 1 / math.sqrt(hd)
    ws = attention.DecodeWorkspace(B, nh, hd, maxblk * bs, DEV)
    ref = attention.decode_attention_ref(q.cpu().float(), kc.cpu().float(), vc.cpu().float(), perm.cpu(), ctx.cpu(),
                                         scale).to(DEV)
    for _ in range(3):
        out = torch.empty_like(q)
        C().decode_attention_tma(out, q, kc, vc, perm, ctx, scale, ws.partial_out, ws.partial_ml, ws.counters,
                                 ws.max_splits, partition, 1, status(torch.device(DEV)))
        torch.cuda.synchronize()
        assert torch.isfinite(out.float()).all()
        assert rel_err(out, ref) < 1e-2
    assert int(ws.counters.abs().sum()) == 0
    old = torch.empty_like(q)
    C().decode_attention(old, q, kc, vc, perm, ctx, scale, ws.partial_out, ws.partial_ml, ws.counters,
                         -(-ws.max_splits * 128 // 256), 256, 0, status(torch.device(DEV)))
    torch.cuda.synchronize()
    assert torch.isfinite(old.float()).all() and rel_err(out, old) < 5e-3


@pytest.mark.parametrize("tma", [True, False])
def test_decode_attention_out_of_range_blocks_and_long_context(tma):
    """A block id outside the pool is never read (zeros, kBadIndex recorded) and a context longer
    than its block-table row is clamped to the row; a correct call afterwards is unaffected."""
    hd, nh, nkv, bs = 128, 8, 2, 64
    B, width = 4, 3
    nblk = B * width
    kc, vc = _pool(nblk, nkv, bs, hd, seed=11)
    tables = torch.randperm(nblk, device=DEV)[: B * width].view(B, width).int().contiguous()
    lens = [100, 150, 192, 30]
    ctx = torch.tensor(lens, dtype=torch.int32, device=DEV)
    q = torch.randn(B, nh, hd, device=DEV).bfloat16()
    scale = 1 / math.sqrt(hd)
    ws = attention.DecodeWorkspace(B, nh, hd, width * bs, DEV)
    st = status(torch.device(DEV))

    def run(t, c):
        out = torch.empty_like(q)
        if tma:
            C().decode_attention_tma(out, q, kc, vc, t, c, scale, ws.partial_out, ws.partial_ml, ws.counters,
                                     ws.max_splits, 128, 1, st)
        else:
            C().decode_attention(out, q, kc, vc, t, c, scale, ws.partial_out, ws.partial_ml, ws.counters,
                                 ws.max_splits, 128, 0, st)
        torch.cuda.synchronize()
        return out

    bad = tables.clone()
    bad[1, 1] = nblk + 1000
    bad[2, 0] = -7
    out = run(bad, ctx)
    assert torch.isfinite(out.float()).all()
    with pytest.raises(RuntimeError, match="out-of-range"):
        check_status(torch.device(DEV))
    # rows whose blocks are all valid are exact
    ref = attention.decode_attention_ref(q.cpu().float(), kc.cpu().float(), vc.cpu().float(), tables.cpu(),
                                         ctx.cpu(), scale).to(DEV)
    for b in (0, 3):
        assert rel_err(out[b], ref[b]) < 1e-2
    # a context past the table row (3 blocks = 192 keys) attends to the whole row, nothing more
    long_ctx = torch.tensor([100, 150, 10_000, 30], dtype=torch.int32, device=DEV)
    out = run(tables, long_ctx)
    check_status(torch.device(DEV))
    assert rel_err(out, ref) < 1e-2          # 192 == the clamp for row 2
    assert int(ws.counters.abs().sum()) == 0
    assert rel_err(run(tables, ctx), ref) < 1e-2


@pytest.mark.parametrize("nq", [1, 2, 4])
@pytest.mark.parametrize("bs", [16, 256])
@pytest.mark.parametrize("hd,nh,nkv", [(128, 32, 8), (64, 8, 4), (64, 16, 2)])
def test_verify_attention_on_decode_kernel_matches_fp32(nq, bs, hd, nh, nkv):
    """A packed verify chunk (nq new tokens per sequence, causal among themselves) on the TMA decode
    kernel, the (query, head) rows of each KV head in one MMA tile, against fp32 varlen attention;
    contexts from a few keys to several split-KV chunks, NaN in every pool slot no context reaches."""
    g = torch.Generator(device=DEV).manual_seed(nq * 10 + bs)
    lens = [nq + 3, 90, 300, 1000, 129, 64 + nq]
    maxblk = max(-(-k // bs) for k in lens)
    nblk = len(lens) * maxblk + 2
    kc = torch.randn(nblk, nkv, bs, hd, device=DEV, generator=g).bfloat16()
    vc = torch.randn(nblk, nkv, bs, hd, device=DEV, generator=g).bfloat16()
    tables = torch.randperm(nblk, device=DEV, generator=g)[:len(lens) * maxblk].to(torch.int32).view(len(lens), maxblk)
    used = torch.zeros(nblk, bs, dtype=torch.bool, device=DEV)
    for i, k in enumerate(lens):
        pos = torch.arange(k, device=DEV)
        used[tables[i, pos // bs].long(), pos % bs] = True
    keep = used.unsqueeze(1).unsqueeze(-1).expand_as(kc)
    ref_k, ref_v = kc.float().cpu(), vc.float().cpu()
    kc[~keep] = float("nan")
    vc[~keep] = float("nan")
    B = len(lens)
    q = torch.randn(B * nq, nh, hd, device=DEV, generator=g).bfloat16()
    seqk = torch.tensor(lens, dtype=torch.int32, device=DEV)
    scale = 1 / math.sqrt(hd)
    ws = attention.DecodeWorkspace(B * nq, nh, hd, maxblk * bs, DEV)
    if nq * (nh // nkv) > 16:
        assert not attention.verify_fits_decode_kernel(nq, nh, nkv, bs, hd)
        return
    assert attention.verify_fits_decode_kernel(nq, nh, nkv, bs, hd)
    cu = torch.arange(0, (B + 1) * nq, nq, dtype=torch.int32)
    ref = attention.prefill_attention_ref(q.cpu().float(), ref_k, ref_v, cu, seqk.cpu(), tables.cpu(), scale)
    for _ in range(2):    # twice: the split counters must reset themselves
        out = attention.verify_attention(q, kc, vc, tables, seqk, scale, nq, ws)
        torch.cuda.synchronize()
        assert torch.isfinite(out.float()).all()
        assert rel_err(out, ref.to(DEV)) < 1e-2
    assert int(ws.counters.abs().sum()) == 0


def test_prefill_and_tree_attention_skip_out_of_range_blocks():
    hd, nh, nkv, bs = 128, 4, 2, 16
    kc, vc = _pool(8, nkv, bs, hd, seed=12)
    tables = torch.tensor([[0, 1, 2, 99]], dtype=torch.int32, device=DEV)
    q = torch.randn(60, nh, hd, device=DEV).bfloat16()
    cu = torch.tensor([0, 60], dtype=torch.int32, device=DEV)
    ks = torch.tensor([60], dtype=torch.int32, device=DEV)
    out = attention.prefill_attention(q, kc, vc, cu, ks, tables, 0.088, 60)
    torch.cuda.synchronize()
    assert torch.isfinite(out.float()).all()
    with pytest.raises(RuntimeError, match="out-of-range"):
        check_status(torch.device(DEV))
    tk = torch.randn(3, nkv, hd, device=DEV).bfloat16()
    mask = torch.ones(3, 3, dtype=torch.bool, device=DEV).tril()
    out = attention.tree_attention(q[:3], kc, vc, tables[0], 60, tk, tk, mask, 0.088)
    torch.cuda.synchronize()
    assert torch.isfinite(out.float()).all()
    with pytest.raises(RuntimeError, match="out-of-range"):
        check_status(torch.device(DEV))


@pytest.mark.parametrize("bs", [16, 256])
@pytest.mark.parametrize("hd,nh,nkv", [(128, 8, 2), (64, 4, 2)])
def test_prefill_attention_varlen_paged(bs, hd, nh, nkv):
    # (q_len, k_len): plain prefill, chunk with cached prefix, verify-sized chunks
    shapes = [(37, 37), (130, 200), (4, 301), (64, 64), (1, 9)]
    maxblk = max(-(-k // bs) for _, k in shapes)
    nblk = len(shapes) * maxblk
    kc, vc = _pool(nblk, nkv, bs, hd, seed=3)
    tables = torch.arange(nblk, dtype=torch.int32, device=DEV)[torch.randperm(nblk)].view(len(shapes), maxblk)
    cu = [0]
    for ql, _ in shapes:
        cu.append(cu[-1] + ql)
    q = torch.randn(cu[-1], nh, hd, device=DEV).bfloat16()
    cu_t = torch.tensor(cu, dtype=torch.int32, device=DEV)
    ks = torch.tensor([k for _, k in shapes], dtype=torch.int32, device=DEV)
    scale = 1 / math.sqrt(hd)
    out = attention.prefill_attention(q, kc, vc, cu_t, ks, tables, scale, max(s[0] for s in shapes))
    ref = attention.prefill_attention_ref(q.cpu().float(), kc.cpu().float(), vc.cpu().float(), cu_t.cpu(), ks.cpu(),
                                          tables.cpu(), scale)
    assert rel_err(out, ref.to(DEV)) < 1e-2


def test_tree_attention():
    from llmserve_b200.speculative.tree import build_fixed_tree_topology
    hd, nh, nkv, bs = 128, 8, 2, 16
    topo = build_fixed_tree_topology(10)
    n = len(topo.parents)
    kc, vc = _pool(20, nkv, bs, hd, seed=5)
    table = torch.randperm(20)[:10].int().to(DEV)
    prefix = 133
    q = torch.randn(n, nh, hd, device=DEV).bfloat16()
    tk = torch.randn(n, nkv, hd, device=DEV).bfloat16()
    tv = torch.randn(n, nkv, hd, device=DEV).bfloat16()
    mask = topo.attention_mask(DEV)
    out = attention.tree_attention(q, kc, vc, table, prefix, tk, tv, mask, 0.088)
    ref = attention.tree_attention_ref(q.cpu().float(), kc.cpu().float(), vc.cpu().float(), table.cpu(), prefix,
                                       tk.cpu().float(), tv.cpu().float(), mask.cpu(), 0.088)
    assert rel_err(out, ref.to(DEV)) < 1e-2


def test_store_kvcache_and_tree_commit():
    nkv, hd, bs = 2, 128, 16
    kc = torch.zeros(4, nkv, bs, hd, device=DEV, dtype=torch.bfloat16)
    vc = torch.zeros_like(kc)
    k = torch.randn(5, nkv, hd, device=DEV).bfloat16()
    v = torch.randn(5, nkv, hd, device=DEV).bfloat16()
    slots = torch.tensor([3, 17, -1, 40, 63], dtype=torch.int32, device=DEV)
    kv.store_kvcache(k, v, kc, vc, slots)
    kr, vr = torch.zeros_like(kc).cpu(), torch.zeros_like(vc).cpu()
    rope.store_kv_ref(k.cpu(), v.cpu(), kr, vr, slots.cpu())
    assert torch.equal(kc.cpu(), kr) and torch.equal(vc.cpu(), vr)
    L = 3
    tk = torch.randn(L, 6, nkv, hd, device=DEV).bfloat16()
    tv = torch.randn(L, 6, nkv, hd, device=DEV).bfloat16()
    KC = torch.zeros(L, 4, nkv, bs, hd, device=DEV, dtype=torch.bfloat16)
    VC = torch.zeros_like(KC)
    nodes = torch.tensor([0, 2, 5], dtype=torch.int32, device=DEV)
    sl = torch.tensor([7, 8, 33], dtype=torch.int32, device=DEV)
    kv.commit_tree_kv(tk, tv, KC, VC, nodes, sl)
    KR, VR = torch.zeros_like(KC).cpu(), torch.zeros_like(VC).cpu()
    kv.commit_tree_kv_ref(tk.cpu(), tv.cpu(), KR, VR, nodes.cpu(), sl.cpu())
    assert torch.equal(KC.cpu(), KR) and torch.equal(VC.cpu(), VR)


def test_argmax_and_sampling():
    logits = torch.randn(9, 151936 // 8, device=DEV).bfloat16()
    logits[3, 100] = 50.0
    logits[3, 7] = 50.0   # tie -> lowest index
    idx = sampling.argmax(logits)
    assert torch.equal(idx.cpu(), logits.float().cpu().argmax(-1))
    assert int(idx[3]) == 7
    temps = torch.full((9,), 0.7, device=DEV)
    got = sampling.sample(logits.float(), temps, 1234)
    want = sampling.sample(logits.float().cpu(), temps.cpu(), 1234)
    assert (got.cpu() == want).float().mean() >= 8 / 9


@pytest.mark.parametrize("S", [2, 3, 4, 5, 6, 7, 8])
def test_qkv_rope_from_splitk_partials(S):
    T, nh, nkv, hd, bs, nblk = 9, 8, 2, 128, 256, 2
    W = (nh + 2 * nkv) * hd
    parts = torch.randn(S, T, W, device=DEV) * 0.5
    pos = torch.arange(T, device=DEV) * 7
    cs = rope.build_cos_sin_cache(hd, 1024, 1e6).to(DEV)
    qw = (1 + 0.1 * torch.randn(hd, device=DEV)).bfloat16()
    kw = (1 + 0.1 * torch.randn(hd, device=DEV)).bfloat16()
    slots = torch.arange(T, dtype=torch.int32, device=DEV) + 17
    kc1 = torch.zeros(nblk, nkv, bs, hd, device=DEV, dtype=torch.bfloat16)
    vc1, kc2, vc2 = torch.zeros_like(kc1), torch.zeros_like(kc1), torch.zeros_like(kc1)
    q1, _, _ = rope.qkv_norm_rope_store(parts, pos, cs, qw, kw, 1e-6, kc1, vc1, slots, nh, nkv, hd)
    q2, _, _ = rope.qkv_norm_rope_store(parts.sum(0).bfloat16(), pos, cs, qw, kw, 1e-6, kc2, vc2, slots, nh, nkv, hd)
    assert rel_err(q1, q2) < 2e-3 and rel_err(kc1, kc2) < 2e-3 and rel_err(vc1, vc2) < 2e-3


@pytest.mark.parametrize("T", [1, 16, 64, 200])
@pytest.mark.parametrize("I,K", [(512, 256), (1536, 4096)])
def test_gate_up_silu_fused_epilogue(T, I, K):
    g = torch.Generator(device=DEV).manual_seed(T + I)
    x = torch.randn(T, K, device=DEV, generator=g).bfloat16()
    w = (torch.randn(2 * I, K, device=DEV, generator=g) * 0.05).bfloat16()
    ref = activation.silu_and_mul_ref((x.float() @ w.float().t()).bfloat16().cpu()).to(DEV)
    wi = gemm.interleave_gate_up(w)
    out = gemm.linear_silu(x, wi)
    assert rel_err(out, ref) < 1e-2
    out2 = gemm.linear_silu(x, wi, max_splits=1)
    assert rel_err(out2, ref) < 1e-2
    # forced split-K path through the interleaved reduction
    parts = gemm.linear_partials(x, wi, 4)
    o3 = torch.empty(T, I, device=DEV, dtype=torch.bfloat16)
    C().splitk_silu(o3, parts)
    assert rel_err(o3, ref) < 1e-2
    # tile-packed interleaved weight (the engine's layout): fused epilogue and split-K paths
    pw = gemm.pack_weight(wi)
    assert rel_err(gemm.linear_silu(x, pw), ref) < 1e-2
    assert rel_err(gemm.linear_silu(x, pw, max_splits=1), ref) < 1e-2


@pytest.mark.parametrize("T", [300, 1024])
def test_gate_up_silu_prefill_sized_interleaved(T):
    """Above the epilogue's token range the interleaved projection runs on the 2-SM kernel and the
    interleaved SiLU-mul kernel."""
    I, K = 1536, 1024
    x = torch.randn(T, K, device=DEV).bfloat16()
    w = (torch.randn(2 * I, K, device=DEV) * 0.05).bfloat16()
    ref = activation.silu_and_mul_ref((x.float() @ w.float().t()).bfloat16().cpu()).to(DEV)
    pw = gemm.pack_weight(gemm.interleave_gate_up(w))
    assert rel_err(gemm.linear_silu(x, pw), ref) < 1e-2


def test_kv_push_blocks_same_gpu_and_bad_ids():
    L, nkv, bs, hd = 3, 2, 16, 64
    src_k = torch.randn(L, 10, nkv, bs, hd, device=DEV).bfloat16()
    src_v = torch.randn_like(src_k)
    dst_k = torch.zeros(L, 7, nkv, bs, hd, device=DEV, dtype=torch.bfloat16)
    dst_v = torch.zeros_like(dst_k)
    kv.push_blocks(src_k, src_v, dst_k, dst_v, [4, 0, 9], [6, 2, 3])
    torch.cuda.synchronize()
    for s, d in ((4, 6), (0, 2), (9, 3)):
        assert torch.equal(dst_k[:, d], src_k[:, s]) and torch.equal(dst_v[:, d], src_v[:, s])
    assert not dst_k[:, [0, 1, 4, 5]].any()
    kv.push_blocks(src_k, src_v, dst_k, dst_v, [1], [7])        # destination id out of range: skipped
    with pytest.raises(RuntimeError, match="out-of-range"):
        check_status(torch.device(DEV))


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_kv_push_blocks_to_peer_gpu():
    src_k = torch.randn(2, 6, 8, 256, 128, device="cuda:0").bfloat16()
    src_v = torch.randn_like(src_k)
    dst_k = torch.zeros(2, 5, 8, 256, 128, device="cuda:1", dtype=torch.bfloat16)
    dst_v = torch.zeros_like(dst_k)
    kv.push_blocks(src_k, src_v, dst_k, dst_v, [5, 2], [0, 4])
    torch.cuda.synchronize(0)
    assert torch.equal(dst_k[:, 0].cpu(), src_k[:, 5].cpu()) and torch.equal(dst_v[:, 4].cpu(), src_v[:, 2].cpu())


def test_greedy_accept_kernel_matches_batched_reference():
    from llmserve_b200.speculative.sampling import greedy_accept_packed
    g = torch.Generator().manual_seed(9)
    B, gam = 37, 3
    draft = torch.randint(0, 5, (B, gam), generator=g)
    target = torch.randint(0, 5, (B, gam + 1), generator=g)
    target[:8, :gam] = draft[:8]                   # full acceptance rows: the bonus token is final
    start = torch.randint(0, 1000, (B,), generator=g)
    want = greedy_accept_packed(target, draft, start)
    got = greedy_accept_packed(target.to(DEV), draft.to(DEV), start.to(DEV))
    assert torch.equal(got.cpu(), want)
    assert (want[:8, 0] == gam).all() and torch.equal(want[:8, 1], target[:8, gam])


def test_fused_collective_wait_on_unset_flag_returns_error_status():
    """Failure detection on the device without a fault: a two-rank fused collective whose second
    rank never runs (its buffer is local memory nothing writes).  Rank 0's polls for the peer's
    epoch-tagged words give up after the (lowered) spin limit, record the error in the status word
    and let the kernel finish; the host raises, and the context stays usable.  The same holds for
    the vocab-parallel argmax exchange."""
    from llmserve_b200.parallel.comm import FusedComm
    hidden, T, cap, world = 4096, 4, 64, 2
    off = FusedComm.offsets(hidden, cap, world)
    bufs = [C().comm_alloc(off["total"]) for _ in range(world)]
    dev = torch.device("cuda", torch.cuda.current_device())
    try:
        res_in = torch.randn(T, hidden, device=dev).bfloat16()
        w = torch.ones(hidden, device=dev).bfloat16()
        C().comm_set_spin_limit(1 << 16)
        C().row_parallel_finish([b + off["ag"] for b in bufs], bufs[0] + off["inbox"], bufs[0], bufs[0] + off["out"],
                                bufs[0] + off["res"], res_in, w, 0, 1, T, hidden, 2, 1e-6, 3, status(dev))
        torch.cuda.synchronize()
        with pytest.raises(RuntimeError, match="peer flag wait timed out"):
            check_status(dev)
        vals = torch.randn(3, device=dev)
        idx = torch.arange(3, device=dev)
        tok = torch.empty(3, dtype=torch.int64, device=dev)
        C().vocab_argmax_exchange(bufs, vals, idx, 0, tok, 0, status(dev))
        torch.cuda.synchronize()
        with pytest.raises(RuntimeError, match="peer flag wait timed out"):
            check_status(dev)
        x = torch.randn(64, 64, device=dev)
        assert torch.isfinite(x @ x).all()
    finally:
        C().comm_set_spin_limit(1 << 40)           # back to the default (clamped to the compile-time limit)
        torch.cuda.synchronize()
        for b in bufs:
            C().comm_free(b)


def _wrap_dev(ptr, nbytes, dtype):
    from llmserve_b200.parallel.comm import _wrap
    return _wrap(ptr, nbytes, torch.device(DEV)).view(dtype)


@pytest.mark.parametrize("reduce", [False, True])
@pytest.mark.parametrize("world,T,packed", [(1, 5, False), (2, 64, True), (4, 7, True), (4, 64, False),
                                            (8, 64, True), (8, 13, False)])
@pytest.mark.parametrize("calls", [1, 2])
def test_row_parallel_push_layout_single_gpu(world, T, packed, reduce, calls):
    """The fused row-parallel path's data layout on one GPU: each emulated rank's GEMM stores its
    epoch-tagged partial planes into the owners' inboxes, then every rank's finish kernel reduces
    the rows it owns, normalises them and pushes them (phase 1, all ranks), then every rank unpacks
    the rows the others own (phase 2), so no launch waits on a later one.  Every rank must then hold
    add+RMSNorm of the full fp32 product; a second call (next epoch, new inputs) must not see the
    first call's words."""
    from llmserve_b200.parallel.comm import FusedComm
    hidden, K, cap, S = 512, 256, 64, 3
    off = FusedComm.offsets(hidden, cap, world)
    bufs = [C().comm_alloc(off["total"]) for _ in range(world)]
    st = status(torch.device(DEV))
    try:
        ags = [b + off["ag"] for b in bufs]
        inboxes = [b + off["inbox"] for b in bufs]
        rows = -(-T // world)
        for call in range(calls):
            g = torch.Generator(device=DEV).manual_seed(world * 100 + T + 7 * call)
            xs = [torch.randn(T, K, device=DEV, generator=g).bfloat16() for _ in range(world)]
            ws = [(torch.randn(hidden, K, device=DEV, generator=g) * 0.05).bfloat16() for _ in range(world)]
            res_in = torch.randn(T, hidden, device=DEV, generator=g).bfloat16()
            nw = (1 + 0.1 * torch.randn(hidden, device=DEV, generator=g)).bfloat16()
            for r in range(world):
                w = gemm.pack_weight(ws[r]).data if packed else ws[r]
                C().gemm_bf16_to_owners(xs[r], w, hidden, packed, inboxes, r, rows, S, reduce, bufs[r], st, 0)
            planes = 1 if reduce else S
            for phase in (1, 2):
                for r in range(world):
                    C().row_parallel_finish(ags, inboxes[r], bufs[r], bufs[r] + off["out"], bufs[r] + off["res"],
                                            res_in, nw, r, planes, T, hidden, rows, 1e-6, phase, st)
            torch.cuda.synchronize()
            y = sum(x.float() @ w.float().t() for x, w in zip(xs, ws)).bfloat16()
            href, rref = norm.add_rms_norm_ref(y.cpu(), res_in.cpu(), nw.cpu(), 1e-6)
            for r in range(world):
                h = _wrap_dev(bufs[r] + off["out"], T * hidden * 2, torch.bfloat16).view(T, hidden)
                rr = _wrap_dev(bufs[r] + off["res"], T * hidden * 2, torch.bfloat16).view(T, hidden)
                assert rel_err(h, href.to(DEV)) < 1e-2, (call, r)
                assert rel_err(rr, rref.to(DEV)) < 1e-2, (call, r)
                assert int(_wrap_dev(bufs[r], 8, torch.int32)[0]) == call + 1     # epoch advanced once per call
    finally:
        torch.cuda.synchronize()
        for b in bufs:
            C().comm_free(b)


def test_vocab_argmax_exchange_single_gpu():
    """Two emulated ranks: rank 1's (value, index) pairs are written into rank 0's slots and its
    arrival flag pre-set, so rank 0's exchange kernel runs alone; ties go to the lower global id."""
    from llmserve_b200.parallel.comm import FusedComm
    world, rows, shard = 2, 37, 1000
    bufs = [C().comm_alloc(FusedComm.buffer_bytes(512, 64, world)) for _ in range(world)]
    try:
        g = torch.Generator(device=DEV).manual_seed(3)
        vals = [torch.randn(rows, device=DEV, generator=g) for _ in range(world)]
        idx = [torch.randint(0, shard, (rows,), device=DEV, generator=g) for _ in range(world)]
        vals[1][:5] = vals[0][:5]                       # ties: rank 0's ids are lower
        slots = _wrap_dev(bufs[0] + 1024, 2 * 8 * 512 * 8, torch.int32).view(2, 8, 512, 2)
        slots[1, 1, :rows, 0] = vals[1].view(torch.int32)     # epoch 1 -> parity 1
        slots[1, 1, :rows, 1] = (idx[1] + shard).int()
        _wrap_dev(bufs[0], 1024, torch.int32)[64 + 1] = 1
        out = torch.empty(rows, dtype=torch.int64, device=DEV)
        C().vocab_argmax_exchange(bufs, vals[0], idx[0], 0, out, 0, status(torch.device(DEV)))
        torch.cuda.synchronize()
        full_v = torch.stack(vals)
        full_i = torch.stack([idx[0], idx[1] + shard])
        best = full_v.argmax(0)                          # first maximum -> rank 0 on ties
        ref = full_i.gather(0, best.view(1, -1)).view(-1)
        assert torch.equal(out, ref)
    finally:
        torch.cuda.synchronize()
        for b in bufs:
            C().comm_free(b)


@pytest.mark.parametrize("T", [1, 16, 33, 64, 100, 256, 300])
@pytest.mark.parametrize("splits", [1, 2, 3, 7, 16])
@pytest.mark.parametrize("packed", [False, True])
def test_cluster_reduced_gemm_matches_fp32(T, splits, packed):
    """K split over a thread-block cluster whose CTAs reduce their accumulators through distributed
    shared memory: bf16 output and the single fp32 plane both equal the fp32 product."""
    N, K = 384, 1088              # 17 K tiles: uneven slices; 3 weight tiles
    g = torch.Generator(device=DEV).manual_seed(T * 31 + splits)
    x = torch.randn(T, K, device=DEV, generator=g).bfloat16()
    w = (torch.randn(N, K, device=DEV, generator=g) * 0.05).bfloat16()
    ref = x.float() @ w.float().t()
    wd = gemm.pack_weight(w).data if packed else w
    out = torch.full((T, N), float("nan"), device=DEV).bfloat16()
    empty = torch.empty(0, device=DEV)
    C().gemm_bf16_reduced(out, x, wd, N, packed, empty, splits, status(torch.device(DEV)), 4 if T <= 64 else 0)
    assert rel_err(out, ref) < 1e-2
    plane = torch.full((1, T, N), float("nan"), device=DEV)
    C().gemm_bf16_reduced(torch.empty(0, device=DEV).bfloat16(), x, wd, N, packed, plane, splits,
                          status(torch.device(DEV)), 0)
    assert rel_err(plane[0], ref) < 1e-3


@pytest.mark.parametrize("T,splits", [(7, 4), (64, 3), (64, 16), (200, 2)])
def test_cluster_reduced_silu_gemm(T, splits):
    I, K = 640, 1024
    g = torch.Generator(device=DEV).manual_seed(T + splits)
    x = torch.randn(T, K, device=DEV, generator=g).bfloat16()
    w = (torch.randn(2 * I, K, device=DEV, generator=g) * 0.05).bfloat16()
    ref = activation.silu_and_mul_ref((x.float() @ w.float().t()).bfloat16().cpu()).to(DEV)
    wi = gemm.pack_weight(gemm.interleave_gate_up(w))
    out = torch.empty(T, I, device=DEV).bfloat16()
    C().gemm_bf16_silu_reduced(out, x, wi.data, wi.n, True, splits, status(torch.device(DEV)), 4 if T <= 64 else 0)
    assert rel_err(out, ref) < 1e-2


def test_linear_uses_cluster_splits_policy():
    """The engine's linear on decode shapes (cluster path by default) equals fp32."""
    for T, N, K in [(64, 6144, 4096), (64, 4096, 512), (16, 24576, 4096), (64, 768, 4096)]:
        x = torch.randn(T, K, device=DEV).bfloat16()
        w = gemm.pack_weight((torch.randn(N, K, device=DEV) * 0.02).bfloat16())
        assert gemm.cluster_splits(T, N, K) >= 1
        assert rel_err(gemm.linear(x, w), x.float() @ w.unpack().float().t()) < 1e-2
