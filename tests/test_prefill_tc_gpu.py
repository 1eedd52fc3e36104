"""The tcgen05 prefill attention kernel (``ops/csrc/prefill_sm100.cu``) against an fp32 PyTorch
reference of varlen causal attention over the paged pool: plain prefill, chunks after a cached
prefix, several 128-row query tiles, block sizes below / at / above the 64-key tile, head dims 64
and 128, a pool whose unused slots hold NaN (nothing outside a sequence's context may reach its
output), and an out-of-range block id (skipped, reported, output finite)."""
import math

import pytest
import torch

pytestmark = pytest.mark.gpu

from llmserve_b200.ops import attention  # noqa: E402
from llmserve_b200.ops._ext import C, check_status  # noqa: E402

DEV = "cuda"


def rel_err(a, b):
    a, b = a.float(), b.float()
    return ((a - b).norm() / (b.norm() + 1e-12)).item()


def _case(shapes, bs, hd, nh, nkv, seed=0, poison=True):
    g = torch.Generator(device=DEV).manual_seed(seed)
    maxblk = max(-(-k // bs) for _, k in shapes)
    nblk = len(shapes) * maxblk + 3
    kc = torch.randn(nblk, nkv, bs, hd, device=DEV, generator=g).bfloat16()
    vc = torch.randn(nblk, nkv, bs, hd, device=DEV, generator=g).bfloat16()
    perm = torch.randperm(nblk, device=DEV, generator=g)[:len(shapes) * maxblk]
    tables = perm.to(torch.int32).view(len(shapes), maxblk).contiguous()
    if poison:
        # NaN everywhere a sequence's context does not reach: unused blocks and the tail of the
        # last block of every sequence
        used = torch.zeros(nblk, bs, dtype=torch.bool, device=DEV)
        for i, (_, k) in enumerate(shapes):
            pos = torch.arange(k, device=DEV)
            used[tables[i, pos // bs].long(), pos % bs] = True
        kc[~used.unsqueeze(1).expand(-1, nkv, -1).unsqueeze(-1).expand_as(kc)] = float("nan")
        vc[~used.unsqueeze(1).expand(-1, nkv, -1).unsqueeze(-1).expand_as(vc)] = float("nan")
    cu = [0]
    for ql, _ in shapes:
        cu.append(cu[-1] + ql)
    q = torch.randn(cu[-1], nh, hd, device=DEV, generator=g).bfloat16()
    cu_t = torch.tensor(cu, dtype=torch.int32, device=DEV)
    ks = torch.tensor([k for _, k in shapes], dtype=torch.int32, device=DEV)
    return q, kc, vc, cu_t, ks, tables


def _ref(q, kc, vc, cu_t, ks, tables, scale):
    kc_c, vc_c = kc.float().cpu(), vc.float().cpu()
    return attention.prefill_attention_ref(q.cpu().float(), torch.nan_to_num(kc_c), torch.nan_to_num(vc_c),
                                           cu_t.cpu(), ks.cpu(), tables.cpu(), scale)


@pytest.mark.parametrize("bs", [16, 64, 256])
@pytest.mark.parametrize("hd,nh,nkv", [(128, 8, 2), (64, 4, 2), (128, 4, 4)])
def test_prefill_tc_matches_fp32_reference(bs, hd, nh, nkv):
    # (q_len, k_len): multi-tile prefill, chunk after a cached prefix, exact tile, one row, short
    shapes = [(300, 300), (130, 500), (128, 128), (1, 9), (257, 1000), (64, 64), (77, 77)]
    q, kc, vc, cu_t, ks, tables = _case(shapes, bs, hd, nh, nkv, seed=bs + hd)
    scale = 1 / math.sqrt(hd)
    assert C().prefill_tc_supported(bs, hd)
    out = attention.prefill_attention(q, kc, vc, cu_t, ks, tables, scale, max(s[0] for s in shapes), kernel="tc")
    torch.cuda.synchronize()
    check_status(torch.device(DEV))
    assert torch.isfinite(out.float()).all()
    ref = _ref(q, kc, vc, cu_t, ks, tables, scale)
    assert rel_err(out, ref.to(DEV)) < 1e-2
    # per sequence as well (a small sequence's error must not hide in a large one's norm)
    c = cu_t.tolist()
    for i in range(len(shapes)):
        assert rel_err(out[c[i]:c[i + 1]], ref[c[i]:c[i + 1]].to(DEV)) < 2e-2, i


def test_prefill_tc_long_prompt_matches_mma_kernel():
    """One 2048-token prompt at the Qwen3-8B head layout: the tcgen05 kernel equals the mma.sync
    kernel within bf16 rounding (both against the same paged pool)."""
    shapes = [(2048, 2048)]
    q, kc, vc, cu_t, ks, tables = _case(shapes, 256, 128, 32, 8, seed=5, poison=False)
    scale = 1 / math.sqrt(128)
    a = attention.prefill_attention(q, kc, vc, cu_t, ks, tables, scale, 2048, kernel="tc")
    b = attention.prefill_attention(q, kc, vc, cu_t, ks, tables, scale, 2048, kernel="mma")
    torch.cuda.synchronize()
    assert rel_err(a, b) < 1e-2


def test_prefill_tc_skips_out_of_range_blocks():
    hd, nh, nkv, bs = 128, 4, 2, 16
    g = torch.Generator(device=DEV).manual_seed(12)
    kc = torch.randn(8, nkv, bs, hd, device=DEV, generator=g).bfloat16()
    vc = torch.randn(8, nkv, bs, hd, device=DEV, generator=g).bfloat16()
    tables = torch.tensor([[0, 1, 2, 99, 3, 4, 5, 6, 7]], dtype=torch.int32, device=DEV)
    q = torch.randn(130, nh, hd, device=DEV, generator=g).bfloat16()
    cu = torch.tensor([0, 130], dtype=torch.int32, device=DEV)
    ks = torch.tensor([130], dtype=torch.int32, device=DEV)
    out = attention.prefill_attention(q, kc, vc, cu, ks, tables, 0.088, 130, kernel="tc")
    torch.cuda.synchronize()
    assert torch.isfinite(out.float()).all()
    with pytest.raises(RuntimeError, match="out-of-range"):
        check_status(torch.device(DEV))
