"""The tcgen05 tree-verify attention kernel (``ops/csrc/tree_sm100.cu``) against an fp32 PyTorch
reference of the reference engine's tree attention (prefix keys all visible, tree keys under the
ancestor mask): the fixed 10-node EAGLE3 tree (11 rows with the root) and a subset of its rows
(the draft's per-depth calls), prefixes of 0 keys (tree tile only), a few tiles (one CTA per tile)
and thousands of keys (chunks merged by log-sum-exp), block sizes below / at / above the 64-key
tile, head dims 64 / 128, group sizes 4 / 8 / 16 (a full 128-row tile), NaN in every pool slot the
prefix does not reach, and an out-of-range block id (skipped, reported, output finite)."""
import math

import pytest
import torch

pytestmark = pytest.mark.gpu

from llmserve_b200.ops import attention  # noqa: E402
from llmserve_b200.ops._ext import C, check_status  # noqa: E402
from llmserve_b200.speculative.tree import build_fixed_tree_topology  # noqa: E402

DEV = "cuda"


def rel_err(a, b):
    a, b = a.float(), b.float()
    return ((a - b).norm() / (b.norm() + 1e-12)).item()


def _case(prefix, bs, hd, nh, nkv, seed=0):
    g = torch.Generator(device=DEV).manual_seed(seed)
    topo = build_fixed_tree_topology(10)
    n = len(topo.parents)
    used_blocks = max(1, -(-prefix // bs))
    nblk = used_blocks + 3
    kc = torch.randn(nblk, nkv, bs, hd, device=DEV, generator=g).bfloat16()
    vc = torch.randn(nblk, nkv, bs, hd, device=DEV, generator=g).bfloat16()
    table = torch.randperm(nblk, device=DEV, generator=g)[:used_blocks].to(torch.int32).contiguous()
    used = torch.zeros(nblk, bs, dtype=torch.bool, device=DEV)
    pos = torch.arange(prefix, device=DEV)
    used[table[pos // bs].long(), pos % bs] = True
    poison = ~used.unsqueeze(1).unsqueeze(-1).expand_as(kc)
    kc[poison] = float("nan")
    vc[poison] = float("nan")
    q = torch.randn(n, nh, hd, device=DEV, generator=g).bfloat16()
    tk = torch.randn(n, nkv, hd, device=DEV, generator=g).bfloat16()
    tv = torch.randn(n, nkv, hd, device=DEV, generator=g).bfloat16()
    return topo, q, kc, vc, table, tk, tv


def _ref(q, kc, vc, table, prefix, tk, tv, mask, scale):
    return attention.tree_attention_ref(q.cpu().float(), torch.nan_to_num(kc.cpu().float()),
                                        torch.nan_to_num(vc.cpu().float()), table.cpu(), prefix, tk.cpu().float(),
                                        tv.cpu().float(), mask.cpu(), scale)


@pytest.mark.parametrize("prefix", [0, 133, 3000])
@pytest.mark.parametrize("bs", [16, 64, 256])
@pytest.mark.parametrize("hd,nh,nkv", [(128, 32, 8), (64, 16, 2), (128, 8, 1)])
def test_tree_tc_matches_fp32_reference(prefix, bs, hd, nh, nkv):
    topo, q, kc, vc, table, tk, tv = _case(prefix, bs, hd, nh, nkv, seed=prefix + bs + hd)
    n = q.shape[0]
    assert C().tree_tc_supported(n, nh, nkv, n, bs, hd)
    mask = topo.attention_mask(DEV)
    scale = 1 / math.sqrt(hd)
    out = attention.tree_attention(q, kc, vc, table, prefix, tk, tv, mask, scale)
    torch.cuda.synchronize()
    check_status(torch.device(DEV))
    ref = _ref(q, kc, vc, table, prefix, tk, tv, mask, scale)
    assert torch.isfinite(out.float()).all()
    assert rel_err(out, ref.to(DEV)) < 1e-2
    # a subset of the rows (one draft depth) against all tree keys
    rows = torch.tensor([0, 2, 3, 7], device=DEV)
    out_s = attention.tree_attention(q[rows].contiguous(), kc, vc, table, prefix, tk, tv, mask[rows], scale)
    ref_s = _ref(q[rows], kc, vc, table, prefix, tk, tv, mask[rows], scale)
    assert rel_err(out_s, ref_s.to(DEV)) < 1e-2


@pytest.mark.parametrize("prefix", [70, 2500])
def test_tree_tc_full_tile_and_cuda_core_agree(prefix):
    # group size 16: 8 nodes x 16 heads fill all 128 rows of the tile
    hd, nh, nkv, bs = 128, 16, 1, 64
    topo, q, kc, vc, table, tk, tv = _case(prefix, bs, hd, nh, nkv, seed=11)
    rows = torch.arange(8, device=DEV)
    q8 = q[rows].contiguous()
    mask = topo.attention_mask(DEV)[rows]
    scale = 0.088
    out = attention.tree_attention(q8, kc, vc, table, prefix, tk, tv, mask, scale)
    saved = attention.TREE_TC
    attention.TREE_TC = False
    try:
        cc = attention.tree_attention(q8, kc, vc, table, prefix, tk, tv, mask, scale)
    finally:
        attention.TREE_TC = saved
    torch.cuda.synchronize()
    check_status(torch.device(DEV))
    ref = _ref(q8, kc, vc, table, prefix, tk, tv, mask, scale)
    assert rel_err(out, ref.to(DEV)) < 1e-2
    assert rel_err(out, cc) < 1e-2


def test_tree_tc_skips_out_of_range_block():
    hd, nh, nkv, bs = 128, 32, 8, 16
    topo, q, kc, vc, table, tk, tv = _case(100, bs, hd, nh, nkv, seed=5)
    table = table.clone()
    table[2] = 10_000
    out = attention.tree_attention(q, kc, vc, table, 100, tk, tv, topo.attention_mask(DEV), 0.088)
    torch.cuda.synchronize()
    assert torch.isfinite(out.float()).all()
    with pytest.raises(RuntimeError, match="out-of-range"):
        check_status(torch.device(DEV))
