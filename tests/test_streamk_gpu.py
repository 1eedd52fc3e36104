"""Persistent stream-K decode GEMM (``gemm_streamk_sm100.cu``) against an fp32 PyTorch product,
and the reducers that consume its partial planes (any slot count 1..8)."""
import pytest
import torch

pytestmark = pytest.mark.gpu

from llmserve_b200.ops import activation, gemm, norm  # noqa: E402
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


@pytest.fixture
def streamk_on(monkeypatch):
    """The engine's entry points with stream-K enabled (``LLMSERVE_STREAMK_MAX_T=64``)."""
    monkeypatch.setattr(gemm, "STREAMK_MAX_T", 64)
    gemm.streamk_plan.cache_clear()
    yield
    monkeypatch.undo()
    gemm.streamk_plan.cache_clear()


SHAPES = [(1, 6144, 4096), (17, 4096, 4096), (64, 24576, 4096), (64, 4096, 12288), (33, 768, 4096),
          (100, 1000, 520), (128, 3072, 4096), (64, 4096, 512), (5, 256, 4096)]


@pytest.mark.parametrize("ctas", [1, 2])
@pytest.mark.parametrize("T,N,K", SHAPES)
def test_streamk_partials_sum_to_product(T, N, K, ctas, streamk_on):
    g = torch.Generator(device=DEV).manual_seed(T * 31 + N + K)
    x = torch.randn(T, K, device=DEV, generator=g).bfloat16()
    w = (torch.randn(N, K, device=DEV, generator=g) * 0.05).bfloat16()
    pw = gemm.pack_weight(w)
    grid, slots, stages = gemm.streamk_schedule(N, K, gemm._num_sms(x.device), ctas)
    # every plane starts as NaN: a slot the schedule leaves unwritten would poison the sum
    part = torch.full((slots, T, N), float("nan"), device=DEV)
    C().gemm_bf16_streamk(part, x, pw.data, N, grid, stages, status(x.device))
    torch.cuda.synchronize()
    ref = x.float() @ w.float().t()
    assert torch.isfinite(part).all()
    assert rel_err(part.sum(0), ref) < 1e-4
    if T > 64 or ctas != gemm.STREAMK_CTAS_PER_SM:
        return
    # through the public entry points: partial planes and the reduced bf16 output
    assert gemm.splits_for(T, pw) == slots
    assert rel_err(gemm.linear_partials(x, pw, slots).sum(0), ref) < 1e-4
    assert rel_err(gemm.linear(x, pw), ref) < 1e-2


def test_streamk_twice_in_a_row_reuses_nothing_stale(streamk_on):
    x = torch.randn(64, 4096, device=DEV).bfloat16()
    w1 = (torch.randn(4096, 4096, device=DEV) * 0.05).bfloat16()
    w2 = (torch.randn(4096, 4096, device=DEV) * 0.05).bfloat16()
    p1, p2 = gemm.pack_weight(w1), gemm.pack_weight(w2)
    s = gemm.splits_for(64, p1)
    a = gemm.linear_partials(x, p1, s).sum(0)
    b = gemm.linear_partials(x, p2, s).sum(0)
    assert rel_err(a, x.float() @ w1.float().t()) < 1e-4
    assert rel_err(b, x.float() @ w2.float().t()) < 1e-4


@pytest.mark.parametrize("T,I", [(1, 12288), (64, 12288), (40, 1536)])
def test_gate_up_silu_from_streamk(T, I, streamk_on):
    x = torch.randn(T, 4096, device=DEV).bfloat16()
    w = (torch.randn(2 * I, 4096, device=DEV) * 0.02).bfloat16()
    out = gemm.gate_up_silu(x, gemm.pack_weight(w))
    assert out is not None
    ref = activation.silu_and_mul_ref((x.float() @ w.float().t()).bfloat16().cpu()).to(DEV)
    assert rel_err(out, ref) < 1e-2


@pytest.mark.parametrize("S", [3, 5, 6, 7])
def test_add_rmsnorm_reducer_odd_slot_counts(S):
    parts = torch.randn(S, 9, 4096, device=DEV)
    r = torch.randn(9, 4096, device=DEV).bfloat16()
    w = (1 + 0.1 * torch.randn(4096, device=DEV)).bfloat16()
    out = torch.empty(9, 4096, device=DEV, dtype=torch.bfloat16)
    res = torch.empty_like(out)
    C().splitk_reduce_add_rmsnorm(out, res, parts, r, w, 1e-6)
    ro, rres = norm.add_rms_norm_ref(parts.sum(0).bfloat16().cpu(), r.cpu(), w.cpu(), 1e-6)
    assert rel_err(out, ro.to(DEV)) < 5e-3 and rel_err(res, rres.to(DEV)) < 5e-3
