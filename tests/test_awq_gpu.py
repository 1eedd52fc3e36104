"""AutoAWQ W4A16 on the sm_100a kernel against the dequantize-then-matmul fp32 reference."""
import os

import pytest
import torch

pytestmark = pytest.mark.gpu

from llmserve_b200.ops import awq as awq_ops  # noqa: E402
from llmserve_b200.ops._ext import check_status  # noqa: E402
from llmserve_b200.models.synthetic import awq_quantize_dense  # noqa: E402
from llmserve_b200.quantization.awq import dequantize_awq_gemm  # noqa: E402

DEV = "cuda"


def rel_err(a, b):
    a, b = a.float(), b.float()
    return ((a - b).norm() / (b.norm() + 1e-12)).item()


@pytest.fixture(autouse=True)
def _status():
    yield
    check_status(torch.device(DEV))


@pytest.mark.parametrize("T", [1, 5, 16, 33, 64, 200, 1000])
@pytest.mark.parametrize("N,K", [(296, 256), (4096, 4096), (1024, 12288)])
def test_awq_linear_matches_dequantized_fp32(T, N, K):
    g = torch.Generator().manual_seed(T * 31 + N + K)
    w = torch.randn(N, K, generator=g) * 0.05
    qw, qz, sc = awq_quantize_dense(w)
    sc = sc.bfloat16()
    dense = dequantize_awq_gemm(qw, qz, sc, group_size=128).float()          # [K, N]
    packed = awq_ops.prepare_awq_weights(qw.to(DEV), qz.to(DEV), sc.to(DEV), 128)
    x = torch.randn(T, K, generator=g).bfloat16()
    ref = x.float() @ dense
    out = awq_ops.awq_linear(x.to(DEV), packed)
    torch.cuda.synchronize()
    assert out.shape == (T, N)
    assert rel_err(out.cpu(), ref) < 1e-2


def test_awq_engine_matches_reference_backend(tmp_path):
    """A random AutoAWQ checkpoint decoded greedily: the W4A16 kernel path and the reference
    dequantize+matmul backend produce the same tokens."""
    from llmserve_b200 import LLM, SamplingParams
    from llmserve_b200.engine.model_runner import GreedySampler
    from llmserve_b200.models.synthetic import TINY, write_awq_checkpoint
    path = write_awq_checkpoint(str(tmp_path / "awq"), dict(TINY, num_hidden_layers=2))
    prompts = [[5, 9, 13, 2, 7], [100, 3, 3, 8]]
    outs = []
    for backend in ("cuda", "reference"):
        llm = LLM(path, awq_backend=backend, enforce_eager=True, max_model_len=128, max_num_seqs=4,
                  gpu_memory_utilization=0.2)
        llm.model_runner.sampler = GreedySampler()
        res = llm.generate(prompts, SamplingParams(max_tokens=8, ignore_eos=True), use_tqdm=False)
        outs.append([r["token_ids"] for r in res])
        llm.exit()
        del llm
    assert outs[0] == outs[1]


@pytest.mark.parametrize("splits", [2, 4, 8])
def test_awq_partials_sum(splits):
    """Split-K fp32 partials of the W4A16 kernel (consumed by the fused QKV / add+RMSNorm reducers)."""
    from llmserve_b200.ops import gemm
    g = torch.Generator().manual_seed(splits)
    w = torch.randn(512, 2048, generator=g) * 0.05
    qw, qz, sc = awq_quantize_dense(w)
    sc = sc.bfloat16()
    dense = dequantize_awq_gemm(qw, qz, sc, group_size=128).float()
    packed = awq_ops.prepare_awq_weights(qw.to(DEV), qz.to(DEV), sc.to(DEV), 128)
    x = torch.randn(48, 2048, generator=g).bfloat16()
    parts = gemm.linear_partials(x.to(DEV), packed, splits)
    torch.cuda.synchronize()
    assert parts.shape == (splits, 48, 512)
    assert rel_err(parts.sum(0).cpu(), x.float() @ dense) < 1e-3


@pytest.mark.parametrize("T", [1, 7, 64, 100])
@pytest.mark.parametrize("splits", [2, 3, 8])
@pytest.mark.parametrize("N,K", [(512, 2048), (6144, 4096)])
def test_awq_cluster_reduced_matches_dequantized_fp32(T, splits, N, K):
    """The W4A16 GEMM whose K-split CTAs reduce in a thread-block cluster (bf16 out, no partial
    planes) against the fp32 product of the dequantised weight, for several split counts."""
    from llmserve_b200.ops._ext import C, status
    g = torch.Generator().manual_seed(T * 7 + splits + N)
    w = torch.randn(N, K, generator=g) * 0.05
    qw, qz, sc = awq_quantize_dense(w)
    sc = sc.bfloat16()
    dense = dequantize_awq_gemm(qw, qz, sc, group_size=128).float()
    packed = awq_ops.prepare_awq_weights(qw.to(DEV), qz.to(DEV), sc.to(DEV), 128)
    x = torch.randn(T, K, generator=g).bfloat16()
    ref = x.float() @ dense
    out = torch.empty(T, N, dtype=torch.bfloat16, device=DEV)
    for _ in range(2):
        C().awq_gemm_reduced(out, x.to(DEV), packed.qtiles, packed.sztiles, N, splits, status(torch.device(DEV)))
        torch.cuda.synchronize()
        assert rel_err(out.cpu(), ref) < 1e-2
