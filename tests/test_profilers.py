"""Linear microprofilers (``benchmarks.linear_profile``, ``benchmarks.awq_linear_profile``): shape
tables, summaries and checkpoint loading on CPU (reference tests ``tests/test_linear_profile.py``,
``tests/test_awq_linear_profile.py``); one timed measurement of each on the GPU."""
from types import SimpleNamespace

import pytest
import torch

from benchmarks import awq_linear_profile as awqp
from benchmarks import linear_profile as lp
from llmserve_b200.models.synthetic import QWEN3_8B, TINY, write_awq_checkpoint


def test_projection_shapes_and_tp_sharding():
    cfg = SimpleNamespace(**QWEN3_8B)
    s1 = {s.name: (s.input_size, s.output_size) for s in lp.qwen3_projection_shapes(cfg)}
    assert s1 == {"qkv": (4096, 6144), "o": (4096, 4096), "gate_up": (4096, 24576), "down": (12288, 4096)}
    s8 = {s.name: (s.input_size, s.output_size) for s in lp.qwen3_projection_shapes(cfg, tp=8)}
    assert s8 == {"qkv": (4096, 768), "o": (512, 4096), "gate_up": (4096, 3072), "down": (1536, 4096)}
    with pytest.raises(ValueError):
        lp.qwen3_projection_shapes(cfg, tp=3)


def test_summary_and_token_parsing():
    s = lp.summarize_latencies({"qkv": 1.0, "o": 1.0, "gate_up": 2.0, "down": 4.0}, num_hidden_layers=36)
    assert s["per_layer_total_ms"] == 8.0 and s["model_projection_total_ms"] == 288.0
    assert s["share_pct"]["down"] == 50.0
    assert lp.parse_num_tokens("1, 4,64") == (1, 4, 64)
    for bad in ("1,1", "0", "a"):
        with pytest.raises(ValueError):
            lp.parse_num_tokens(bad)
    rows = lp.profile_projection_shapes(lp.qwen3_projection_shapes(SimpleNamespace(**QWEN3_8B)), num_hidden_layers=2,
                                        num_tokens=(1, 8), measure_latency=lambda s, t: {"ms": t * 0.1, "gbps": 1})
    assert [r["num_tokens"] for r in rows] == [1, 8] and rows[1]["detail"]["qkv"] == {"gbps": 1}


def test_awq_layer_loading_merges_projections(tmp_path):
    path = write_awq_checkpoint(str(tmp_path / "awq"), TINY)
    projs = awqp.load_layer_projections(path, layer_id=1)
    assert [p.name for p in projs] == list(lp.PROJECTION_NAMES)
    q = TINY["num_attention_heads"] * TINY["head_dim"]
    kv = TINY["num_key_value_heads"] * TINY["head_dim"]
    assert (projs[0].input_size, projs[0].output_size) == (256, q + 2 * kv)
    assert (projs[3].input_size, projs[3].output_size) == (512, 256)
    rnd = awqp.random_layer_projections(QWEN3_8B)
    assert rnd[2].output_size == 24576 and rnd[2].qweight.dtype == torch.int32
    meas = {n: {s: 1.0 for s in awqp.STAGES} for n in lp.PROJECTION_NAMES}
    summ = awqp.summarize_stage_latencies(meas, num_hidden_layers=36)
    assert summ["per_layer_ms"]["cuda"] == 4.0 and summ["cuda_speedup_vs_reference"] == 1.0


@pytest.mark.gpu
def test_profilers_measure_on_gpu():
    dev = torch.device("cuda")
    m = lp.measure_dense_cuda(lp.LinearShape("o", 4096, 4096), num_tokens=16, device=dev, warmup=2, repeats=5,
                              hbm_gbs=6553.0)
    assert m["ms"] > 0 and m["cublas_ms"] > 0 and 0 < m["fraction_of_measured_hbm"] < 2
    p = awqp.random_layer_projections(dict(QWEN3_8B, hidden_size=1024, intermediate_size=2048,
                                           num_attention_heads=8, num_key_value_heads=2))[1]
    r = awqp.measure_projection_cuda(p, num_tokens=8, group_size=128, device=dev, warmup=2, repeats=5)
    assert all(r[s] > 0 for s in awqp.STAGES)


def test_step_timeline_exclusive_time_and_gaps():
    from benchmarks.step_timeline import exclusive_times, short_name
    rows = [("a", 0.0, 10.0), ("b", 5.0, 12.0), ("a", 20.0, 25.0), ("c", 21.0, 23.0)]
    excl, cnt, idle = exclusive_times(rows)
    assert excl == {"a": 15.0, "b": 2.0, "c": 0.0} and cnt["a"] == 2 and idle == 8.0
    assert short_name("void lsb::(anonymous namespace)::gemm_bf16_kernel<64, 4, 0>(CUtensorMap_st, int)") == \
        "gemm_bf16_kernel<64, 4, 0>"


def test_fused_collective_roofline_terms():
    from benchmarks.collective_profile import fused_roofline_us
    r = fused_roofline_us(T=64, hidden=4096, inner_shard=512, world=8, planes=1, hbm_gbs=6553.0, bf16_tflops=1655.0)
    # weights 4096 x 512 bf16 = 4 MiB at 6553 GB/s; NVLink, 8-byte words: 56 other rows' partials
    # to their owners + this rank's 8 rows to 7 peers
    assert r["weight_bytes"] == 4096 * 512 * 2 and r["nvlink_bytes"] == 56 * 4096 * 8 + 7 * 8 * 4096 * 8
    assert abs(r["hbm_us"] - 4096 * 512 * 2 / 6553e3) < 1e-9
    assert r["roofline_us"] == max(r["hbm_us"], r["compute_us"], r["nvlink_us"])


def test_attention_profile_counts_causal_work_only():
    from benchmarks.attention_profile import causal_flops
    # 3 query rows over 3 keys: 1 + 2 + 3 key visits; a 2-row chunk after a 4-key prefix: 5 + 6
    assert causal_flops([(3, 3)], heads=2, head_dim=8) == 4 * 8 * 2 * 6
    assert causal_flops([(2, 6)], heads=1, head_dim=128) == 4 * 128 * 11
