"""Benchmark harness with a fake clock and a fake engine (no model), plus metric parity with the
reference harness where it is importable."""
import json
import random
from types import SimpleNamespace

import pytest

from benchmarks.arrivals import poisson_arrival_times
from benchmarks.metrics import percentile, summarize_serving_run, summarize_values
from benchmarks.run_suite import execute_suite
from benchmarks.runtime import run_closed_loop, run_poisson
from benchmarks.schema import compact_request_record
from benchmarks.serve import run_point
from benchmarks.suite import aggregate_results, build_summary_rows, expand_suite
from benchmarks.workloads import WorkloadClass, build_request_specs, class_counts, iter_request_specs
from tests.support import reference_module


class FakeClock:
    def __init__(self):
        self.t = 100.0

    def __call__(self):
        return self.t

    def sleep(self, dt):
        self.t += max(dt, 1e-6)   # a real sleep always lets time pass


class FakeEngine:
    """Emits one token per request per step; each step takes 10 ms of fake time."""

    def __init__(self, clock, step_s=0.01):
        self.clock, self.step_s = clock, step_s
        self.reqs = {}
        self.next_id = 0
        self.last_step_events = {}
        self.model_runner = SimpleNamespace(sampler=None)

    def add_request(self, prompt, sp):
        sid = self.next_id
        self.next_id += 1
        self.reqs[sid] = dict(seq_id=sid, prompt_tokens=len(prompt), output_tokens=0, target=sp.max_tokens,
                              arrival_time=self.clock(), first_token_time=None, token_times=[], output_event_times=[],
                              finish_time=None, success=False, failure_reason=None)
        return sid

    def is_finished(self):
        return all(r["finish_time"] is not None for r in self.reqs.values())

    def step(self):
        self.clock.t += self.step_s
        now = self.clock()
        done = []
        ids = [i for i, r in self.reqs.items() if r["finish_time"] is None]
        for i in ids:
            r = self.reqs[i]
            r["output_tokens"] += 1
            r["token_times"].append(now)
            r["output_event_times"].append(now)
            r["first_token_time"] = r["first_token_time"] or now
            if r["output_tokens"] == r["target"]:
                r["finish_time"], r["success"] = now, True
                done.append((i, [0] * r["output_tokens"]))
        self.last_step_events = {"step_end": now, "scheduled_seq_ids": ids, "waiting_queue_size": 0,
                                 "running_queue_size": len(ids)}
        return done, len(ids)

    def get_metrics(self):
        return {"summary": {"kv_cache": {"total_blocks": 10}}, "requests": [dict(r) for r in self.reqs.values()]}

    def reset_metrics(self):
        self.reqs.clear()

    def exit(self):
        pass


def _sp(spec):
    return SimpleNamespace(max_tokens=spec.output_len)


def test_class_counts_largest_remainder_and_specs():
    classes = [WorkloadClass("short", 0.8, 4, 2), WorkloadClass("long", 0.2, 8, 2)]
    assert class_counts(classes, 7) == [6, 1]
    specs = build_request_specs(classes, 10, seed=3)
    assert [s.request_id for s in specs] == list(range(10))
    assert sum(s.request_class == "long" for s in specs) == 2
    assert build_request_specs(classes, 10, seed=3) == specs
    it = iter_request_specs(classes, seed=0, cycle_size=5)
    assert [next(it).request_id for _ in range(12)] == list(range(12))


def test_workloads_and_arrivals_match_reference():
    ref = _ref_bench("workloads")
    ref_a = _ref_bench("arrivals")
    classes = [WorkloadClass("a", 1, 5, 3), WorkloadClass("b", 2, 7, 1)]
    rclasses = [ref.WorkloadClass("a", 1, 5, 3), ref.WorkloadClass("b", 2, 7, 1)]
    ours = build_request_specs(classes, 13, seed=5)
    theirs = ref.build_request_specs(rclasses, 13, seed=5)
    assert [(s.request_class, s.prompt_token_ids) for s in ours] == [(s.request_class, s.prompt_token_ids) for s in theirs]
    assert poisson_arrival_times(9, 1.5, 2) == ref_a.poisson_arrival_times(9, 1.5, 2)


def _ref_bench(name):
    import importlib
    import sys
    reference_module("llmserve.sampling_params")   # puts the reference root on sys.path (or skips)
    saved = {k: sys.modules.pop(k) for k in list(sys.modules) if k == "benchmarks" or k.startswith("benchmarks.")}
    root = [p for p in sys.path if p.endswith("reference") or p.endswith("_ref")][0]
    sys.path.insert(0, root)
    try:
        return importlib.import_module(f"benchmarks.{name}")
    finally:
        sys.path.remove(root)
        for k in list(sys.modules):
            if k == "benchmarks" or k.startswith("benchmarks."):
                sys.modules.pop(k)
        sys.modules.update(saved)


def test_percentiles_match_reference():
    ref = _ref_bench("metrics")
    rng = random.Random(0)
    vals = [rng.random() for _ in range(37)]
    for q in (0, 50, 90, 99, 100):
        assert percentile(vals, q) == pytest.approx(ref.percentile(vals, q))
    assert summarize_values(vals) == ref.summarize_values(vals)


def test_closed_loop_window_rules():
    clock = FakeClock()
    eng = FakeEngine(clock)
    classes = [WorkloadClass("decode", 1, 4, 5)]
    obs = run_closed_loop(eng, iter_request_specs(classes, 0), max_concurrency=3, warmup_seconds=0.05,
                          measurement_seconds=0.2, make_sampling_params=_sp, clock=clock)
    assert obs["duration"] == 0.2
    for r in obs["latency_requests"]:
        assert r["arrival_time"] >= obs["measurement_start"] and r["finish_time"] < obs["measurement_end"]
    assert obs["window_output_tokens"] > 0 and eng.is_finished()
    metrics = summarize_serving_run(obs["latency_requests"], obs["duration"])
    assert metrics["latency"]["overall"]["tpot"]["p50"] == pytest.approx(0.01)


def test_poisson_run_admits_by_arrival_and_sleeps():
    clock = FakeClock()
    eng = FakeEngine(clock)
    specs = build_request_specs([WorkloadClass("d", 1, 3, 2)], 4, seed=1)
    arrivals = [0.0, 0.5, 0.5, 2.0]
    obs = run_poisson(eng, specs, arrivals, _sp, clock=clock, sleep=clock.sleep)
    assert obs["admitted"] == 4
    assert [r["request_id"] for r in obs["requests"]] == [0, 1, 2, 3]
    assert obs["duration"] >= 2.0


def test_run_point_and_schema_with_fake_engine():
    clock = FakeClock()
    suite = json.load(open("benchmarks/suites/smoke.json"))
    point = expand_suite(suite)[0]
    result = run_point(point, "/models/tiny", speculative_model="/models/draft",
                       engine_factory=lambda m, **kw: FakeEngine(clock), make_sampling_params=_sp, clock=clock,
                       sleep=clock.sleep, metadata={"git_commit": "abc"})
    assert result["schema_version"] == 2 and result["complete"]
    assert result["config"]["model"] == "tiny"
    assert set(result["requests"][0]) >= {"ttft_ms", "tpot_ms", "e2e_ms", "burst_itl_ms", "speculative"}
    rows = build_summary_rows([result])
    assert rows[0]["output_throughput_tps"] > 0


def test_suite_expansion_ids_and_aggregate():
    suite = json.load(open("benchmarks/suites/formal-closed-loop.json"))
    pts = expand_suite(suite)
    assert pts[0]["point_id"] == "eagle-closed-loop-baseline-concurrency-1-r1"
    assert {p["workload_seed"] for p in pts} == {0, 1, 2}
    res = [{"complete": True, "config": p, "metrics": {"x": {"y": float(i)}}} for i, p in enumerate(pts[:4])]
    rows = aggregate_results(res, "metrics.x.y")
    assert any(r["ratio_to_baseline"] is not None for r in rows)


def test_suite_expansion_matches_reference():
    ref = _ref_bench("suite")
    import os
    ref_suites = os.path.join(os.path.dirname(os.path.dirname(ref.__file__)), "benchmarks", "suites")
    for name in ("smoke", "formal-closed-loop", "formal-poisson", "pilot", "awq-capacity-confirm"):
        suite = json.load(open(f"benchmarks/suites/{name}.json"))
        assert expand_suite(suite) == ref.expand_suite(suite)
        # the experiment definitions behind the published numbers are the same
        if name != "smoke" and os.path.exists(os.path.join(ref_suites, f"{name}.json")):
            with open(os.path.join(ref_suites, f"{name}.json")) as f:
                assert json.load(f) == suite, name


def test_execute_suite_records_failures_and_continues(tmp_path):
    suite = json.load(open("benchmarks/suites/smoke.json"))
    calls = []

    def runner(cmd, **kw):
        calls.append(cmd)
        return SimpleNamespace(returncode=1, stderr="boom /secret/model/path")

    rc = execute_suite(suite, tmp_path, "/secret/model/path", None, {"git_commit": "c0"}, command_runner=runner)
    assert rc == 1 and len(calls) == 4
    manifest = json.loads((tmp_path / "manifest.json").read_text())
    assert manifest["failed_points"] == 4
    run = json.loads(next((tmp_path / "runs").iterdir()).read_text())
    assert "/secret" not in run["error"]["message"] and run["complete"] is False
    assert (tmp_path / "summary.csv").exists()


def test_compact_record_units():
    rec = compact_request_record(dict(seq_id=1, request_class="d", arrival_time=1.0, first_token_time=1.5,
                                      finish_time=2.5, output_tokens=3, prompt_tokens=4, success=True,
                                      token_times=[1.5, 2.0, 2.5], output_event_times=[1.5, 2.5]))
    assert rec["ttft_ms"] == 500 and rec["tpot_ms"] == 500 and rec["e2e_ms"] == 1500


def test_run_point_with_real_cpu_engines_plain_and_disaggregated(tmp_path):
    """A closed-loop point through benchmarks.serve with the engine itself (CPU tier): the plain
    engine and the prefill/decode-disaggregated variant both complete and emit tokens."""
    from llmserve_b200 import LLM
    from llmserve_b200.models.synthetic import TINY, write_qwen3_checkpoint
    path = write_qwen3_checkpoint(str(tmp_path / "m"), TINY)
    suite = {"schema_version": 1, "name": "cpu-pd", "runs": 1,
             "profiles": {"p": {"classes": [{"name": "c", "weight": 1, "input_len": 24, "output_len": 12}],
                                "prompt_id_high": 1000}},
             "experiments": [{"name": "e", "arrival": "closed-loop", "profile": "p", "max_concurrencies": [3],
                              "warmup_seconds": 0.2, "measurement_seconds": 1.0,
                              "variants": [{"name": "baseline"},
                                           {"name": "pd", "pd_disaggregation": True, "pd_prefill_devices": [0],
                                            "pd_decode_devices": [0]}],
                              "runtime": {"argmax_sampler": True, "max_model_len": 128,
                                          "max_num_batched_tokens": 256, "kvcache_block_size": 16}}]}

    def factory(model, **kw):
        return LLM(model, **dict(kw, device="cpu", num_kvcache_blocks=64))

    for point in expand_suite(suite):
        result = run_point(point, path, engine_factory=factory, metadata={"git_commit": "abc"})
        assert result["complete"], point["variant"]
        assert result["metrics"]["throughput"]["output_tokens_per_second"] > 0


def test_b200_suite_pd_variant_reaches_the_engine_factory():
    """The disaggregated variant of the B200 suite passes its device split and the overlapped-loop
    default through ``run_point`` to the engine constructor."""
    suite = json.load(open("benchmarks/suites/b200-serving.json"))
    points = [p for p in expand_suite(suite) if p["experiment"] == "pd-closed-loop-1p1d"]
    assert {p["variant"] for p in points} == {"baseline", "pd"}
    seen = {}
    clock = FakeClock()

    def factory(model, **kw):
        seen[kw.get("pd_disaggregation")] = kw
        return FakeEngine(clock)

    for p in points[:2]:
        p = dict(p, warmup_seconds=0.05, measurement_seconds=0.1)
        run_point(p, "/models/tiny", engine_factory=factory, make_sampling_params=_sp, clock=clock, sleep=clock.sleep,
                  metadata={"git_commit": "abc"})
    assert seen[True]["pd_prefill_devices"] == [0] and seen[True]["pd_decode_devices"] == [1]
    assert seen[False]["overlap_decode"] is True and seen[False]["pd_disaggregation"] is False


def _point_result(point, commit, tps, complete=True):
    return {"schema_version": 2, "complete": complete, "point_id": point["point_id"], "git_commit": commit,
            "config": point, "metrics": {"throughput": {"output_tokens_per_second": tps}}}


def test_execute_suite_resume_start_failure_timeout_and_bad_exit(tmp_path):
    import subprocess

    from benchmarks.environment import atomic_write_json
    suite = json.load(open("benchmarks/suites/smoke.json"))
    points = expand_suite(suite)
    assert len(points) == 4
    runs = tmp_path / "runs"
    runs.mkdir()
    atomic_write_json(runs / f"{points[0]['point_id']}.json", _point_result(points[0], "c1", 10.0))   # resumable
    atomic_write_json(runs / f"{points[1]['point_id']}.json", _point_result(points[1], "c0", 11.0))   # old commit
    seen = []

    def runner(cmd, **kw):
        pid = next(p["point_id"] for p in points if p["point_id"] in cmd[cmd.index("--point-config") + 1])
        seen.append(pid)
        out = cmd[cmd.index("--output") + 1]
        if pid == points[1]["point_id"]:
            raise OSError("exec format error")
        if pid == points[2]["point_id"]:
            raise subprocess.TimeoutExpired(cmd, 5)
        point = next(p for p in points if p["point_id"] == pid)
        atomic_write_json(out, _point_result(point, "c1", 12.0))            # complete, but the worker failed
        return SimpleNamespace(returncode=3, stderr="late crash")

    rc = execute_suite(suite, tmp_path, "/m/model", None, {"git_commit": "c1"}, resume=True, timeout_seconds=5,
                       command_runner=runner)
    assert rc == 1
    assert seen == [p["point_id"] for p in points[1:]]                  # the matching result was resumed
    res = {p["point_id"]: json.loads((runs / f"{p['point_id']}.json").read_text()) for p in points}
    assert res[points[0]["point_id"]]["complete"] is True
    assert res[points[1]["point_id"]]["error"]["type"] == "WorkerStartError"
    assert "timed out" in res[points[2]["point_id"]]["error"]["message"]
    assert res[points[3]["point_id"]]["complete"] is False
    manifest = json.loads((tmp_path / "manifest.json").read_text())
    assert manifest["completed_points"] == 1 and manifest["failed_points"] == 3 and not manifest["complete"]


def test_summary_rows_and_aggregates_match_reference_on_sparse_results():
    ref = _ref_bench("suite")
    suite = json.load(open("benchmarks/suites/formal-closed-loop.json"))
    points = expand_suite(suite)[:6]
    results = []
    for i, p in enumerate(points):
        r = _point_result(p, "c", None if i == 2 else 100.0 + 7 * i, complete=i != 4)
        r["metrics"]["latency"] = {"overall": {"ttft": {"p50": 0.01 * i, "p99": 0.02 * i}}}
        if i == 1:
            r["metrics"]["speculative"] = {"acceptance_rate": 0.5, "acceptance_length": 2.5}
        results.append(r)
    assert build_summary_rows(results) == ref.build_summary_rows(results)
    for path, kw in (("metrics.throughput.output_tokens_per_second", {}),
                     ("metrics.latency.overall.ttft.p99", {"scale": 1000.0, "unit": "ms"})):
        assert aggregate_results(results, path, **kw) == ref.aggregate_results(results, path, **kw)


def test_expand_suite_rejects_unknown_profile_like_the_reference():
    ref = _ref_bench("suite")
    suite = json.load(open("benchmarks/suites/smoke.json"))
    suite["experiments"][0]["profile"] = "no-such-profile"
    with pytest.raises(Exception) as ours:
        expand_suite(suite)
    with pytest.raises(Exception) as theirs:
        ref.expand_suite(suite)
    assert type(ours.value) is type(theirs.value)


def test_run_point_result_equals_reference_with_the_same_fake_engine():
    """Poisson and closed-loop points through both harnesses with one fake engine and fake clock:
    the result documents (config, metrics, per-request records, KV summary) are identical."""
    ref = _ref_bench("serve")

    def run(fn, point):
        clock = FakeClock()
        return fn(point, "/models/tiny", speculative_model="/models/draft",
                  engine_factory=lambda m, **kw: FakeEngine(clock), make_sampling_params=_sp, clock=clock,
                  sleep=clock.sleep, metadata={"git_commit": "abc"})

    for name in ("smoke", "formal-closed-loop"):
        for point in expand_suite(json.load(open(f"benchmarks/suites/{name}.json")))[:3]:
            if point["arrival"] == "closed-loop":
                point = dict(point, warmup_seconds=0.05, measurement_seconds=0.5)
            ours, theirs = run(run_point, point), run(ref.run_point, point)
            ours.pop("environment", None)
            theirs.pop("environment", None)
            assert ours == theirs, point["point_id"]


def test_run_suite_command_line_end_to_end_on_the_host_tier(tmp_path):
    """``python -m benchmarks.run_suite`` exactly as a user runs it: one subprocess per point
    (``benchmarks.serve``), a real engine on the host tier, manifest and CSVs written."""
    import csv
    import os
    import subprocess
    import sys

    from llmserve_b200.models.synthetic import TINY, write_qwen3_checkpoint
    path = write_qwen3_checkpoint(str(tmp_path / "m"), TINY)
    suite = {"schema_version": 1, "name": "cpu-cli", "runs": 1,
             "profiles": {"p": {"classes": [{"name": "c", "weight": 1, "input_len": 20, "output_len": 8}],
                                "prompt_id_high": 1000}},
             "experiments": [{"name": "e", "arrival": "closed-loop", "profile": "p", "max_concurrencies": [2],
                              "warmup_seconds": 0.2, "measurement_seconds": 1.0,
                              "variants": [{"name": "baseline"}, {"name": "chunked", "enable_chunked_prefill": True}],
                              "runtime": {"argmax_sampler": True, "max_model_len": 128, "max_num_batched_tokens": 256,
                                          "kvcache_block_size": 16, "device": "cpu", "num_kvcache_blocks": 64}}]}
    (tmp_path / "suite.json").write_text(json.dumps(suite))
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    proc = subprocess.run([sys.executable, "-m", "benchmarks.run_suite", "--suite", str(tmp_path / "suite.json"),
                           "--output-dir", str(tmp_path / "out"), "--model", path, "--allow-dirty",
                           "--timeout-seconds", "300"], cwd=root, capture_output=True, text=True, timeout=600)
    assert proc.returncode == 0, proc.stdout[-2000:] + proc.stderr[-2000:]
    manifest = json.loads((tmp_path / "out" / "manifest.json").read_text())
    assert manifest["complete"] and manifest["completed_points"] == 2
    rows = list(csv.DictReader(open(tmp_path / "out" / "summary.csv")))
    assert len(rows) == 2 and all(float(r["output_throughput_tps"]) > 0 for r in rows)
    assert str(tmp_path) not in (tmp_path / "out" / "runs" / f"{rows[0]['point_id']}.json").read_text()


def test_b200_tp1_suite_expands_and_runs_with_a_fake_engine():
    """The one-GPU B200 suite (decode-heavy closed loop, EAGLE3 graphs, chunked prefill on the mixed
    profile, closed loop and Poisson) expands to its 16 points, each of which runs through
    ``run_point`` against a fake engine with the runtime knobs it names."""
    suite = json.load(open("benchmarks/suites/b200-serving-tp1.json"))
    points = expand_suite(suite)
    assert len(points) == 16 and len({p["point_id"] for p in points}) == 16
    assert {p["experiment"] for p in points} == {"bf16-closed-loop-tp1", "eagle-closed-loop-tp1",
                                                 "chunked-closed-loop-tp1", "chunked-poisson-tp1"}
    seen = []
    clock = FakeClock()

    def factory(model, **kw):
        seen.append(kw)
        return FakeEngine(clock)

    for p in points:
        p = dict(p, warmup_seconds=0.05, measurement_seconds=0.1)
        result = run_point(p, "/models/tiny", speculative_model="/models/eagle3", engine_factory=factory,
                           make_sampling_params=_sp, clock=clock, sleep=clock.sleep, metadata={"git_commit": "abc"})
        assert result["complete"], p["point_id"]
    assert all(kw["tensor_parallel_size"] == 1 for kw in seen)
    assert sum(bool(kw.get("enable_chunked_prefill")) for kw in seen) == 4
    assert sum(bool(kw.get("speculative_cuda_graphs")) for kw in seen) == 2


def test_b200_two_gpu_suite_expands_to_tp2_and_pd_points():
    """The two-GPU B200 suite: TP = 2 with the NCCL path and the fused collective at C = 1 / 64, and
    the 1P1D disaggregated variant beside its one-GPU baseline at C = 16."""
    suite = json.load(open("benchmarks/suites/b200-serving-2gpu.json"))
    points = expand_suite(suite)
    got = sorted((p["experiment"], p["variant"], p["max_concurrency"]) for p in points)
    assert got == sorted([("bf16-closed-loop-tp2", v, c) for v in ("baseline", "fused") for c in (1, 64)] +
                         [("pd-closed-loop-1p1d", v, 16) for v in ("baseline", "pd")])
    assert all(p["runtime"]["tensor_parallel_size"] == 2 for p in points if p["experiment"].endswith("tp2"))
