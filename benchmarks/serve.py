"""Run one benchmark point in-process (``benchmarks/serve.py`` of the reference).

Builds the engine from the point's ``runtime`` block, optionally swaps in the argmax sampler,
runs a Poisson or closed-loop experiment and writes a schema-v2 result JSON (paths redacted to
basenames).  Runtime keys beyond the reference's: ``tensor_parallel_size``, ``load_format``,
``fused_collectives``, ``kvcache_block_size``, ``enable_kv_capacity_admission`` (already there),
``prompt_id_high`` (in the workload profile).
"""
import argparse
import json
import os
import sys
import time
from copy import deepcopy
from pathlib import Path
from random import Random

from benchmarks.arrivals import poisson_arrival_times
from benchmarks.environment import atomic_write_json, build_environment_metadata, discover_model_revision
from benchmarks.metrics import summarize_serving_run, summarize_speculative_requests, summarize_values
from benchmarks.runtime import run_closed_loop, run_poisson
from benchmarks.schema import compact_request_record
from benchmarks.workloads import (DEFAULT_PROMPT_ID_HIGH, RequestSpec, WorkloadClass, build_request_specs,
                                  iter_request_specs)


class ArgmaxSampler:
    """Greedy sampler used by the benchmarks (vocab-parallel on the tensor-parallel engine)."""
    is_greedy = True

    def __call__(self, logits, temperatures):
        return logits.argmax(dim=-1)


def _default_engine_factory(model, **kwargs):
    from llmserve_b200 import LLM
    return LLM(model, **kwargs)


def _default_sampling_params(spec):
    from llmserve_b200 import SamplingParams
    return SamplingParams(temperature=0.01, max_tokens=spec.output_len, ignore_eos=True)


def _classes(point):
    return [WorkloadClass(**c) for c in point["workload"]["classes"]]


def _prompt_id_high(point):
    return point["workload"].get("prompt_id_high", DEFAULT_PROMPT_ID_HIGH)


def _warmup_engine(engine, classes, make_sampling_params, prompt_id_high=DEFAULT_PROMPT_ID_HIGH):
    rng = Random(0)
    for i, c in enumerate(classes):
        spec = RequestSpec(-(i + 1), c.name, c.input_len, min(c.output_len, 8),
                           tuple(rng.randint(0, prompt_id_high) for _ in range(c.input_len)))
        engine.add_request(list(spec.prompt_token_ids), make_sampling_params(spec))
    while not engine.is_finished():
        engine.step()
    engine.reset_metrics()


def _closed_loop_metrics(obs: dict, slo_ms):
    metrics = summarize_serving_run(obs["latency_requests"], obs["duration"], slo_ms=slo_ms)
    done = [r for r in obs["requests"] if r["finish_time"] is not None
            and obs["measurement_start"] <= r["finish_time"] < obs["measurement_end"]]
    n_in = sum(r["prompt_tokens"] for r in done)
    d = obs["duration"]
    metrics["completed"] = obs["window_completed"]
    metrics["latency_sample_requests"] = len(obs["latency_requests"])
    metrics["failed"] = sum(not r["success"] for r in done)
    metrics["throughput"] = {
        "requests_per_second": obs["window_completed"] / d, "input_tokens_per_second": n_in / d,
        "output_tokens_per_second": obs["window_output_tokens"] / d,
        "total_tokens_per_second": (n_in + obs["window_output_tokens"]) / d,
    }
    return metrics


ENGINE_KEYS = {
    # key: default
    "enforce_eager": True, "awq_backend": "cuda", "enable_chunked_prefill": False,
    "enable_kv_capacity_admission": False, "max_num_seqs": 512, "gpu_memory_utilization": 0.9,
    "speculative_gamma": 3, "speculative_tree_nodes": 0, "speculative_accept_mode": "greedy",
    "speculative_trace": False, "tensor_parallel_size": 1, "load_format": "auto", "fused_collectives": True,
    "kvcache_block_size": 256, "overlap_decode": True, "pd_disaggregation": False, "pd_prefill_devices": (),
    "pd_decode_devices": (), "speculative_cuda_graphs": False, "device": "cuda", "num_kvcache_blocks": -1,
}


def run_point(point: dict, model: str, speculative_model: str | None = None,
              distributed_init_method: str | None = None, *, engine_factory=None, make_sampling_params=None,
              clock=time.perf_counter, sleep=time.sleep, metadata: dict | None = None,
              model_revision: str | None = None, speculative_model_revision: str | None = None):
    runtime = point["runtime"]
    speculative = runtime.get("enable_speculative", False)
    if speculative and not speculative_model:
        raise ValueError("speculative_model is required for speculative variants")
    engine_factory = engine_factory or _default_engine_factory
    make_sampling_params = make_sampling_params or _default_sampling_params
    active_draft = speculative_model if speculative else None
    kwargs = {k: runtime.get(k, v) for k, v in ENGINE_KEYS.items()}
    kwargs.update(max_model_len=runtime["max_model_len"], max_num_batched_tokens=runtime["max_num_batched_tokens"],
                  speculative_model=active_draft)
    if distributed_init_method is not None:
        kwargs["distributed_init_method"] = distributed_init_method
    engine = engine_factory(model, **kwargs)
    if runtime.get("argmax_sampler", False):
        engine.model_runner.sampler = ArgmaxSampler()
    classes = _classes(point)
    hi = _prompt_id_high(point)
    try:
        if point["arrival"] == "poisson":
            if runtime.get("warmup", False):
                _warmup_engine(engine, classes, make_sampling_params, hi)
            specs = build_request_specs(classes, point["num_requests"], point["workload_seed"], prompt_id_high=hi)
            arrivals = poisson_arrival_times(point["num_requests"], point["request_rate"], point["arrival_seed"])
            obs = run_poisson(engine, specs, arrivals, make_sampling_params, clock=clock, sleep=sleep)
            metrics = summarize_serving_run(obs["requests"], obs["duration"], slo_ms=point.get("slo_ms"))
            metrics["offered_request_rate"] = point["request_rate"]
            metric_requests = obs["requests"]
        elif point["arrival"] == "closed-loop":
            obs = run_closed_loop(engine, iter_request_specs(classes, point["workload_seed"], prompt_id_high=hi),
                                  point["max_concurrency"], point["warmup_seconds"], point["measurement_seconds"],
                                  make_sampling_params, clock=clock)
            metrics = _closed_loop_metrics(obs, point.get("slo_ms"))
            metrics["max_concurrency"] = point["max_concurrency"]
            metric_requests = obs["latency_requests"]
        else:
            raise ValueError(f"unsupported arrival: {point['arrival']}")
    finally:
        if hasattr(engine, "exit"):
            engine.exit()
    metrics["scheduled_batch_size"] = summarize_values(obs["scheduled_batch_sizes"])
    metrics["speculative_batch_size"] = summarize_values(obs["speculative_batch_sizes"])
    metrics["waiting_queue_size"] = summarize_values(obs["waiting_queue_sizes"])
    metrics["running_queue_size"] = summarize_values(obs["running_queue_sizes"])
    metrics["speculative"] = summarize_speculative_requests(metric_requests)
    spec_engine = obs["engine_summary"].get("speculative", {})
    for name in ("batch_calls", "mean_batch_size", "max_batch_size"):
        if name in spec_engine:
            metrics["speculative"][name] = spec_engine[name]
    metrics["kv_cache"] = obs["engine_summary"].get("kv_cache", {})
    public = deepcopy(point)
    public["model"] = Path(model).name
    public["model_revision"] = model_revision
    public["speculative_model"] = Path(active_draft).name if active_draft else None
    public["speculative_model_revision"] = speculative_model_revision if active_draft else None
    metadata = dict(metadata or {})
    return {
        "schema_version": 2, "complete": metrics["failed"] == 0, "point_id": point["point_id"],
        "git_commit": metadata.get("git_commit"), "metadata": metadata, "config": public, "metrics": metrics,
        "requests": [compact_request_record(r) for r in obs["requests"]],
    }


def _redact(message: str, paths) -> str:
    for p in paths:
        if p:
            message = message.replace(p, Path(p).name)
    return message


def failure_result(point: dict, metadata: dict, error: Exception, paths=()) -> dict:
    return {"schema_version": 2, "complete": False, "point_id": point.get("point_id"),
            "git_commit": metadata.get("git_commit"), "metadata": metadata, "config": deepcopy(point),
            "metrics": None, "requests": [],
            "error": {"type": type(error).__name__, "message": _redact(str(error), paths)}}


_failure_result = failure_result


def _parse_args(argv=None):
    p = argparse.ArgumentParser(description="Run one in-process llmserve_b200 benchmark point")
    p.add_argument("--point-config", required=True)
    p.add_argument("--model", required=True)
    p.add_argument("--speculative-model")
    p.add_argument("--model-revision")
    p.add_argument("--speculative-model-revision")
    p.add_argument("--expected-git-commit")
    p.add_argument("--distributed-init-method", default="tcp://127.0.0.1:2333")
    p.add_argument("--output", required=True)
    return p.parse_args(argv)


def main(argv=None):
    args = _parse_args(argv)
    point = json.loads(Path(args.point_config).read_text())
    metadata = build_environment_metadata()
    out = Path(args.output)
    if args.expected_git_commit and metadata.get("git_commit") != args.expected_git_commit:
        atomic_write_json(out, failure_result(point, metadata, RuntimeError("worker git commit does not match suite manifest")))
        return 1
    model = os.path.expanduser(args.model)
    draft = os.path.expanduser(args.speculative_model) if args.speculative_model else None
    try:
        result = run_point(point, model=model, speculative_model=draft,
                           distributed_init_method=args.distributed_init_method, metadata=metadata,
                           model_revision=args.model_revision or discover_model_revision(model),
                           speculative_model_revision=(args.speculative_model_revision
                                                       or discover_model_revision(draft) if draft else None))
    except Exception as e:
        atomic_write_json(out, failure_result(point, metadata, e, (model, draft)))
        print(f"FAILED {point.get('point_id')}: {e}", file=sys.stderr)
        return 1
    atomic_write_json(out, result)
    print(f"PASS {point['point_id']}: {result['metrics']['throughput']['output_tokens_per_second']:.3f} output tok/s")
    return 0 if result["complete"] else 1


if __name__ == "__main__":
    raise SystemExit(main())
