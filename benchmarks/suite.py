"""Suite expansion, resume check, summary rows and aggregates (``benchmarks/suite.py`` of the
reference).  The point-id format, the ``workload_seed = arrival_seed = run`` rule and the CSV
column set are part of the result format and are kept."""
import json
from copy import deepcopy
from pathlib import Path
from statistics import mean, stdev


def _rate_label(rate: float) -> str:
    return str(rate).replace(".", "p")


def _dimension(experiment: dict):
    kind = experiment["arrival"]
    if kind == "poisson":
        return [("request_rate", v, f"rate-{_rate_label(v)}") for v in experiment["request_rates"]]
    if kind == "closed-loop":
        return [("max_concurrency", v, f"concurrency-{v}") for v in experiment["max_concurrencies"]]
    raise ValueError(f"unsupported arrival: {kind}")


def expand_suite(suite: dict) -> list[dict]:
    if suite.get("schema_version") != 1:
        raise ValueError("unsupported suite schema_version")
    runs = suite.get("runs", 0)
    if runs <= 0:
        raise ValueError("suite runs must be positive")
    profiles = suite.get("profiles", {})
    points = []
    for exp in suite.get("experiments", []):
        if exp["profile"] not in profiles:
            raise ValueError(f"unknown profile: {exp['profile']}")
        base_runtime = deepcopy(exp.get("runtime", {}))
        base_runtime.setdefault("enable_chunked_prefill", False)
        for dim_name, dim_value, dim_label in _dimension(exp):
            for run in range(runs):
                for variant in exp["variants"]:
                    runtime = deepcopy(base_runtime)
                    runtime.update({k: v for k, v in variant.items() if k != "name"})
                    point = {
                        "point_id": f"{exp['name']}-{variant['name']}-{dim_label}-r{run + 1}",
                        "suite": suite["name"], "experiment": exp["name"], "arrival": exp["arrival"],
                        "variant": variant["name"], "run": run, "workload_seed": run, "arrival_seed": run,
                        "workload": deepcopy(profiles[exp["profile"]]), "runtime": runtime,
                        "slo_ms": deepcopy(exp.get("slo_ms")),
                        dim_name: dim_value,
                    }
                    if exp["arrival"] == "poisson":
                        point["num_requests"] = exp["num_requests"]
                    else:
                        point["warmup_seconds"] = exp["warmup_seconds"]
                        point["measurement_seconds"] = exp["measurement_seconds"]
                    points.append(point)
    if len({p["point_id"] for p in points}) != len(points):
        raise ValueError("suite expands to duplicate point_id values")
    return points


def can_resume_result(path: Path, point: dict, git_commit: str) -> bool:
    try:
        result = json.loads(Path(path).read_text())
    except (OSError, json.JSONDecodeError):
        return False
    return (result.get("schema_version") == 2 and result.get("complete") is True
            and result.get("point_id") == point["point_id"] and result.get("git_commit") == git_commit)


def _get(value, path: str):
    for part in path.split("."):
        value = value[part]
    return value


def _optional(value, path: str, scale: float = 1.0):
    try:
        v = _get(value, path)
    except (KeyError, TypeError):
        return None
    return v * scale if v is not None else None


_MS = 1000.0
SUMMARY_FIELDS = {
    "request_throughput_rps": ("metrics.throughput.requests_per_second", 1.0),
    "input_throughput_tps": ("metrics.throughput.input_tokens_per_second", 1.0),
    "output_throughput_tps": ("metrics.throughput.output_tokens_per_second", 1.0),
    "total_throughput_tps": ("metrics.throughput.total_tokens_per_second", 1.0),
    "ttft_p50_ms": ("metrics.latency.overall.ttft.p50", _MS),
    "ttft_p99_ms": ("metrics.latency.overall.ttft.p99", _MS),
    "tpot_p50_ms": ("metrics.latency.overall.tpot.p50", _MS),
    "tpot_p99_ms": ("metrics.latency.overall.tpot.p99", _MS),
    "burst_itl_p50_ms": ("metrics.latency.overall.burst_itl.p50", _MS),
    "burst_itl_p99_ms": ("metrics.latency.overall.burst_itl.p99", _MS),
    "output_event_latency_p50_ms": ("metrics.latency.overall.output_event_latency.p50", _MS),
    "output_event_latency_p99_ms": ("metrics.latency.overall.output_event_latency.p99", _MS),
    "speculative_step_latency_p50_ms": ("metrics.latency.overall.speculative_step_latency.p50", _MS),
    "speculative_step_latency_p99_ms": ("metrics.latency.overall.speculative_step_latency.p99", _MS),
    "e2e_p50_ms": ("metrics.latency.overall.e2e.p50", _MS),
    "e2e_p99_ms": ("metrics.latency.overall.e2e.p99", _MS),
    "acceptance_rate": ("metrics.speculative.acceptance_rate", 1.0),
    "acceptance_length": ("metrics.speculative.acceptance_length", 1.0),
    "scheduled_batch_size_mean": ("metrics.scheduled_batch_size.mean", 1.0),
    "waiting_queue_size_p99": ("metrics.waiting_queue_size.p99", 1.0),
    "running_queue_size_p99": ("metrics.running_queue_size.p99", 1.0),
    "goodput_rps": ("metrics.goodput.requests_per_second", 1.0),
    "speculative_batch_size_mean": ("metrics.speculative_batch_size.mean", 1.0),
    "kv_total_blocks": ("metrics.kv_cache.total_blocks", 1.0),
    "kv_peak_reserved_blocks": ("metrics.kv_cache.peak_reserved_blocks", 1.0),
    "kv_preemptions": ("metrics.kv_cache.preemptions", 1.0),
    "kv_admission_deferrals": ("metrics.kv_cache.admission_deferrals", 1.0),
    "kv_cache_gib": ("metrics.kv_cache.kv_cache_bytes", 1.0 / 2**30),
    "model_runtime_gib": ("metrics.kv_cache.model_runtime_bytes", 1.0 / 2**30),
}
for _cls in ("short", "long"):
    for _name in ("ttft", "tpot", "e2e"):
        for _p in ("p50", "p99"):
            SUMMARY_FIELDS[f"{_cls}_{_name}_{_p}_ms"] = (f"metrics.latency.{_cls}.{_name}.{_p}", _MS)


def build_summary_rows(results: list[dict]) -> list[dict]:
    rows = []
    for result in results:
        cfg = result.get("config", {})
        row = {
            "point_id": result.get("point_id"), "complete": result.get("complete", False),
            "git_commit": result.get("git_commit"), "experiment": cfg.get("experiment"),
            "arrival": cfg.get("arrival"), "variant": cfg.get("variant"), "run": cfg.get("run"),
            "request_rate": cfg.get("request_rate"), "max_concurrency": cfg.get("max_concurrency"),
            "completed": _optional(result, "metrics.completed"), "failed": _optional(result, "metrics.failed"),
            "latency_sample_requests": _optional(result, "metrics.latency_sample_requests"),
        }
        row.update({name: _optional(result, path, scale) for name, (path, scale) in SUMMARY_FIELDS.items()})
        rows.append(row)
    return rows


def aggregate_results(results: list[dict], metric_path: str, *, scale: float = 1.0, unit: str | None = None):
    groups: dict[tuple, list[float]] = {}
    for result in results:
        if not result.get("complete"):
            continue
        cfg = result["config"]
        key = (cfg["experiment"], cfg["arrival"], cfg.get("request_rate"), cfg.get("max_concurrency"), cfg["variant"])
        try:
            value = float(_get(result, metric_path))
        except (KeyError, TypeError, ValueError):
            continue
        groups.setdefault(key, []).append(value * scale)
    baselines = {k[:4]: mean(v) for k, v in groups.items() if k[4] == "baseline"}
    rows = []
    for key in sorted(groups, key=lambda k: tuple(str(x) for x in k)):
        exp, arrival, rate, conc, variant = key
        vals = groups[key]
        base = baselines.get(key[:4])
        m = mean(vals)
        rows.append({"experiment": exp, "arrival": arrival, "request_rate": rate, "max_concurrency": conc,
                     "variant": variant, "metric": metric_path, "unit": unit, "runs": len(vals), "mean": m,
                     "stddev": stdev(vals) if len(vals) > 1 else 0.0,
                     "ratio_to_baseline": m / base if base not in (None, 0) else None})
    return rows
