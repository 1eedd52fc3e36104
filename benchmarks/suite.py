"""Benchmark suites: expansion into points, the resume rule, per-point summary rows and
cross-run aggregates.

What is fixed by the result format (shared with the reference harness, ``benchmarks/suite.py``
there, so suites and result trees of both engines are interchangeable): suite schema v1, the
point id ``<experiment>-<variant>-<rate-R|concurrency-C>-r<run+1>`` with ``.`` written ``p`` in
rates, ``workload_seed = arrival_seed = run``, chunked prefill off unless a runtime turns it on,
the summary columns and their order, and the aggregate row keys with the ratio to the
``baseline`` variant.  The parsing and table construction here are this module's own.
"""
import itertools
import json
from copy import deepcopy
from pathlib import Path
from statistics import mean, stdev

SUITE_SCHEMA = 1
RESULT_SCHEMA = 2


def _axis(experiment: dict) -> list[tuple[str, object, str]]:
    """(point key, value, id label) for each value of the experiment's swept dimension."""
    arrival = experiment["arrival"]
    if arrival == "poisson":
        return [("request_rate", r, "rate-" + str(r).replace(".", "p")) for r in experiment["request_rates"]]
    if arrival == "closed-loop":
        return [("max_concurrency", c, f"concurrency-{c}") for c in experiment["max_concurrencies"]]
    raise ValueError(f"unsupported arrival: {arrival}")


def _check_suite(suite: dict) -> int:
    if suite.get("schema_version") != SUITE_SCHEMA:
        raise ValueError("unsupported suite schema_version")
    runs = suite.get("runs", 0)
    if runs <= 0:
        raise ValueError("suite runs must be positive")
    profiles = suite.get("profiles", {})
    for experiment in suite.get("experiments", []):
        if experiment["profile"] not in profiles:
            raise ValueError(f"unknown profile: {experiment['profile']}")
    return runs


def _window(experiment: dict) -> dict:
    """How long a point runs: a request count for Poisson arrivals, a timed window otherwise."""
    if experiment["arrival"] == "poisson":
        return {"num_requests": experiment["num_requests"]}
    return {"warmup_seconds": experiment["warmup_seconds"], "measurement_seconds": experiment["measurement_seconds"]}


def expand_suite(suite: dict) -> list[dict]:
    """Every point of the suite, in run order: experiment, swept value, run, variant."""
    runs = _check_suite(suite)
    points = []
    for experiment in suite.get("experiments", []):
        runtime_base = {"enable_chunked_prefill": False, **deepcopy(experiment.get("runtime", {}))}
        workload = suite["profiles"][experiment["profile"]]
        for (key, value, label), run, variant in itertools.product(_axis(experiment), range(runs),
                                                                   experiment["variants"]):
            overrides = {k: v for k, v in variant.items() if k != "name"}
            point = {
                "point_id": f"{experiment['name']}-{variant['name']}-{label}-r{run + 1}",
                "suite": suite["name"],
                "experiment": experiment["name"],
                "arrival": experiment["arrival"],
                "variant": variant["name"],
                "run": run,
                "workload_seed": run,
                "arrival_seed": run,
                "workload": deepcopy(workload),
                "runtime": {**deepcopy(runtime_base), **deepcopy(overrides)},
                "slo_ms": deepcopy(experiment.get("slo_ms")),
                key: value,
            }
            point.update(_window(experiment))
            points.append(point)
    ids = [p["point_id"] for p in points]
    if len(set(ids)) != len(ids):
        raise ValueError("suite expands to duplicate point_id values")
    return points


def can_resume_result(path: Path, point: dict, git_commit: str) -> bool:
    """A stored result may be kept on ``--resume`` when it is a complete v2 result of this point
    produced by the same commit."""
    try:
        stored = json.loads(Path(path).read_text())
    except (OSError, json.JSONDecodeError):
        return False
    expected = {"schema_version": RESULT_SCHEMA, "complete": True, "point_id": point["point_id"],
                "git_commit": git_commit}
    return all(stored.get(k) == v for k, v in expected.items())


def _lookup(doc, dotted: str):
    """Value at a dotted path, or None when any step is missing."""
    for part in dotted.split("."):
        if not isinstance(doc, dict) or part not in doc:
            return None
        doc = doc[part]
    return doc


def _summary_columns() -> list[tuple[str, str, float]]:
    """(column, result path, scale) in the format's column order."""
    ms, gib = 1000.0, 1.0 / (1 << 30)
    cols = [(f"{k}_throughput_{u}", f"metrics.throughput.{n}", 1.0) for k, n, u in (
        ("request", "requests_per_second", "rps"), ("input", "input_tokens_per_second", "tps"),
        ("output", "output_tokens_per_second", "tps"), ("total", "total_tokens_per_second", "tps"))]
    for name in ("ttft", "tpot", "burst_itl", "output_event_latency", "speculative_step_latency", "e2e"):
        cols += [(f"{name}_{p}_ms", f"metrics.latency.overall.{name}.{p}", ms) for p in ("p50", "p99")]
    cols += [("acceptance_rate", "metrics.speculative.acceptance_rate", 1.0),
             ("acceptance_length", "metrics.speculative.acceptance_length", 1.0),
             ("scheduled_batch_size_mean", "metrics.scheduled_batch_size.mean", 1.0),
             ("waiting_queue_size_p99", "metrics.waiting_queue_size.p99", 1.0),
             ("running_queue_size_p99", "metrics.running_queue_size.p99", 1.0),
             ("goodput_rps", "metrics.goodput.requests_per_second", 1.0),
             ("speculative_batch_size_mean", "metrics.speculative_batch_size.mean", 1.0)]
    cols += [(f"kv_{k}", f"metrics.kv_cache.{k}", 1.0)
             for k in ("total_blocks", "peak_reserved_blocks", "preemptions", "admission_deferrals")]
    cols += [("kv_cache_gib", "metrics.kv_cache.kv_cache_bytes", gib),
             ("model_runtime_gib", "metrics.kv_cache.model_runtime_bytes", gib)]
    for cls, name, p in itertools.product(("short", "long"), ("ttft", "tpot", "e2e"), ("p50", "p99")):
        cols.append((f"{cls}_{name}_{p}_ms", f"metrics.latency.{cls}.{name}.{p}", ms))
    return cols


SUMMARY_COLUMNS = _summary_columns()
_CONFIG_COLUMNS = ("experiment", "arrival", "variant", "run", "request_rate", "max_concurrency")


def build_summary_rows(results: list[dict]) -> list[dict]:
    """One row per point result (complete or not) with the headline metrics in the format's units."""
    rows = []
    for result in results:
        config = result.get("config", {})
        row = {"point_id": result.get("point_id"), "complete": result.get("complete", False),
               "git_commit": result.get("git_commit")}
        row.update({k: config.get(k) for k in _CONFIG_COLUMNS})
        for name in ("completed", "failed", "latency_sample_requests"):
            row[name] = _lookup(result, f"metrics.{name}")
        for column, path, scale in SUMMARY_COLUMNS:
            value = _lookup(result, path)
            row[column] = None if value is None else value * scale
        rows.append(row)
    return rows


def aggregate_results(results: list[dict], metric_path: str, *, scale: float = 1.0, unit: str | None = None):
    """Mean and sample standard deviation of one metric over the runs of each (experiment, arrival,
    rate, concurrency, variant), with the ratio to the ``baseline`` variant of the same point."""
    samples: dict[tuple, list[float]] = {}
    for result in results:
        if not result.get("complete"):
            continue
        config = result["config"]
        raw = _lookup(result, metric_path)
        try:
            value = float(raw)
        except (TypeError, ValueError):
            continue
        key = (config["experiment"], config["arrival"], config.get("request_rate"), config.get("max_concurrency"),
               config["variant"])
        samples.setdefault(key, []).append(value * scale)
    rows = []
    for key in sorted(samples, key=lambda k: tuple(map(str, k))):
        values = samples[key]
        avg = mean(values)
        base_values = samples.get(key[:4] + ("baseline",))
        base = mean(base_values) if base_values else None
        rows.append(dict(zip(("experiment", "arrival", "request_rate", "max_concurrency", "variant"), key),
                         metric=metric_path, unit=unit, runs=len(values), mean=avg,
                         stddev=stdev(values) if len(values) > 1 else 0.0,
                         ratio_to_baseline=avg / base if base else None))
    return rows
