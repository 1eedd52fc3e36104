"""Run a benchmark suite: one subprocess per point (``benchmarks/run_suite.py`` of the reference).

Points are expanded from the suite JSON, each is run by ``python -m benchmarks.serve`` in its
own process with an optional timeout; a failed or timed-out point becomes a ``complete: false``
result and the suite continues.  ``--resume`` skips points whose result is complete and was made
at the same commit.  Writes ``runs/*.json``, ``summary.csv``, ``aggregate.csv`` (mean, sample
stddev, ratio to the "baseline" variant) and ``manifest.json``.  A dirty work tree is refused
unless ``--allow-dirty``.
"""
import argparse
import csv
import json
import os
import subprocess
import sys
from pathlib import Path
from types import SimpleNamespace

from benchmarks.environment import atomic_write_json, build_environment_metadata, discover_model_revision
from benchmarks.suite import aggregate_results, build_summary_rows, can_resume_result, expand_suite

_S, _MS = 1.0, 1000.0
AGGREGATE_METRICS = (
    [("metrics.throughput.requests_per_second", _S, "req/s"),
     ("metrics.throughput.input_tokens_per_second", _S, "tok/s"),
     ("metrics.throughput.output_tokens_per_second", _S, "tok/s"),
     ("metrics.throughput.total_tokens_per_second", _S, "tok/s"),
     ("metrics.goodput.requests_per_second", _S, "req/s")]
    + [(f"metrics.latency.overall.{name}.{p}", _MS, "ms")
       for name in ("ttft", "tpot", "burst_itl", "output_event_latency", "speculative_step_latency", "e2e")
       for p in ("p50", "p99")]
    + [(f"metrics.latency.{cls}.{name}.{p}", _MS, "ms")
       for cls in ("short", "long") for name in ("ttft", "tpot", "e2e") for p in ("p50", "p99")]
    + [("metrics.speculative.acceptance_rate", _S, "ratio"),
       ("metrics.speculative.acceptance_length", _S, "tokens/step"),
       ("metrics.scheduled_batch_size.mean", _S, "requests"),
       ("metrics.speculative_batch_size.mean", _S, "requests"),
       ("metrics.waiting_queue_size.p99", _S, "requests"),
       ("metrics.running_queue_size.p99", _S, "requests"),
       ("metrics.kv_cache.total_blocks", _S, "blocks"),
       ("metrics.kv_cache.peak_reserved_blocks", _S, "blocks"),
       ("metrics.kv_cache.preemptions", _S, "count"),
       ("metrics.kv_cache.admission_deferrals", _S, "count"),
       ("metrics.kv_cache.kv_cache_bytes", 1.0 / 2**30, "GiB"),
       ("metrics.kv_cache.model_runtime_bytes", 1.0 / 2**30, "GiB")]
)


def _write_csv(path: Path, rows: list[dict]):
    path.parent.mkdir(parents=True, exist_ok=True)
    if not rows:
        path.write_text("")
        return
    with path.open("w", newline="") as f:
        w = csv.DictWriter(f, fieldnames=list(rows[0]), lineterminator="\n")
        w.writeheader()
        w.writerows(rows)


def _load(path: Path):
    try:
        return json.loads(path.read_text())
    except (OSError, json.JSONDecodeError):
        return None


def _redact(message: str, paths):
    for p in paths:
        if p:
            message = message.replace(p, Path(p).name)
    return message


def _failure(point, metadata, process, error_type="WorkerProcessError", paths=()):
    stderr = (getattr(process, "stderr", "") or "").strip()
    return {"schema_version": 2, "complete": False, "point_id": point["point_id"],
            "git_commit": metadata.get("git_commit"), "metadata": metadata, "config": point, "metrics": None,
            "requests": [], "error": {"type": error_type, "returncode": getattr(process, "returncode", None),
                                      "message": _redact(stderr[-2000:] or "worker did not write a result", paths)}}


def _aggregate_all(results):
    rows = []
    for path, scale, unit in AGGREGATE_METRICS:
        rows.extend(aggregate_results(results, path, scale=scale, unit=unit))
    return rows


def execute_suite(suite: dict, output_dir: Path, model: str, speculative_model: str | None, metadata: dict, *,
                  model_revision: str | None = None, speculative_model_revision: str | None = None,
                  distributed_init_method: str = "tcp://127.0.0.1:2333", resume: bool = False,
                  timeout_seconds: float | None = None, command_runner=subprocess.run):
    output_dir = Path(output_dir)
    runs_dir, points_dir = output_dir / "runs", output_dir / "points"
    runs_dir.mkdir(parents=True, exist_ok=True)
    points_dir.mkdir(parents=True, exist_ok=True)
    points = expand_suite(suite)
    commit = metadata.get("git_commit")
    model_revision = model_revision or discover_model_revision(model)
    speculative_model_revision = speculative_model_revision or discover_model_revision(speculative_model)
    manifest = {
        "schema_version": 1, "suite": suite["name"], "complete": False, "git_commit": commit, "metadata": metadata,
        "model": Path(model).name, "model_revision": model_revision,
        "speculative_model": Path(speculative_model).name if speculative_model else None,
        "speculative_model_revision": speculative_model_revision,
        "distributed_init_method": distributed_init_method, "total_points": len(points),
        "completed_points": 0, "failed_points": 0,
    }
    atomic_write_json(output_dir / "manifest.json", manifest)
    paths = (model, speculative_model)
    results = []
    for i, point in enumerate(points, start=1):
        point_path = points_dir / f"{point['point_id']}.json"
        result_path = runs_dir / f"{point['point_id']}.json"
        atomic_write_json(point_path, point)
        if resume and can_resume_result(result_path, point, commit):
            print(f"[{i}/{len(points)}] RESUME {point['point_id']}", flush=True)
            results.append(_load(result_path))
            continue
        result_path.unlink(missing_ok=True)
        cmd = [sys.executable, "-m", "benchmarks.serve", "--point-config", str(point_path), "--model", model,
               "--output", str(result_path), "--distributed-init-method", distributed_init_method]
        if speculative_model:
            cmd += ["--speculative-model", speculative_model]
        if model_revision:
            cmd += ["--model-revision", model_revision]
        if speculative_model_revision:
            cmd += ["--speculative-model-revision", speculative_model_revision]
        if commit:
            cmd += ["--expected-git-commit", commit]
        print(f"[{i}/{len(points)}] RUN {point['point_id']}", flush=True)
        error_type = "WorkerProcessError"
        try:
            process = command_runner(cmd, capture_output=True, text=True, timeout=timeout_seconds)
        except subprocess.TimeoutExpired as e:
            process = e
            process.returncode = None
            process.stderr = f"worker timed out after {timeout_seconds}s"
        except OSError as e:
            error_type = "WorkerStartError"
            process = SimpleNamespace(returncode=None, stderr=str(e))
        result = _load(result_path)
        if result is None:
            result = _failure(point, metadata, process, error_type, paths)
            atomic_write_json(result_path, result)
        elif result.get("complete") and not can_resume_result(result_path, point, commit):
            result["complete"] = False
            result["error"] = {"type": "InvalidWorkerResult", "returncode": process.returncode,
                               "message": "worker result identity does not match suite point"}
            atomic_write_json(result_path, result)
        if process.returncode != 0 and result.get("complete"):
            result["complete"] = False
            result["error"] = _failure(point, metadata, process, paths=paths)["error"]
            atomic_write_json(result_path, result)
        results.append(result)
    _write_csv(output_dir / "summary.csv", build_summary_rows(results))
    _write_csv(output_dir / "aggregate.csv", _aggregate_all(results))
    failed = sum(not r.get("complete") for r in results)
    manifest.update(complete=failed == 0, completed_points=len(results) - failed, failed_points=failed)
    atomic_write_json(output_dir / "manifest.json", manifest)
    return 0 if failed == 0 else 1


def _parse_args(argv=None):
    p = argparse.ArgumentParser(description="Run a reproducible llmserve_b200 benchmark suite")
    p.add_argument("--suite", required=True)
    p.add_argument("--output-dir", required=True)
    p.add_argument("--model", default=os.environ.get("MODEL_PATH"))
    p.add_argument("--speculative-model", default=os.environ.get("SPECULATIVE_MODEL"))
    p.add_argument("--model-revision")
    p.add_argument("--speculative-model-revision")
    p.add_argument("--distributed-init-method", default="tcp://127.0.0.1:2333")
    p.add_argument("--resume", action="store_true")
    p.add_argument("--allow-dirty", action="store_true")
    p.add_argument("--timeout-seconds", type=float)
    args = p.parse_args(argv)
    if not args.model:
        p.error("--model or MODEL_PATH is required")
    return args


def main(argv=None):
    args = _parse_args(argv)
    suite = json.loads(Path(args.suite).read_text())
    metadata = build_environment_metadata()
    if metadata.get("git_dirty") and not args.allow_dirty:
        print("refusing formal benchmark on a dirty worktree; use --allow-dirty for smoke/pilot runs",
              file=sys.stderr)
        return 2
    return execute_suite(suite, Path(args.output_dir), model=os.path.expanduser(args.model),
                         speculative_model=os.path.expanduser(args.speculative_model) if args.speculative_model else None,
                         metadata=metadata, model_revision=args.model_revision,
                         speculative_model_revision=args.speculative_model_revision,
                         distributed_init_method=args.distributed_init_method, resume=args.resume,
                         timeout_seconds=args.timeout_seconds)


if __name__ == "__main__":
    raise SystemExit(main())
