"""Driving loops (``benchmarks/runtime.py`` of the reference).

``run_poisson`` admits requests when their arrival time has passed, steps the engine, and sleeps
when idle.  ``run_closed_loop`` keeps ``max_concurrency`` requests in flight: after a warm-up it
measures for a fixed window, stops refilling at the window's end and drains.  Latency statistics
use only requests that both arrived and finished inside the window; throughput counts completions
and output tokens whose timestamps fall inside it.  The engine is duck-typed (``add_request``,
``step``, ``is_finished``, ``last_step_events``, ``get_metrics``).
"""
import time
from collections import deque
from collections.abc import Callable, Sequence

from benchmarks.workloads import RequestSpec


def _record_step(events: dict, sizes: dict):
    sizes["scheduled"].append(len(events.get("scheduled_seq_ids", [])))
    sizes["waiting"].append(events.get("waiting_queue_size", 0))
    sizes["running"].append(events.get("running_queue_size", 0))
    if events.get("speculative"):
        sizes["speculative"].append(events.get("speculative_batch_size", 0))


def _label(engine_metrics: dict, seq_to_spec: dict):
    out = []
    for request in engine_metrics["requests"]:
        request = dict(request)
        spec = seq_to_spec[request["seq_id"]]
        request["request_id"] = spec.request_id
        request["request_class"] = spec.request_class
        out.append(request)
    out.sort(key=lambda r: r["request_id"])
    return out


def run_poisson(engine, request_specs: Sequence[RequestSpec], arrival_times: Sequence[float],
                make_sampling_params: Callable[[RequestSpec], object], clock: Callable[[], float] = time.perf_counter,
                sleep: Callable[[float], None] = time.sleep):
    if len(request_specs) != len(arrival_times):
        raise ValueError("request_specs and arrival_times must have the same length")
    if not request_specs:
        raise ValueError("request_specs cannot be empty")
    pending = deque(zip(arrival_times, request_specs))
    seq_to_spec, seq_to_arrival = {}, {}
    sizes = {"scheduled": [], "speculative": [], "waiting": [], "running": []}
    start = clock()
    while pending or not engine.is_finished():
        now = clock() - start
        while pending and pending[0][0] <= now:
            at, spec = pending.popleft()
            sid = engine.add_request(list(spec.prompt_token_ids), make_sampling_params(spec))
            seq_to_spec[sid] = spec
            seq_to_arrival[sid] = start + at
        if not engine.is_finished():
            engine.step()
            _record_step(engine.last_step_events, sizes)
            continue
        if pending:
            delay = pending[0][0] - (clock() - start)
            if delay > 0:
                sleep(delay)
    metrics = engine.get_metrics()
    requests = _label(metrics, seq_to_spec)
    for r in requests:
        r["arrival_time"] = seq_to_arrival[r["seq_id"]]
    first = min(r["arrival_time"] for r in requests)
    finished = [r["finish_time"] for r in requests if r["finish_time"] is not None]
    end = max(finished) if finished else clock()
    return {
        "admitted": len(seq_to_spec), "duration": end - first, "requests": requests,
        "scheduled_batch_sizes": sizes["scheduled"], "speculative_batch_sizes": sizes["speculative"],
        "waiting_queue_sizes": sizes["waiting"], "running_queue_sizes": sizes["running"],
        "engine_summary": metrics.get("summary", {}),
    }


def run_closed_loop(engine, request_specs, max_concurrency: int, warmup_seconds: float,
                    measurement_seconds: float, make_sampling_params: Callable[[RequestSpec], object],
                    clock: Callable[[], float] = time.perf_counter):
    if max_concurrency <= 0:
        raise ValueError("max_concurrency must be positive")
    if warmup_seconds < 0:
        raise ValueError("warmup_seconds must be non-negative")
    if measurement_seconds <= 0:
        raise ValueError("measurement_seconds must be positive")
    specs = iter(request_specs)
    seq_to_spec = {}
    in_flight = 0

    def refill():
        nonlocal in_flight
        while in_flight < max_concurrency:
            spec = next(specs)
            sid = engine.add_request(list(spec.prompt_token_ids), make_sampling_params(spec))
            seq_to_spec[sid] = spec
            in_flight += 1

    refill()
    window_start = clock() + warmup_seconds
    window_end = window_start + measurement_seconds
    sizes = {"scheduled": [], "speculative": [], "waiting": [], "running": []}
    while clock() < window_end:
        outputs, _ = engine.step()
        in_flight -= len(outputs)
        events = engine.last_step_events
        step_end = events.get("step_end", clock())
        if window_start <= step_end < window_end:
            _record_step(events, sizes)
        if step_end < window_end:
            refill()
    while not engine.is_finished():
        engine.step()
    metrics = engine.get_metrics()
    requests = _label(metrics, seq_to_spec)
    in_window = [r for r in requests if r["arrival_time"] >= window_start and r["finish_time"] is not None
                 and r["finish_time"] < window_end]
    completed = sum(r["finish_time"] is not None and window_start <= r["finish_time"] < window_end for r in requests)
    out_tokens = sum(window_start <= t < window_end for r in requests for t in r.get("token_times", []))
    return {
        "admitted": len(seq_to_spec), "duration": measurement_seconds, "measurement_start": window_start,
        "measurement_end": window_end, "requests": requests, "latency_requests": in_window,
        "window_completed": completed, "window_output_tokens": out_tokens,
        "scheduled_batch_sizes": sizes["scheduled"], "speculative_batch_sizes": sizes["speculative"],
        "waiting_queue_sizes": sizes["waiting"], "running_queue_sizes": sizes["running"],
        "engine_summary": metrics.get("summary", {}),
    }
