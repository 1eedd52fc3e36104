"""Compact per-request records of result schema v2 (``benchmarks/schema.py`` of the reference):
latencies in milliseconds, no absolute timestamps."""
from benchmarks.metrics import summarize_values


def _ms_summary(values):
    return summarize_values([v * 1000 for v in values])


def _gaps(times):
    return [b - a for a, b in zip(times, times[1:])]


def compact_request_record(request: dict) -> dict:
    first, finish, arrival = request.get("first_token_time"), request.get("finish_time"), request["arrival_time"]
    n = request["output_tokens"]
    ttft = (first - arrival) * 1000 if first is not None else None
    e2e = (finish - arrival) * 1000 if finish is not None else None
    if n > 1 and first is not None and finish is not None:
        tpot = (finish - first) * 1000 / (n - 1)
    elif n == 1 and first is not None:
        tpot = 0.0
    else:
        tpot = None
    burst = request.get("burst_itl")
    if burst is None:
        burst = _gaps(request.get("token_times", []))
    events = request.get("output_event_latency")
    if events is None:
        events = _gaps(request.get("output_event_times", []))
    return {
        "seq_id": request["seq_id"], "request_id": request.get("request_id"),
        "request_class": request["request_class"], "prompt_tokens": request["prompt_tokens"], "output_tokens": n,
        "success": request["success"], "failure_reason": request.get("failure_reason"),
        "ttft_ms": ttft, "tpot_ms": tpot, "e2e_ms": e2e,
        "burst_itl_ms": _ms_summary(burst), "output_event_latency_ms": _ms_summary(events),
        "speculative_step_latency_ms": _ms_summary(request.get("speculative_step_latency", [])),
        "speculative": {
            "steps": request.get("speculative_steps", 0),
            "draft_tokens": request.get("speculative_draft_tokens", 0),
            "accepted_tokens": request.get("speculative_accepted_tokens", 0),
            "emitted_tokens": request.get("speculative_emitted_tokens", 0),
            "accept_all_count": request.get("speculative_accept_all_count", 0),
            "gamma_counts": request.get("speculative_gamma_counts", {}),
            "timing_ms": {k: v * 1000 for k, v in sorted(request.get("speculative_timing", {}).items())},
        },
    }
