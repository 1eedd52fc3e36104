"""Serving metrics (``benchmarks/metrics.py`` of the reference).

Linear-interpolation percentiles; per-class latency summaries of ttft / tpot / e2e (one value per
request) and burst ITL / output-event latency / speculative step latency (all samples); goodput =
requests meeting every SLO per second; speculative aggregates.
"""
from collections.abc import Mapping, Sequence

SCALARS = ("ttft", "tpot", "e2e")
SAMPLES = ("burst_itl", "output_event_latency", "speculative_step_latency")


def percentile(values: Sequence[float], q: float):
    if not values:
        return None
    v = sorted(values)
    if len(v) == 1:
        return v[0]
    rank = (len(v) - 1) * q / 100
    lo = int(rank)
    hi = min(lo + 1, len(v) - 1)
    frac = rank - lo
    return v[lo] * (1 - frac) + v[hi] * frac


def summarize_values(values: Sequence[float]):
    if not values:
        return {"count": 0, "mean": None, "p50": None, "p90": None, "p99": None, "max": None}
    return {"count": len(values), "mean": sum(values) / len(values), "p50": percentile(values, 50),
            "p90": percentile(values, 90), "p99": percentile(values, 99), "max": max(values)}


def _gaps(times):
    return [b - a for a, b in zip(times, times[1:])]


def request_latency(request: Mapping) -> dict:
    arrival, first, finish = request["arrival_time"], request["first_token_time"], request["finish_time"]
    n = request["output_tokens"]
    burst = request.get("burst_itl")
    if burst is None:
        burst = _gaps(request.get("token_times", []))
    events = request.get("output_event_latency")
    if events is None:
        events = _gaps(request.get("output_event_times", []))
    return {
        "ttft": first - arrival,
        "tpot": (finish - first) / (n - 1) if n > 1 else 0.0,
        "burst_itl": burst,
        "output_event_latency": events,
        "speculative_step_latency": request.get("speculative_step_latency", []),
        "e2e": finish - arrival,
    }


_request_latency = request_latency


def latency_summary(requests: Sequence[Mapping]) -> dict:
    values = {name: [] for name in SCALARS + SAMPLES}
    for r in requests:
        lat = request_latency(r)
        for name in SCALARS:
            values[name].append(lat[name])
        for name in SAMPLES:
            values[name].extend(lat[name])
    return {name: summarize_values(v) for name, v in values.items()}


def summarize_speculative_requests(requests: Sequence[Mapping]) -> dict:
    def total(key):
        return sum(r.get(key, 0) for r in requests)

    steps, drafts = total("speculative_steps"), total("speculative_draft_tokens")
    accepted, emitted = total("speculative_accepted_tokens"), total("speculative_emitted_tokens")
    gamma_counts, timing = {}, {}
    for r in requests:
        for g, c in r.get("speculative_gamma_counts", {}).items():
            gamma_counts[g] = gamma_counts.get(g, 0) + c
        for name, value in r.get("speculative_timing", {}).items():
            timing[name] = timing.get(name, 0.0) + value
    return {
        "steps": steps, "draft_tokens": drafts, "accepted_tokens": accepted, "emitted_tokens": emitted,
        "acceptance_rate": accepted / drafts if drafts > 0 else None,
        "acceptance_length": emitted / steps if steps > 0 else None,
        "accepted_length": accepted / steps if steps > 0 else None,
        "draft_tokens_per_step": drafts / steps if steps > 0 else None,
        "accept_all_count": total("speculative_accept_all_count"),
        "gamma_counts": dict(sorted(gamma_counts.items(), key=lambda kv: int(kv[0]))),
        "timing": {name: {"total_ms": t * 1000, "mean_ms": t * 1000 / steps if steps > 0 else None}
                   for name, t in sorted(timing.items())},
    }


def goodput_summary(requests: Sequence[Mapping], duration: float, slo_ms: Mapping[str, float]) -> dict:
    unknown = set(slo_ms) - set(SCALARS)
    if unknown:
        raise ValueError(f"unsupported SLO metrics: {sorted(unknown)}")
    limits = {k: v / 1000 for k, v in slo_ms.items()}
    good = sum(1 for r in requests if all(request_latency(r)[k] <= lim for k, lim in limits.items()))
    return {"completed": good, "requests_per_second": good / duration, "slo_ms": dict(slo_ms)}


_goodput_summary = goodput_summary


def summarize_serving_run(requests: Sequence[Mapping], duration: float, slo_ms: Mapping[str, float] | None = None):
    if duration <= 0:
        raise ValueError("duration must be positive")
    ok = [r for r in requests if r["success"]]
    groups = {"overall": ok}
    for r in ok:
        groups.setdefault(r["request_class"], []).append(r)
    n_in = sum(r["prompt_tokens"] for r in ok)
    n_out = sum(r["output_tokens"] for r in ok)
    return {
        "completed": len(ok), "failed": len(requests) - len(ok), "duration": duration,
        "throughput": {"requests_per_second": len(ok) / duration, "input_tokens_per_second": n_in / duration,
                       "output_tokens_per_second": n_out / duration,
                       "total_tokens_per_second": (n_in + n_out) / duration},
        "latency": {name: latency_summary(group) for name, group in groups.items()},
        "goodput": goodput_summary(ok, duration, slo_ms) if slo_ms is not None else None,
    }
