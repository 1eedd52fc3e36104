"""Poisson arrivals (``benchmarks/arrivals.py`` of the reference): first arrival at t=0, then
exponential gaps of rate ``request_rate`` drawn from ``Random(seed)``."""
from random import Random


def poisson_arrival_times(num_requests: int, request_rate: float, seed: int) -> list[float]:
    if num_requests < 0:
        raise ValueError("num_requests must be non-negative")
    if request_rate <= 0:
        raise ValueError("request_rate must be positive")
    if num_requests == 0:
        return []
    rng = Random(seed)
    times = [0.0]
    while len(times) < num_requests:
        times.append(times[-1] + rng.expovariate(request_rate))
    return times
