"""Request mixes (``benchmarks/workloads.py`` of the reference).

A profile is a list of weighted classes (input length, output length).  ``build_request_specs``
draws a finite shuffled list with exact per-class counts (largest remainder); ``iter_request_specs``
repeats that in cycles of ``cycle_size`` for closed-loop runs.  Prompt ids are uniform in
``[0, prompt_id_high]`` (10000 in the reference; the B200 suites set the vocabulary size).
"""
from dataclasses import dataclass
from math import floor
from random import Random
from typing import Sequence

DEFAULT_PROMPT_ID_HIGH = 10000


@dataclass(frozen=True)
class WorkloadClass:
    name: str
    weight: float
    input_len: int
    output_len: int

    def __post_init__(self):
        bad = [f"{field}={getattr(self, field)!r}" for field in ("weight", "input_len", "output_len")
               if not getattr(self, field) > 0]
        if not self.name:
            bad.insert(0, "name is empty")
        if bad:
            raise ValueError(f"invalid request class {self.name!r}: " + ", ".join(bad) + " (lengths and weight must be > 0)")


@dataclass(frozen=True)
class RequestSpec:
    request_id: int
    request_class: str
    input_len: int
    output_len: int
    prompt_token_ids: tuple[int, ...]


def class_counts(classes: Sequence[WorkloadClass], total: int) -> list[int]:
    """Largest-remainder apportionment of ``total`` requests by class weight (ties -> lower index)."""
    weight_sum = sum(c.weight for c in classes)
    exact = [total * c.weight / weight_sum for c in classes]
    counts = [floor(x) for x in exact]
    left = total - sum(counts)
    order = sorted(range(len(classes)), key=lambda i: (-(exact[i] - counts[i]), i))
    for i in order[:left]:
        counts[i] += 1
    return counts


_class_counts = class_counts


def _need_classes(classes):
    if not classes:
        raise ValueError("a workload profile needs at least one request class")


def _assignments(classes, counts):
    out = []
    for c, n in zip(classes, counts):
        out.extend([c] * n)
    return out


def build_request_specs(classes: Sequence[WorkloadClass], num_requests: int, seed: int,
                        prompt_id_high: int = DEFAULT_PROMPT_ID_HIGH) -> list[RequestSpec]:
    _need_classes(classes)
    if num_requests < 0:
        raise ValueError(f"num_requests={num_requests}: a workload cannot have a negative size")
    rng = Random(seed)
    picks = _assignments(classes, class_counts(classes, num_requests))
    rng.shuffle(picks)
    return [RequestSpec(i, c.name, c.input_len, c.output_len,
                        tuple(rng.randint(0, prompt_id_high) for _ in range(c.input_len)))
            for i, c in enumerate(picks)]


def iter_request_specs(classes: Sequence[WorkloadClass], seed: int, cycle_size: int = 100,
                       prompt_id_high: int = DEFAULT_PROMPT_ID_HIGH):
    _need_classes(classes)
    if cycle_size <= 0:
        raise ValueError(f"cycle_size={cycle_size}: each cycle must hold at least one request")
    rng = Random(seed)
    counts = class_counts(classes, cycle_size)
    request_id = 0
    while True:
        picks = _assignments(classes, counts)
        rng.shuffle(picks)
        for c in picks:
            ids = tuple(rng.randint(0, prompt_id_high) for _ in range(c.input_len))
            yield RequestSpec(request_id, c.name, c.input_len, c.output_len, ids)
            request_id += 1
