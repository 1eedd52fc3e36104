"""Per-request sampling knobs.

Parity: ``llmserve/sampling_params.py:4-11`` of the reference -- same three fields,
same defaults, and the same refusal of temperature ~0 (greedy decoding is obtained
by swapping the runner's sampler for an argmax sampler, as the benchmarks do).
"""
from dataclasses import dataclass


@dataclass(slots=True)
class SamplingParams:
    temperature: float = 1.0
    max_tokens: int = 64
    ignore_eos: bool = False

    def __post_init__(self):
        if not self.temperature > 1e-10:
            raise ValueError("temperature must be > 1e-10 (greedy sampling is not permitted)")
        if self.max_tokens <= 0:
            raise ValueError("max_tokens must be positive")
