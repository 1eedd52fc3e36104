"""Result records exchanged by draft, verify and accept (``llmserve/speculative/types.py``)."""
from dataclasses import dataclass

import torch


@dataclass(slots=True)
class SpeculativeSampleResult:
    token_ids: list[int]
    accepted_token_ids: list[int]
    final_token_id: int
    num_accepted: int
    accepted_all: bool


@dataclass(slots=True)
class Eagle3TargetVerifyOutput:
    target_logits: torch.Tensor
    target_aux_hidden: torch.Tensor


@dataclass(slots=True)
class SpeculativeDecodeOutput:
    token_ids: list[int]
    num_draft_tokens: int
    num_accepted: int
    accepted_all: bool
    emitted_tokens: int
    timing: dict | None = None
    debug: dict | None = None
