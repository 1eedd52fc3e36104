"""Request state.

Behavioural parity with ``llmserve/engine/sequence.py:19-102``: ``num_cached_tokens`` doubles as
the computed-token cursor for chunked prefill, and the pickled form sent to tensor-parallel
workers carries only what a worker needs (the full token list while the prompt is still being
computed, otherwise only the last token).  Unlike the reference the pickled form also carries
the sequence id and temperature, which workers need for speculative state and sampling.
"""
from copy import copy
from enum import Enum, auto
from itertools import count

from llmserve_b200.sampling_params import SamplingParams


class SequenceStatus(Enum):
    WAITING = auto()
    RUNNING = auto()
    FINISHED = auto()


class Sequence:
    block_size = 256
    counter = count()

    def __init__(self, token_ids: list[int], sampling_params: SamplingParams = SamplingParams()):
        if not token_ids:
            raise ValueError("a sequence needs at least one prompt token")
        self.seq_id = next(Sequence.counter)
        self.status = SequenceStatus.WAITING
        self.token_ids = copy(token_ids)
        self.last_token = token_ids[-1]
        self.num_tokens = len(self.token_ids)
        self.num_prompt_tokens = len(token_ids)
        self.num_cached_tokens = 0
        self.num_scheduled_tokens = 0
        self.block_table: list[int] = []
        self.temperature = sampling_params.temperature
        self.max_tokens = sampling_params.max_tokens
        self.ignore_eos = sampling_params.ignore_eos

    def __len__(self):
        return self.num_tokens

    def __getitem__(self, key):
        return self.token_ids[key]

    @property
    def is_finished(self) -> bool:
        return self.status == SequenceStatus.FINISHED

    @property
    def num_computed_tokens(self) -> int:
        return self.num_cached_tokens

    @property
    def is_prefilling(self) -> bool:
        return self.num_cached_tokens < self.num_tokens

    @property
    def num_uncomputed_tokens(self) -> int:
        return max(self.num_tokens - self.num_cached_tokens, 0)

    @property
    def num_completion_tokens(self) -> int:
        return self.num_tokens - self.num_prompt_tokens

    @property
    def prompt_token_ids(self) -> list[int]:
        return self.token_ids[: self.num_prompt_tokens]

    @property
    def completion_token_ids(self) -> list[int]:
        return self.token_ids[self.num_prompt_tokens:]

    @property
    def num_blocks(self) -> int:
        return -(-self.num_tokens // self.block_size)

    @property
    def last_block_num_tokens(self) -> int:
        return self.num_tokens - (self.num_blocks - 1) * self.block_size

    def block(self, i: int) -> list[int]:
        if not 0 <= i < self.num_blocks:
            raise IndexError(i)
        return self.token_ids[i * self.block_size:(i + 1) * self.block_size]

    def slot(self, position: int) -> int:
        """Flat KV-pool slot of ``position`` through this sequence's block table."""
        return self.block_table[position // self.block_size] * self.block_size + position % self.block_size

    def append_token(self, token_id: int):
        self.token_ids.append(token_id)
        self.last_token = token_id
        self.num_tokens += 1

    def __getstate__(self):
        ship_all = self.num_completion_tokens == 0 or self.num_cached_tokens < self.num_tokens
        tail = self.token_ids if ship_all else self.last_token
        return (self.seq_id, self.num_tokens, self.num_prompt_tokens, self.num_cached_tokens,
                self.num_scheduled_tokens, self.block_table, self.temperature, tail)

    def __setstate__(self, state):
        (self.seq_id, self.num_tokens, self.num_prompt_tokens, self.num_cached_tokens,
         self.num_scheduled_tokens, self.block_table, self.temperature, tail) = state
        self.status = SequenceStatus.RUNNING
        self.max_tokens = 0
        self.ignore_eos = True
        if isinstance(tail, list):
            self.token_ids = tail
            self.last_token = tail[-1]
        else:
            self.token_ids = []
            self.last_token = tail
