"""Offline EAGLE3 drafting: serial and batched draft generation, one speculative cycle, and an
offline draft -> target verify -> accept step, each with per-stage timing.

Parity with ``llmserve/speculative/draft.py`` of the reference: ``generate_eagle3_draft_tokens``
(``:52-107``), ``generate_eagle3_draft_tokens_batched`` with per-request gammas (``:156-238``),
``run_eagle3_speculative_cycle`` (``:241-263``), ``run_eagle3_target_verify`` (``:266-277``),
``run_eagle3_offline_step`` (``:280-307``) and the four stage timings of ``_DraftStageProfiler``
(``:17-49``).  The serving engine does not call these functions: its batched drafting runs in the
speculative executor over the engine's own paged draft pool.

Draft models are duck-typed: ``propose(input_ids [B, 1], aux_hidden [B, 1, W], positions [B, 1],
temperature=, past_kv=, kv_valid_lens=)`` returns an :class:`Eagle3DraftOutput`, and
``greedy_sample(draft_logits)`` turns a draft-vocabulary argmax into target ids.  The draft K/V
comes in one of two forms:

* paged (``Eagle3Speculator.propose``): a :class:`DraftKVPool` keeps every request's history in
  fixed-size blocks, one block list per request, in the engine's pool layout, and ``past_kv`` is a
  :class:`DraftKVRef` naming the pool and the rows.  A batched step hands the active rows to the
  model where they lie, so no K/V is copied between depths;
* contiguous ``(k, v)`` pairs ``[B, kv_heads, L, head_dim]`` (the reference's layout, and what
  simple test doubles return): before a batched step the active requests' pairs are padded to one
  length and described by ``kv_valid_lens``; afterwards each request keeps its valid prefix plus
  the position the step appended.
"""
import contextlib
from dataclasses import dataclass
from time import perf_counter

import torch
import torch.nn.functional as F

from llmserve_b200.speculative.sampling import speculative_accept_reject_from_logits
from llmserve_b200.speculative.types import (Eagle3CycleResult, Eagle3DraftOutput, Eagle3DraftSequence,
                                             Eagle3OfflineStepResult, Eagle3TargetVerifyOutput)

__all__ = ["STAGES", "DraftStageProfiler", "DraftKVPool", "DraftKVRef", "Eagle3DraftOutput",
           "generate_eagle3_draft_tokens", "generate_eagle3_draft_tokens_batched",
           "run_eagle3_speculative_cycle", "run_eagle3_target_verify", "run_eagle3_offline_step"]

STAGES = ("draft_pack_time", "draft_forward_time", "draft_sample_time", "draft_compact_time")
_MODES = ("sample", "greedy")


class DraftStageProfiler:
    """Seconds per drafting stage: CUDA events on a GPU, read once in :meth:`finish` (so timing adds
    no synchronisation inside the loop); the host clock otherwise."""

    def __init__(self, device):
        self.device = torch.device(device)
        self.totals = dict.fromkeys(STAGES, 0.0)
        self._events = []

    @contextlib.contextmanager
    def stage(self, name: str):
        if self.device.type == "cuda":
            begin = torch.cuda.Event(enable_timing=True)
            end = torch.cuda.Event(enable_timing=True)
            begin.record()
            try:
                yield
            finally:
                end.record()
                self._events.append((name, begin, end))
        else:
            t0 = perf_counter()
            try:
                yield
            finally:
                self.totals[name] += perf_counter() - t0

    def finish(self) -> dict:
        if self._events:
            torch.cuda.synchronize(self.device)
            for name, begin, end in self._events:
                self.totals[name] += begin.elapsed_time(end) / 1e3
            self._events.clear()
        return dict(self.totals)


class DraftKVPool:
    """Paged draft K/V for offline use.

    ``k`` / ``v`` are ``[num_blocks, kv_heads, block_size, head_dim]``, the layout of the engine's
    draft pool, so the draft's store and decode-attention kernels read them unchanged.  Each row
    (one request) owns a block list and a length; the slot of its position ``p`` is
    ``blocks[p // block_size] * block_size + p % block_size``.  When the free list is empty the pool
    doubles (a copy; offline use only)."""

    def __init__(self, num_kv_heads: int, head_dim: int, dtype=torch.float32, device="cpu",
                 block_size: int = 256, num_blocks: int = 4):
        if block_size <= 0 or num_blocks <= 0:
            raise ValueError("block_size and num_blocks must be positive")
        self.k = torch.zeros(num_blocks, num_kv_heads, block_size, head_dim, dtype=dtype, device=device)
        self.v = torch.zeros_like(self.k)
        self.block_size = block_size
        self.free = list(range(num_blocks - 1, -1, -1))
        self.blocks: dict[int, list[int]] = {}
        self.lengths: dict[int, int] = {}
        self._next_row = 0

    @classmethod
    def for_model(cls, model, device, **kw) -> "DraftKVPool":
        dtype = kw.pop("dtype", model.embed_tokens.weight.dtype)
        return cls(model.num_kv_heads, model.head_dim, dtype, device, **kw)

    @property
    def device(self):
        return self.k.device

    def new_rows(self, n: int) -> list[int]:
        rows = list(range(self._next_row, self._next_row + n))
        self._next_row += n
        for r in rows:
            self.blocks[r], self.lengths[r] = [], 0
        return rows

    def release(self, row: int):
        self.free.extend(reversed(self.blocks.pop(row)))
        del self.lengths[row]

    def set_length(self, row: int, length: int):
        """Keep the first ``length`` positions of ``row`` (a rejected draft suffix is dropped)."""
        if not 0 <= length <= self.lengths[row]:
            raise ValueError(f"row {row} holds {self.lengths[row]} positions, cannot keep {length}")
        keep = -(-length // self.block_size)
        self.free.extend(reversed(self.blocks[row][keep:]))
        del self.blocks[row][keep:]
        self.lengths[row] = length

    def _grow(self):
        n = self.k.shape[0]
        self.k = torch.cat([self.k, torch.zeros_like(self.k)])
        self.v = torch.cat([self.v, torch.zeros_like(self.v)])
        self.free.extend(range(2 * n - 1, n - 1, -1))

    def append_slots(self, rows) -> list[int]:
        """Reserve the next position of every row and return its slot."""
        slots = []
        for r in rows:
            pos = self.lengths[r]
            blocks = self.blocks[r]
            if pos == len(blocks) * self.block_size:
                if not self.free:
                    self._grow()
                blocks.append(self.free.pop())
            slots.append(blocks[pos // self.block_size] * self.block_size + pos % self.block_size)
            self.lengths[r] = pos + 1
        return slots

    def block_table(self, rows, device=None) -> torch.Tensor:
        """int32 ``[len(rows), max blocks]``; unused entries hold block 0 and are never read."""
        width = max(1, max(len(self.blocks[r]) for r in rows))
        table = torch.zeros(len(rows), width, dtype=torch.int32)
        for i, r in enumerate(rows):
            table[i, :len(self.blocks[r])] = torch.tensor(self.blocks[r], dtype=torch.int32)
        return table.to(device if device is not None else self.device)

    def gather(self, row: int) -> tuple[torch.Tensor, torch.Tensor]:
        """The row's K and V as contiguous ``[kv_heads, length, head_dim]`` (for inspection)."""
        n = self.lengths[row]
        idx = torch.tensor(self.blocks[row], dtype=torch.long, device=self.device)

        def flat(pool):
            pages = pool[idx]                                   # [nb, kvh, bs, hd]
            return pages.permute(1, 0, 2, 3).reshape(pool.shape[1], -1, pool.shape[3])[:, :n]
        return flat(self.k), flat(self.v)


@dataclass
class DraftKVRef:
    """The draft K/V of ``rows`` (one per request of a step) in ``pool``."""
    pool: DraftKVPool
    rows: list

    @property
    def lengths(self) -> list[int]:
        return [self.pool.lengths[r] for r in self.rows]

    def select(self, i: int) -> "DraftKVRef":
        return DraftKVRef(self.pool, [self.rows[i]])


# ---- how per-request draft K/V enters and leaves one batched step --------------------------------

class _BatchedKV:
    """Per-request draft K/V of a batched draft (paged refs, contiguous pairs, or None)."""

    def __init__(self, entries):
        self.entries = entries

    def pack(self, active, depth, device):
        items = [self.entries[i] for i in active]
        if all(e is None for e in items):
            return None, None
        if any(isinstance(e, DraftKVRef) for e in items):
            pool = next(e for e in items if isinstance(e, DraftKVRef)).pool
            rows = []
            for e in items:
                if e is None:
                    rows.extend(pool.new_rows(1))
                elif isinstance(e, DraftKVRef) and e.pool is pool and len(e.rows) == 1:
                    rows.append(e.rows[0])
                else:
                    raise ValueError("a batched draft step needs every request's paged K/V in one pool")
            return DraftKVRef(pool, rows), None
        lens = [0 if e is None else int(e[0].shape[2]) for e in items]
        ref = next(e for e in items if e is not None)
        width = max(lens)

        def padded(e, j):
            if e is None:
                t = ref[j]
                return t.new_zeros(1, t.shape[1], width, t.shape[3])
            if e[j].shape[0] != 1:
                raise ValueError("per-request draft K/V must have batch size 1")
            return F.pad(e[j], (0, 0, 0, width - e[j].shape[2]))
        packed = tuple(torch.cat([padded(e, j) for e in items]) for j in (0, 1))
        return packed, torch.tensor(lens, dtype=torch.long, device=device)

    def unpack(self, active, packed, valid, new):
        if isinstance(new, DraftKVRef):
            for j, i in enumerate(active):
                self.entries[i] = new.select(j)
            return
        lens = valid.tolist() if valid is not None else [0] * len(active)
        for j, i in enumerate(active):
            pair = []
            for which in (0, 1):
                last = new[which][j:j + 1, :, -1:]
                if packed is not None and lens[j]:
                    last = torch.cat([packed[which][j:j + 1, :, :lens[j]], last], dim=2)
                pair.append(last.contiguous())
            self.entries[i] = tuple(pair)


class _SerialKV:
    """One request's draft K/V handed back to the model as returned; ``kv_valid_len`` (if given)
    is the number of valid cached positions before the first step."""

    def __init__(self, past, kv_valid_len):
        self.entries = [past]
        self.kv_valid_len = kv_valid_len

    def pack(self, active, depth, device):
        valid = None
        if self.kv_valid_len is not None:
            valid = torch.tensor([self.kv_valid_len + depth], dtype=torch.long, device=device)
        return self.entries[0], valid

    def unpack(self, active, packed, valid, new):
        self.entries[0] = new


def _check_mode(gamma, mode):
    if gamma <= 0:
        raise ValueError("gamma must be positive")
    if mode not in _MODES:
        raise ValueError(f"draft_sampling_mode must be one of {_MODES}")


def _draft_loop(draft_model, token_ids, positions, aux, gammas, temperature, mode, kv):
    """Run ``max(gammas)`` draft depths; request ``i`` takes part in its first ``gammas[i]``.

    ``token_ids`` / ``positions`` are int64 ``[B]`` tensors and ``aux`` is ``[B, 1, W]``; at depth 0
    the inputs are the target's auxiliary hidden states (width 3H), afterwards the draft's own
    hidden state (width H) of the previous depth.  One host read of the sampled ids per depth."""
    B = len(gammas)
    dev = aux.device
    prof = DraftStageProfiler(dev)
    ids = [[] for _ in range(B)]
    rows = [[] for _ in range(B)]
    for depth in range(max(gammas)):
        active = [i for i in range(B) if depth < gammas[i]]
        sel = torch.tensor(active, dtype=torch.long, device=dev)
        with prof.stage("draft_pack_time"):
            past, valid = kv.pack(active, depth, dev)
            step_ids = token_ids[sel].view(-1, 1)
            step_pos = positions[sel].view(-1, 1)
            step_aux = aux[sel]
        with prof.stage("draft_forward_time"):
            out = draft_model.propose(step_ids, step_aux, step_pos, temperature=temperature, past_kv=past,
                                      kv_valid_lens=valid)
        with prof.stage("draft_sample_time"):
            if mode == "greedy":
                nxt = draft_model.greedy_sample(out.draft_logits[:, -1:, :])
            else:
                nxt = out.token_ids
            nxt = nxt.reshape(len(active), -1)[:, -1]
            host = nxt.tolist()
        with prof.stage("draft_compact_time"):
            kv.unpack(active, past, valid, out.past_kv)
            for j, i in enumerate(active):
                ids[i].append(int(host[j]))
                rows[i].append(out.target_logits[j, -1])
            hidden = out.hidden_states[:, -1:, :]
            if depth == 0:
                aux = hidden.new_zeros(B, 1, hidden.shape[-1])
            aux[sel.to(aux.device)] = hidden.to(aux.dtype)
            token_ids[sel] = nxt.to(token_ids.device)
            positions[sel] += 1
    return ids, rows, prof.finish()


def _as_batch_aux(aux: torch.Tensor, batch: int) -> torch.Tensor:
    return aux.reshape(batch, 1, aux.shape[-1])


def generate_eagle3_draft_tokens(draft_model, start_token_id: int, start_aux_hidden: torch.Tensor,
                                 start_position: int, gamma: int, temperature: float, past_kv=None,
                                 kv_valid_len: int | None = None, draft_sampling_mode: str = "sample"
                                 ) -> Eagle3DraftSequence:
    """Draft ``gamma`` tokens for one request, starting from ``start_token_id`` at
    ``start_position`` with the target's auxiliary hidden state of the previous position."""
    _check_mode(gamma, draft_sampling_mode)
    dev = start_aux_hidden.device
    kv = _SerialKV(past_kv, kv_valid_len)
    ids, rows, timing = _draft_loop(
        draft_model, torch.tensor([start_token_id], dtype=torch.long, device=dev),
        torch.tensor([start_position], dtype=torch.long, device=dev), _as_batch_aux(start_aux_hidden, 1),
        [gamma], temperature, draft_sampling_mode, kv)
    return Eagle3DraftSequence(ids[0], torch.stack(rows[0]), kv.entries[0], timing)


def generate_eagle3_draft_tokens_batched(draft_model, start_token_ids: list[int], start_aux_hidden: torch.Tensor,
                                         start_positions: list[int], gamma: int, temperature: float,
                                         past_kv: list | None = None, draft_sampling_mode: str = "sample",
                                         gammas: list[int] | None = None) -> list[Eagle3DraftSequence]:
    """Draft for several requests at once: one ``propose`` per depth over the requests whose own
    gamma (``gammas``, default ``gamma`` for all) reaches that depth.  The stage timings are
    averaged over the requests."""
    _check_mode(gamma, draft_sampling_mode)
    B = len(start_token_ids)
    if B == 0:
        return []
    if len(start_positions) != B or start_aux_hidden.shape[0] != B:
        raise ValueError("batched draft inputs have inconsistent sizes")
    gammas = [gamma] * B if gammas is None else list(gammas)
    if len(gammas) != B or min(gammas) <= 0:
        raise ValueError("per-request gammas must be positive and one per request")
    entries = [None] * B if past_kv is None else list(past_kv)
    if len(entries) != B:
        raise ValueError("one draft K/V entry per request is required")
    dev = start_aux_hidden.device
    kv = _BatchedKV(entries)
    ids, rows, timing = _draft_loop(
        draft_model, torch.tensor(start_token_ids, dtype=torch.long, device=dev),
        torch.tensor(start_positions, dtype=torch.long, device=dev), _as_batch_aux(start_aux_hidden, B),
        gammas, temperature, draft_sampling_mode, kv)
    timing = {k: v / B for k, v in timing.items()}
    return [Eagle3DraftSequence(ids[i], torch.stack(rows[i]), kv.entries[i], dict(timing)) for i in range(B)]


def _accept(target_logits, draft: Eagle3DraftSequence, temperature, random_values):
    drafted = torch.tensor(draft.draft_token_ids, dtype=torch.long, device=target_logits.device)
    return speculative_accept_reject_from_logits(target_logits, draft.draft_target_logits.to(target_logits.device),
                                                 drafted, temperature=temperature, random_values=random_values)


def run_eagle3_speculative_cycle(draft_model, start_token_id: int, start_aux_hidden: torch.Tensor,
                                 start_position: int, target_verify_logits: torch.Tensor, gamma: int,
                                 temperature: float, random_values: torch.Tensor | None = None
                                 ) -> Eagle3CycleResult:
    """Draft ``gamma`` tokens, then accept them against given target verify logits
    (``[gamma + 1, vocab]``) by rejection sampling."""
    if gamma <= 0 or target_verify_logits.ndim != 2 or target_verify_logits.shape[0] != gamma + 1:
        raise ValueError("target_verify_logits must be [gamma + 1, vocab] with gamma > 0")
    draft = generate_eagle3_draft_tokens(draft_model, start_token_id, start_aux_hidden, start_position, gamma,
                                         temperature)
    sample = _accept(target_verify_logits, draft, temperature, random_values)
    return Eagle3CycleResult(draft.draft_token_ids, draft.draft_target_logits, sample, draft.past_kv)


def _device_of(model) -> torch.device:
    try:
        return next(model.parameters()).device
    except (AttributeError, StopIteration, TypeError):
        return torch.device("cpu")


def run_eagle3_target_verify(target_model, start_token_id: int, draft_token_ids: list[int],
                             start_position: int) -> Eagle3TargetVerifyOutput:
    """Score ``[start] + drafted`` at consecutive positions with the target.

    ``target_model`` provides ``forward_with_eagle3_aux(input_ids, positions)`` returning
    ``(hidden, aux)`` and ``compute_logits(hidden)`` for every row (the engine verifies inside its
    runner, with the packed paged-KV verify)."""
    dev = _device_of(target_model)
    tokens = [int(start_token_id), *map(int, draft_token_ids)]
    input_ids = torch.tensor(tokens, dtype=torch.long, device=dev)
    positions = torch.arange(start_position, start_position + len(tokens), dtype=torch.long, device=dev)
    hidden, aux = target_model.forward_with_eagle3_aux(input_ids, positions)
    return Eagle3TargetVerifyOutput(target_model.compute_logits(hidden), aux)


def run_eagle3_offline_step(target_model, draft_model, start_token_id: int, start_aux_hidden: torch.Tensor,
                            start_position: int, gamma: int, temperature: float,
                            random_values: torch.Tensor | None = None) -> Eagle3OfflineStepResult:
    """Draft, verify with the target, accept: one speculative step outside the engine."""
    draft = generate_eagle3_draft_tokens(draft_model, start_token_id, start_aux_hidden, start_position, gamma,
                                         temperature)
    verify = run_eagle3_target_verify(target_model, start_token_id, draft.draft_token_ids, start_position)
    sample = _accept(verify.target_logits, draft, temperature, random_values)
    return Eagle3OfflineStepResult(draft.draft_token_ids, draft.draft_target_logits, verify, sample, draft.past_kv)
