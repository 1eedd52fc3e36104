"""Continuous-batching scheduler.

Policies and their reference counterparts (``llmserve/engine/scheduler.py``):

* default (``schedule``, ``:118-166``): admit waiting prompts first -- only the first admitted
  prompt may be cut to fit the token budget -- and run decodes only in steps without prefill;
  when a decode cannot get a block, preempt from the tail of the running queue (recompute);
* chunked prefill (``schedule_chunked_prefill``, ``:179-241``): decode-first; every running
  sequence takes one token of the budget, the remainder goes to prefill chunks;
* KV-capacity admission (``_try_reserve``, ``:75-90``): reserve the projected final block count
  (prompt + max_tokens + speculative margin) and defer admission instead of preempting later.

Postprocessing appends sampled tokens and retires sequences on EOS / max_tokens; the
speculative variant appends several tokens at once and returns unused reserved slots.
"""
from collections import deque
from dataclasses import dataclass

from llmserve_b200.config import Config
from llmserve_b200.engine.block_manager import BlockManager
from llmserve_b200.engine.sequence import Sequence, SequenceStatus


@dataclass(slots=True)
class SchedulerOutput:
    """One step's work: prefill chunks first, then single-token decodes."""

    scheduled_seqs: list[Sequence]
    prefill_seqs: list[Sequence]
    decode_seqs: list[Sequence]
    num_batched_tokens: int

    def __post_init__(self):
        if self.scheduled_seqs != self.prefill_seqs + self.decode_seqs:
            raise ValueError("scheduled sequences must be ordered as prefill then decode")
        if self.num_batched_tokens < 0:
            raise ValueError("num_batched_tokens cannot be negative")

    @classmethod
    def build(cls, prefill_seqs: list[Sequence], decode_seqs: list[Sequence]) -> "SchedulerOutput":
        seqs = prefill_seqs + decode_seqs
        return cls(seqs, prefill_seqs, decode_seqs, sum(s.num_scheduled_tokens for s in seqs))


class Scheduler:

    def __init__(self, config: Config):
        self.max_num_seqs = config.max_num_seqs
        self.max_num_batched_tokens = config.max_num_batched_tokens
        self.eos = config.eos
        self.block_manager = BlockManager(config.num_kvcache_blocks, config.kvcache_block_size)
        self.enable_chunked_prefill = config.enable_chunked_prefill
        self.enable_kv_capacity_admission = config.enable_kv_capacity_admission
        self.max_model_len = config.max_model_len
        self.speculative_reserve_tokens = (
            config.speculative_gamma + 2 if config.speculative_model is not None else 0)
        self._reserved_blocks: dict[int, int] = {}
        self.preemption_count = 0
        self.admission_deferred_count = 0
        self.peak_reserved_blocks = 0
        self.waiting: deque[Sequence] = deque()
        self.running: deque[Sequence] = deque()

    def is_finished(self) -> bool:
        return not self.waiting and not self.running

    def add(self, seq: Sequence):
        if self.enable_kv_capacity_admission:
            need = self._projected_blocks(seq)
            total = len(self.block_manager.blocks)
            if need > total:
                raise ValueError(f"request requires {need} KV blocks but KV capacity is {total}")
        self.waiting.append(seq)

    # ---- capacity admission ----------------------------------------------------------------
    def _projected_blocks(self, seq: Sequence) -> int:
        final_tokens = min(seq.num_prompt_tokens + seq.max_tokens, self.max_model_len)
        return -(-(final_tokens + self.speculative_reserve_tokens) // self.block_manager.block_size)

    def _try_reserve(self, seq: Sequence) -> bool:
        if not self.enable_kv_capacity_admission or seq.seq_id in self._reserved_blocks:
            return True
        need = self._projected_blocks(seq)
        held = sum(self._reserved_blocks.values())
        if held + need > len(self.block_manager.blocks):
            self.admission_deferred_count += 1
            return False
        self._reserved_blocks[seq.seq_id] = need
        self.peak_reserved_blocks = max(self.peak_reserved_blocks, held + need)
        return True

    def _release_reservation(self, seq: Sequence):
        self._reserved_blocks.pop(seq.seq_id, None)

    def reset_metrics(self):
        self.preemption_count = 0
        self.admission_deferred_count = 0
        self.peak_reserved_blocks = sum(self._reserved_blocks.values())

    def kv_capacity_metrics(self) -> dict:
        total = len(self.block_manager.blocks)
        reserved = sum(self._reserved_blocks.values())
        return {
            "enabled": self.enable_kv_capacity_admission,
            "total_blocks": total,
            "used_blocks": len(self.block_manager.used_block_ids),
            "free_blocks": len(self.block_manager.free_block_ids),
            "reserved_blocks": reserved,
            "active_reservations": len(self._reserved_blocks),
            "peak_reserved_blocks": self.peak_reserved_blocks,
            "reservation_utilization": reserved / total if total else 0.0,
            "preemptions": self.preemption_count,
            "admission_deferrals": self.admission_deferred_count,
        }

    # ---- scheduling ------------------------------------------------------------------------
    def _make_room_for_decode(self, seq: Sequence) -> bool:
        """Preempt from the tail until ``seq`` can append; False if ``seq`` itself was evicted."""
        while not self.block_manager.can_append(seq):
            if self.running:
                self.preempt(self.running.pop())
            else:
                self.preempt(seq)
                return False
        return True

    def schedule(self) -> SchedulerOutput:
        if self.enable_chunked_prefill:
            return self.schedule_chunked_prefill()
        prefills: list[Sequence] = []
        budget = self.max_num_batched_tokens
        while self.waiting and len(prefills) < self.max_num_seqs:
            seq = self.waiting[0]
            todo = max(seq.num_tokens - seq.num_cached_tokens, 1)
            if budget == 0 or not self._try_reserve(seq):
                break
            if not seq.block_table and not self.block_manager.can_allocate(seq):
                break
            if budget < todo and prefills:
                break
            if not seq.block_table:
                self.block_manager.allocate(seq)
                # a prefix-cache hit shrinks the work (the reference keeps the pre-hit count here,
                # which schedules more query tokens than remain)
                todo = max(seq.num_tokens - seq.num_cached_tokens, 1)
            seq.num_scheduled_tokens = min(todo, budget)
            if seq.num_scheduled_tokens == todo:
                seq.status = SequenceStatus.RUNNING
                self.waiting.popleft()
                self.running.append(seq)
            prefills.append(seq)
            budget -= seq.num_scheduled_tokens
        if prefills:
            return SchedulerOutput.build(prefills, [])

        decodes: list[Sequence] = []
        while self.running and len(decodes) < self.max_num_seqs:
            seq = self.running.popleft()
            if self._make_room_for_decode(seq):
                seq.num_scheduled_tokens = 1
                self.block_manager.may_append(seq)
                decodes.append(seq)
        assert decodes, "scheduler has no sequence to schedule"
        self.running.extendleft(reversed(decodes))
        return SchedulerOutput.build([], decodes)

    def schedule_chunked_prefill(self) -> SchedulerOutput:
        decodes: list[Sequence] = []
        prefills: list[Sequence] = []
        promoted: list[Sequence] = []
        budget = self.max_num_batched_tokens
        count = 0
        while self.running and count < self.max_num_seqs and budget > 0:
            seq = self.running.popleft()
            if not self._make_room_for_decode(seq):
                continue
            seq.num_scheduled_tokens = 1
            self.block_manager.may_append(seq)
            decodes.append(seq)
            count += 1
            budget -= 1
        left_over = list(self.running)
        self.running.clear()

        while self.waiting and count < self.max_num_seqs and budget > 0:
            seq = self.waiting[0]
            if not self._try_reserve(seq):
                break
            if not seq.block_table:
                if not self.block_manager.can_allocate(seq):
                    break
                self.block_manager.allocate(seq)
            todo = max(seq.num_tokens - seq.num_cached_tokens, 1)
            chunk = min(todo, budget)
            if chunk == 0:
                break
            seq.num_scheduled_tokens = chunk
            prefills.append(seq)
            budget -= chunk
            count += 1
            if chunk != todo:
                break
            seq.status = SequenceStatus.RUNNING
            self.waiting.popleft()
            promoted.append(seq)

        self.running = deque(decodes + promoted + left_over)
        if prefills or decodes:
            return SchedulerOutput.build(prefills, decodes)
        raise AssertionError("scheduler has no sequence to schedule")

    def preempt(self, seq: Sequence):
        self.preemption_count += 1
        seq.status = SequenceStatus.WAITING
        self.block_manager.deallocate(seq)
        self.waiting.appendleft(seq)

    # ---- postprocessing --------------------------------------------------------------------
    def _retire(self, seq: Sequence):
        seq.status = SequenceStatus.FINISHED
        self.block_manager.deallocate(seq)
        self._release_reservation(seq)
        if seq in self.running:
            self.running.remove(seq)

    def postprocess(self, output: SchedulerOutput, token_ids: list[int]):
        if len(output.scheduled_seqs) != len(token_ids):
            raise ValueError("token count does not match scheduled sequences")
        n_prefill = len(output.prefill_seqs)
        for i, seq in enumerate(output.scheduled_seqs):
            self._postprocess_sequence(seq, token_ids[i], is_prefill=i < n_prefill)

    def _postprocess_sequence(self, seq: Sequence, token_id: int, is_prefill: bool):
        if is_prefill:
            seq.num_cached_tokens = min(seq.num_cached_tokens + seq.num_scheduled_tokens, seq.num_tokens)
            # A non-final chunk, or the re-prefill of a preempted sequence, emits nothing.
            if seq.num_cached_tokens < seq.num_tokens or seq.num_completion_tokens > 0:
                seq.num_scheduled_tokens = 0
                return
        seq.append_token(token_id)
        seq.num_cached_tokens += 1
        seq.num_scheduled_tokens = 0
        hit_eos = not seq.ignore_eos and token_id == self.eos
        if hit_eos or seq.num_completion_tokens == seq.max_tokens:
            self._retire(seq)

    def postprocess_speculative(self, seq: Sequence, token_ids: list[int]):
        room = max(seq.max_tokens - seq.num_completion_tokens, 0)
        for token_id in token_ids[:room]:
            seq.append_token(token_id)
            seq.num_cached_tokens += 1
            if not seq.ignore_eos and token_id == self.eos:
                break
        self.block_manager.finalize_full_blocks(seq)
        self.block_manager.release_extra_slots(seq)
        seq.num_scheduled_tokens = 0
        ended_on_eos = (not seq.ignore_eos and seq.num_completion_tokens > 0
                        and seq.token_ids[-1] == self.eos)
        if seq.num_completion_tokens == seq.max_tokens or ended_on_eos:
            self._retire(seq)
