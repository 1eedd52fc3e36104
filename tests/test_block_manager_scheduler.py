"""Sequence / BlockManager / Scheduler: behaviour tests and step-by-step parity with the
reference implementation on random workloads (default, chunked prefill, capacity admission,
preemption, speculative slot helpers)."""
import random
import zlib
from types import SimpleNamespace

import pytest

from llmserve_b200.engine.block_manager import BlockManager
from llmserve_b200.engine.scheduler import Scheduler, SchedulerOutput
from llmserve_b200.engine.sequence import Sequence, SequenceStatus
from llmserve_b200.sampling_params import SamplingParams
from tests.support import reference_module


def _cfg(**kw):
    base = dict(max_num_seqs=8, max_num_batched_tokens=64, eos=2, num_kvcache_blocks=24, kvcache_block_size=16,
                enable_chunked_prefill=False, enable_kv_capacity_admission=False, max_model_len=512,
                speculative_gamma=3, speculative_model=None)
    base.update(kw)
    return SimpleNamespace(**base)


@pytest.fixture(autouse=True)
def _block16():
    old = Sequence.block_size
    Sequence.block_size = 16
    yield
    Sequence.block_size = old


def test_sampling_params_rejects_greedy():
    with pytest.raises(ValueError):
        SamplingParams(temperature=0.0)


def test_prefix_cache_hits_full_blocks_only():
    bm = BlockManager(8, 16)
    a = Sequence(list(range(40)))
    bm.allocate(a)
    assert a.num_cached_tokens == 0 and len(a.block_table) == 3
    b = Sequence(list(range(32)) + [999, 998])
    bm.allocate(b)
    assert b.num_cached_tokens == 32
    assert b.block_table[:2] == a.block_table[:2] and b.block_table[2] != a.block_table[2]
    assert bm.blocks[a.block_table[0]].ref_count == 2
    bm.deallocate(a)
    bm.deallocate(b)
    assert len(bm.free_block_ids) == 8


def test_speculative_slot_helpers():
    bm = BlockManager(6, 16)
    s = Sequence(list(range(15)))
    bm.allocate(s)
    assert bm.ensure_slots(s, 5)            # 15 + 5 -> 2 blocks
    assert len(s.block_table) == 2
    for t in range(3):
        s.append_token(100 + t)
    bm.finalize_full_blocks(s)
    assert bm.blocks[s.block_table[0]].hash != -1
    bm.release_extra_slots(s)
    assert len(s.block_table) == s.num_blocks == 2
    other = [Sequence(list(range(16 * 2))) for _ in range(2)]
    for o in other:
        bm.allocate(o)
    assert not bm.ensure_slots_batch(other, 17)   # needs 4 blocks, none free -> no change
    assert all(len(o.block_table) == 2 for o in other)


def _overscheduled(out):
    """The reference keeps a prefill's pre-prefix-hit token count; this engine does not."""
    return any(s.num_scheduled_tokens > max(s.num_tokens - s.num_cached_tokens, 1) for s in out.prefill_seqs)


def _snapshot(sched, out):
    return ([s.seq_id for s in out.prefill_seqs], [s.seq_id for s in out.decode_seqs],
            [(s.seq_id, list(s.block_table), s.num_cached_tokens, s.num_scheduled_tokens) for s in out.scheduled_seqs],
            out.num_batched_tokens)


def _drive(sched_cls, seq_cls, cfg, workload, eos, steps, spec_every=0):
    rng = random.Random(1234)
    sched = sched_cls(cfg)
    seqs = []
    trace = []
    pending = list(workload)
    for step in range(steps):
        while pending and pending[0][0] <= step:
            _, prompt, max_tokens = pending.pop(0)
            seq = seq_cls(prompt, SimpleNamespace(temperature=1.0, max_tokens=max_tokens, ignore_eos=False))
            seqs.append(seq)
            sched.add(seq)
        if sched.is_finished():
            continue
        out = sched.schedule()
        if _overscheduled(out):
            trace.append("DIVERGE")
            break
        trace.append(_snapshot(sched, out))
        if spec_every and not out.prefill_seqs and step % spec_every == 0:
            bm = sched.block_manager
            if bm.ensure_slots_batch(out.scheduled_seqs, cfg.speculative_gamma + 2):
                for s in out.scheduled_seqs:
                    sched.postprocess_speculative(s, [rng.randrange(3, 50) for _ in range(rng.randrange(1, 5))])
                trace.append([(s.seq_id, list(s.block_table), s.num_tokens) for s in out.scheduled_seqs])
                continue
        tokens = [eos if rng.random() < 0.05 else rng.randrange(3, 50) for _ in out.scheduled_seqs]
        sched.postprocess(out, tokens)
        trace.append([(s.seq_id, s.status.name, s.num_tokens) for s in out.scheduled_seqs])
    return trace


def _workload(n, rng, max_prompt=80):
    return [(rng.randrange(0, 30), [rng.randrange(3, 50) for _ in range(rng.randrange(1, max_prompt))],
             rng.randrange(1, 40)) for _ in range(n)]


@pytest.mark.parametrize("variant", ["default", "chunked", "admission", "tight", "speculative"])
def test_scheduler_matches_reference_step_by_step(variant):
    ref_sched = reference_module("llmserve.engine.scheduler")
    ref_seq = reference_module("llmserve.engine.sequence")
    kw = {"default": {}, "chunked": {"enable_chunked_prefill": True},
          "admission": {"enable_kv_capacity_admission": True, "num_kvcache_blocks": 40},
          "tight": {"num_kvcache_blocks": 10, "max_num_batched_tokens": 48},
          "speculative": {"speculative_model": "draft", "num_kvcache_blocks": 40}}[variant]
    rng = random.Random(zlib.crc32(variant.encode()))
    work = sorted(_workload(24, rng), key=lambda w: w[0])
    ours = _drive(Scheduler, Sequence, _cfg(**kw), work, 2, 160, spec_every=3 if variant == "speculative" else 0)
    ref_seq.Sequence.block_size = 16
    ref_seq.Sequence.counter = iter(range(next(Sequence.counter) + 1000000, 10**9))
    # align id spaces: compare traces with ids renumbered by first appearance
    theirs = _drive(ref_sched.Scheduler, ref_seq.Sequence, _cfg(**kw), work, 2, 160,
                    spec_every=3 if variant == "speculative" else 0)
    if "DIVERGE" in theirs:
        cut = theirs.index("DIVERGE")
        theirs, ours = theirs[:cut], ours[:cut]
    assert len(theirs) >= 40, "compared prefix too short to be meaningful"
    assert _renumber(ours) == _renumber(theirs)


def _renumber(trace):
    ids = {}

    def rid(x):
        return ids.setdefault(x, len(ids))

    def walk(v, key_is_id=False):
        if isinstance(v, tuple):
            return tuple(rid(v[0]) if i == 0 and isinstance(v[0], int) else walk(x) for i, x in enumerate(v))
        if isinstance(v, list):
            return [walk(x) for x in v]
        return v
    out = []
    for entry in trace:
        if entry == "DIVERGE":
            out.append(entry)
            continue
        if isinstance(entry, tuple) and len(entry) == 4:
            pre, dec, rows, n = entry
            out.append(([rid(i) for i in pre], [rid(i) for i in dec], walk(rows), n))
        else:
            out.append(walk(entry))
    return out


def test_chunked_prefill_is_decode_first():
    sched = Scheduler(_cfg(enable_chunked_prefill=True, max_num_batched_tokens=20))
    a = Sequence(list(range(3, 13)), SamplingParams(max_tokens=5))
    sched.add(a)
    out = sched.schedule()
    sched.postprocess(out, [7])
    b = Sequence(list(range(3, 60)), SamplingParams(max_tokens=5))
    sched.add(b)
    out = sched.schedule()
    assert out.decode_seqs == [a] and out.prefill_seqs == [b]
    assert b.num_scheduled_tokens == 19 and out.num_batched_tokens == 20


def test_capacity_admission_defers_instead_of_preempting():
    sched = Scheduler(_cfg(enable_kv_capacity_admission=True, num_kvcache_blocks=6))
    big = [Sequence(list(range(3, 35)), SamplingParams(max_tokens=40)) for _ in range(3)]
    for s in big:
        sched.add(s)
    out = sched.schedule()
    assert len(out.prefill_seqs) == 1
    assert sched.admission_deferred_count >= 1
    m = sched.kv_capacity_metrics()
    assert m["reserved_blocks"] == 5 and m["enabled"]
    with pytest.raises(ValueError):
        sched.add(Sequence(list(range(3, 200)), SamplingParams(max_tokens=10)))


def test_scheduler_output_validation():
    s = Sequence([1, 2, 3])
    with pytest.raises(ValueError):
        SchedulerOutput([s], [], [], 1)


def test_sequence_pickle_ships_minimal_state():
    import pickle
    s = Sequence(list(range(5)), SamplingParams(max_tokens=3, temperature=0.5))
    s.num_cached_tokens = 5
    s.append_token(9)
    s.num_cached_tokens = 6
    w = pickle.loads(pickle.dumps(s))
    assert w.token_ids == [] and w.last_token == 9 and len(w) == 6 and w.seq_id == s.seq_id
    assert w.temperature == 0.5 and w.status == SequenceStatus.RUNNING


def _running(sched, prompt, max_tokens, ignore_eos=False):
    seq = Sequence(prompt, SamplingParams(max_tokens=max_tokens, ignore_eos=ignore_eos))
    sched.add(seq)
    out = sched.schedule()
    sched.postprocess(out, [7] * len(out.scheduled_seqs))          # prefill samples its first token
    return seq


def test_postprocess_speculative_appends_stops_at_eos_and_max_tokens():
    sched = Scheduler(_cfg(enable_kv_capacity_admission=True))
    bm = sched.block_manager
    a = _running(sched, list(range(3, 18)), 10)                      # 15 prompt + 1 sampled = 16 tokens
    assert bm.ensure_slots(a, 6)                                     # reserves a second block
    sched.postprocess_speculative(a, [11, 12, 13])
    assert a.token_ids[-3:] == [11, 12, 13] and a.num_cached_tokens == len(a) and not a.is_finished
    assert len(a.block_table) == a.num_blocks                         # unused reserved blocks released
    assert bm.blocks[a.block_table[0]].hash != -1                      # the full block got its hash
    # tokens after an EOS are dropped and the sequence retires (its reservation too)
    assert bm.ensure_slots(a, 4)
    sched.postprocess_speculative(a, [14, 2, 15])
    assert a.token_ids[-2:] == [14, 2] and a.is_finished and a.seq_id not in sched._reserved_blocks
    # max_tokens caps what is appended
    b = _running(sched, list(range(3, 10)), 3)
    assert bm.ensure_slots(b, 4)
    sched.postprocess_speculative(b, [20, 21, 22, 23])
    assert b.num_completion_tokens == 3 and b.token_ids[-2:] == [20, 21] and b.is_finished
    # ignore_eos keeps going through an EOS
    c = _running(sched, list(range(3, 10)), 8, ignore_eos=True)
    assert bm.ensure_slots(c, 4)
    sched.postprocess_speculative(c, [2, 2, 30])
    assert c.token_ids[-3:] == [2, 2, 30] and not c.is_finished
