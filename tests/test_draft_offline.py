"""Offline EAGLE3 drafting API: the paged draft K/V pool, serial vs batched drafting with per-request
gammas, contiguous-K/V draft models, one speculative cycle and one offline step."""
import pytest
import torch

from llmserve_b200.models.eagle3 import Eagle3Speculator
from llmserve_b200.models.synthetic import TINY, write_eagle3_checkpoint, write_qwen3_checkpoint
from llmserve_b200.speculative.draft import (STAGES, DraftKVPool, DraftKVRef, generate_eagle3_draft_tokens,
                                             generate_eagle3_draft_tokens_batched, run_eagle3_offline_step,
                                             run_eagle3_speculative_cycle)
from llmserve_b200.speculative.types import Eagle3DraftOutput
from llmserve_b200.utils.context import reset_context, set_context


@pytest.fixture(scope="module")
def draft(tmp_path_factory):
    root = tmp_path_factory.mktemp("draft")
    tgt = write_qwen3_checkpoint(str(root / "t"), TINY)
    model = Eagle3Speculator.from_pretrained(write_eagle3_checkpoint(str(root / "d"), TINY, 512), target_model_path=tgt)
    model.prepare()
    return model


def _aux(batch, width, seed):
    g = torch.Generator().manual_seed(seed)
    return torch.randn(batch, 1, width, generator=g)


def test_pool_slots_growth_trim_and_release():
    pool = DraftKVPool(2, 8, block_size=4, num_blocks=1)
    a, b = pool.new_rows(2)
    slots = []
    for _ in range(6):
        slots += pool.append_slots([a, b])
    assert pool.k.shape[0] >= 4 and len(set(slots)) == 12          # grew, no slot reused
    assert pool.lengths[a] == pool.lengths[b] == 6
    table = pool.block_table([a, b])
    assert table.shape == (2, 2) and table.dtype == torch.int32
    for r, row_slots in ((a, slots[0::2]), (b, slots[1::2])):
        assert row_slots == [pool.blocks[r][p // 4] * 4 + p % 4 for p in range(6)]
    free0 = len(pool.free)
    pool.set_length(a, 3)
    assert len(pool.blocks[a]) == 1 and len(pool.free) == free0 + 1
    with pytest.raises(ValueError):
        pool.set_length(a, 5)
    pool.release(b)
    assert b not in pool.blocks and len(pool.free) == free0 + 3


def test_serial_draft_matches_one_causal_pass(draft):
    """The paged decode steps give the same hidden states as one causal prefill over the same inputs."""
    width = 3 * TINY["hidden_size"]
    pool = DraftKVPool.for_model(draft, "cpu", block_size=2, num_blocks=1)      # forces growth
    ref = DraftKVRef(pool, pool.new_rows(1))
    start_aux = _aux(1, width, 0)
    seq = generate_eagle3_draft_tokens(draft, 17, start_aux, 9, 4, 0.0, past_kv=ref, draft_sampling_mode="greedy")
    assert len(seq.draft_token_ids) == 4 and seq.draft_target_logits.shape == (4, TINY["vocab_size"])
    assert set(seq.proposal_timing) == set(STAGES)
    assert seq.past_kv.lengths == [4]
    # replay the four steps as one prefill: inputs are the start token and the drafted tokens, the
    # start aux row then the draft's own hidden states
    hs, toks = [], []
    ids, aux, pos, past = torch.tensor([[17]]), start_aux, torch.tensor([[9]]), None
    for _ in range(4):
        out = draft.propose(ids, aux, pos, 0.0, past_kv=past)
        hs.append(out.hidden_states[0, 0])
        toks.append(int(out.token_ids))
        ids, aux, pos, past = out.token_ids, out.hidden_states, pos + 1, out.past_kv
    assert toks == seq.draft_token_ids
    pool2 = DraftKVPool.for_model(draft, "cpu")
    (row,) = pool2.new_rows(1)
    slots = [pool2.append_slots([row])[0] for _ in range(4)]
    fc_in = torch.cat([draft.fc(start_aux.reshape(1, -1)), torch.stack(hs[:3])])
    attn = draft.midlayer.self_attn
    bound = attn.k_cache, attn.v_cache
    attn.k_cache, attn.v_cache = pool2.k, pool2.v
    set_context(True, cu_seqlens_q=torch.tensor([0, 4], dtype=torch.int32), max_seqlen_q=4,
                slot_mapping=torch.tensor(slots, dtype=torch.int32), seqlens_k=torch.tensor([4], dtype=torch.int32),
                block_tables=pool2.block_table([row]))
    try:
        tokens = torch.tensor([17, *seq.draft_token_ids[:3]])
        hidden, _ = draft(tokens, fc_in, torch.arange(9, 13))
    finally:
        reset_context()
        attn.k_cache, attn.v_cache = bound
    torch.testing.assert_close(hidden, torch.stack(hs), atol=1e-4, rtol=1e-4)
    k_serial, _ = pool.gather(ref.rows[0])
    k_prefill, _ = pool2.gather(row)
    torch.testing.assert_close(k_serial, k_prefill, atol=1e-4, rtol=1e-4)


def test_batched_equals_serial_with_per_request_gammas(draft):
    width = 3 * TINY["hidden_size"]
    aux = _aux(3, width, 1)
    starts, positions, gammas = [5, 300, 77], [4, 11, 30], [3, 1, 2]
    batch = generate_eagle3_draft_tokens_batched(draft, starts, aux, positions, 3, 0.0,
                                                 draft_sampling_mode="greedy", gammas=gammas)
    for i in range(3):
        one = generate_eagle3_draft_tokens(draft, starts[i], aux[i:i + 1], positions[i], gammas[i], 0.0,
                                           draft_sampling_mode="greedy")
        assert batch[i].draft_token_ids == one.draft_token_ids
        torch.testing.assert_close(batch[i].draft_target_logits, one.draft_target_logits, atol=1e-4, rtol=1e-4)
        assert batch[i].past_kv.lengths == [gammas[i]]
        assert set(batch[i].proposal_timing) == set(STAGES)
    pools = {id(s.past_kv.pool) for s in batch}
    assert len(pools) == 1                                         # one pool, one row per request
    # a second round continues from the returned rows
    more = generate_eagle3_draft_tokens_batched(draft, [s.draft_token_ids[-1] for s in batch], aux, positions, 1,
                                                0.0, past_kv=[s.past_kv for s in batch],
                                                draft_sampling_mode="greedy")
    assert [m.past_kv.lengths[0] for m in more] == [g + 1 for g in gammas]
    with pytest.raises(ValueError):
        generate_eagle3_draft_tokens_batched(draft, [1, 2], aux[:2], [0, 0], 2, 0.0, gammas=[1, 0])


class _ContiguousDraft:
    """A test double with the reference's contiguous K/V: each step appends one position whose
    value is the input token id; logits peak at ``input + 1``."""
    vocab = 64

    def __init__(self):
        self.calls = []

    def propose(self, input_ids, aux_hidden, positions, temperature, past_kv=None, kv_valid_lens=None):
        self.calls.append((input_ids.reshape(-1).tolist(), aux_hidden.shape[-1],
                           None if kv_valid_lens is None else kv_valid_lens.tolist(),
                           None if past_kv is None else past_kv[0].shape[2]))
        B = input_ids.shape[0]
        new = input_ids.float().view(B, 1, 1, 1).expand(B, 1, 1, 2)
        past = new.clone() if past_kv is None else torch.cat([past_kv[0], new], dim=2)
        logits = torch.full((B, 1, self.vocab), -50.0)
        logits[torch.arange(B), 0, (input_ids.reshape(-1) + 1) % self.vocab] = 50.0
        return Eagle3DraftOutput(torch.ones(B, 1, 4), logits, logits, logits.argmax(-1), (past, past.clone()))

    def greedy_sample(self, draft_logits):
        return draft_logits.argmax(-1)


def test_contiguous_kv_is_padded_and_split_per_request():
    model = _ContiguousDraft()
    past = [(torch.full((1, 1, 2, 2), 7.0),) * 2, None, (torch.full((1, 1, 5, 2), 9.0),) * 2]
    out = generate_eagle3_draft_tokens_batched(model, [1, 10, 20], torch.zeros(3, 1, 12), [0, 0, 0], 2, 1.0,
                                               past_kv=past, gammas=[2, 1, 2])
    assert [o.draft_token_ids for o in out] == [[2, 3], [11], [21, 22]]
    assert model.calls[0] == ([1, 10, 20], 12, [2, 0, 5], 5)        # padded to the longest, valid lengths
    assert model.calls[1] == ([2, 21], 4, [3, 6], 6)                # request 1 has finished
    k0 = out[0].past_kv[0][0, 0, :, 0].tolist()
    assert k0 == [7.0, 7.0, 1.0, 2.0]                               # valid prefix + one new position per step
    assert out[1].past_kv[0][0, 0, :, 0].tolist() == [10.0]
    assert out[2].past_kv[0][0, 0, :, 0].tolist() == [9.0] * 5 + [20.0, 21.0]


def test_offline_step_and_cycle(draft):
    width = 3 * TINY["hidden_size"]
    V = TINY["vocab_size"]

    class Target:
        """Verify logits that peak at the next input token, and at 7 after the last one."""

        def __init__(self):
            self.inputs = None

        def parameters(self):
            return iter([torch.zeros(1)])

        def forward_with_eagle3_aux(self, input_ids, positions):
            self.inputs = (input_ids.tolist(), positions.tolist())
            return input_ids, torch.zeros(input_ids.numel(), width)

        def compute_logits(self, hidden):
            nxt = hidden.tolist()[1:] + [7]
            logits = torch.full((len(nxt), V), -100.0)
            logits[torch.arange(len(nxt)), torch.tensor(nxt)] = 100.0
            return logits

    target = Target()
    torch.manual_seed(0)
    res = run_eagle3_offline_step(target, draft, 3, _aux(1, width, 2), 20, 3, 1.0, random_values=torch.zeros(3))
    assert target.inputs == ([3, *res.draft_token_ids], [20, 21, 22, 23])
    assert res.sample_result.accepted_token_ids == res.draft_token_ids
    assert res.sample_result.token_ids == res.draft_token_ids + [7]
    assert res.past_kv.lengths == [3]

    cyc = run_eagle3_speculative_cycle(draft, 3, _aux(1, width, 2), 20, torch.zeros(4, V), 3, 1.0,
                                       random_values=torch.zeros(3))
    assert cyc.sample_result.accepted_all and cyc.sample_result.num_accepted == 3
    assert cyc.draft_target_logits.shape == (3, V)
    with pytest.raises(ValueError):
        run_eagle3_speculative_cycle(draft, 3, _aux(1, width, 2), 20, torch.zeros(3, V), 3, 1.0)


def test_compute_logits_maps_the_draft_head_into_the_target_vocab(draft):
    width = 3 * TINY["hidden_size"]
    out = draft.propose(torch.tensor([[5]]), _aux(1, width, 4), torch.tensor([[3]]), 0.0)
    mapped = draft.compute_logits(out.hidden_states[:, 0])
    torch.testing.assert_close(mapped, out.target_logits[:, 0])
    assert torch.isinf(mapped).sum() == TINY["vocab_size"] - 512


@pytest.mark.parametrize("norm_before_residual", [False, True])
def test_drafts_equal_the_reference_speculator(tmp_path, norm_before_residual):
    """The same EAGLE3 checkpoint (random norm weights too) in both implementations: serial greedy
    drafts give the same tokens and target-vocabulary logits, and so do batched drafts with
    per-request gammas (paged draft K/V here, padded contiguous K/V in the reference)."""
    import json
    import os

    from safetensors.torch import load_file, save_file

    from tests.support import reference_module
    ref_eagle = reference_module("llmserve.models.eagle3")
    target_cfg = dict(TINY, num_hidden_layers=6)          # the reference wants >= 6 target layers
    tgt = write_qwen3_checkpoint(str(tmp_path / "t"), target_cfg)
    d = write_eagle3_checkpoint(str(tmp_path / "d"), target_cfg, 512, seed=5)
    cfg = json.load(open(os.path.join(d, "config.json")))
    cfg["norm_before_residual"] = norm_before_residual
    json.dump(cfg, open(os.path.join(d, "config.json"), "w"))
    sd = load_file(os.path.join(d, "model.safetensors"))
    g = torch.Generator().manual_seed(9)
    for k in sd:
        if k.endswith("norm.weight"):
            sd[k] = 1 + 0.1 * torch.randn(sd[k].shape, generator=g)
    save_file(sd, os.path.join(d, "model.safetensors"))
    ours = Eagle3Speculator.from_pretrained(d, target_model_path=tgt)
    ours.prepare()
    theirs = ref_eagle.Eagle3Speculator.from_pretrained(d, target_model_path=tgt).eval()
    width = 3 * TINY["hidden_size"]
    aux = _aux(3, width, 6)
    with torch.no_grad():
        a = generate_eagle3_draft_tokens(ours, 11, aux[:1], 7, 4, 1.0, draft_sampling_mode="greedy")
        b = ref_eagle.generate_eagle3_draft_tokens(theirs, 11, aux[:1], 7, 4, 1.0, draft_sampling_mode="greedy")
        assert a.draft_token_ids == b.draft_token_ids
        torch.testing.assert_close(a.draft_target_logits, b.draft_target_logits, atol=2e-4, rtol=2e-4)
        gammas = [3, 1, 2]
        xs = generate_eagle3_draft_tokens_batched(ours, [4, 99, 500], aux, [2, 9, 30], 3, 1.0,
                                                  draft_sampling_mode="greedy", gammas=gammas)
        ys = ref_eagle.generate_eagle3_draft_tokens_batched(theirs, [4, 99, 500], aux, [2, 9, 30], 3, 1.0,
                                                            draft_sampling_mode="greedy", gammas=gammas)
    for x, y in zip(xs, ys):
        assert x.draft_token_ids == y.draft_token_ids
        torch.testing.assert_close(x.draft_target_logits, y.draft_target_logits, atol=2e-4, rtol=2e-4)
        assert x.past_kv.lengths[0] == y.past_kv[0].shape[2]


class _FakeTarget:
    """Verify logits over 8 tokens: row j is uniform-ish with a bump at ``(input_j * 3) % 8``."""

    def forward_with_eagle3_aux(self, input_ids, positions):
        h = input_ids.float().unsqueeze(-1).repeat(1, 4)
        return h, torch.cat([h + 1, h + 2, h + 3], -1)

    def compute_logits(self, hidden):
        logits = torch.zeros(hidden.shape[0], 8)
        logits[torch.arange(hidden.shape[0]), (hidden[:, 0].long() * 3) % 8] = 1.5
        return logits


class _FakeDraft:
    """Deterministic draft over 8 tokens whose target-vocabulary logits favour ``step + 2``."""
    hidden_size = 4

    def __init__(self, out_type):
        self.out_type, self.step = out_type, 0

    def propose(self, input_ids, aux_hidden_states, positions, temperature, past_kv=None, kv_valid_lens=None):
        s = self.step
        self.step += 1
        logits = torch.zeros(1, 1, 8)
        logits[0, 0, (s + 2) % 8] = 1.0
        past = (torch.zeros(1, 1, s + 1, 1), torch.zeros(1, 1, s + 1, 1))
        return self.out_type(torch.full((1, 1, 4), float(s)), logits, logits, torch.tensor([[(s + 2) % 8]]), past)


def test_offline_step_and_cycle_equal_the_reference():
    from tests.support import reference_module
    ref_eagle = reference_module("llmserve.models.eagle3")
    for seed in range(6):
        rv = torch.rand(3, generator=torch.Generator().manual_seed(seed))
        torch.manual_seed(seed)
        ours = run_eagle3_offline_step(_FakeTarget(), _FakeDraft(Eagle3DraftOutput), 5, torch.zeros(1, 1, 12), 4, 3,
                                       1.0, random_values=rv)
        torch.manual_seed(seed)
        theirs = ref_eagle.run_eagle3_offline_step(_FakeTarget(), _FakeDraft(ref_eagle.Eagle3DraftOutput), 5,
                                                   torch.zeros(1, 1, 12), 4, 3, 1.0, random_values=rv)
        assert ours.draft_token_ids == theirs.draft_token_ids
        torch.testing.assert_close(ours.verify_output.target_logits, theirs.verify_output.target_logits)
        for f in ("token_ids", "accepted_token_ids", "final_token_id", "num_accepted", "accepted_all"):
            assert getattr(ours.sample_result, f) == getattr(theirs.sample_result, f), (seed, f)
        logits = torch.randn(4, 8, generator=torch.Generator().manual_seed(100 + seed))
        torch.manual_seed(seed)
        a = run_eagle3_speculative_cycle(_FakeDraft(Eagle3DraftOutput), 5, torch.zeros(1, 1, 12), 4, logits, 3, 1.0,
                                         random_values=rv)
        torch.manual_seed(seed)
        b = ref_eagle.run_eagle3_speculative_cycle(_FakeDraft(ref_eagle.Eagle3DraftOutput), 5, torch.zeros(1, 1, 12),
                                                   4, logits, 3, 1.0, random_values=rv)
        assert (a.draft_token_ids, a.sample_result.token_ids) == (b.draft_token_ids, b.sample_result.token_ids)
