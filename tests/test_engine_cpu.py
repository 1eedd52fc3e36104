"""End-to-end engine on the CPU fp32 path.

Tiny random Qwen3-style decoder (2 layers, hidden 256, 4/2 heads, head_dim 64, MLP 512, vocab
1024), 1-layer EAGLE3 draft over aux layers {0, 1, 1} with a 512-token draft vocabulary, paged KV
with block 16 and 64 blocks, prefix caching; 8 requests with prompts of 8-64 uniform random ids
and 32 output tokens, greedy, gamma = 3: speculative output equals non-speculative output token
for token.  Also: chunked prefill, tree speculation, rejection mode, metrics schema, prefix hits.
"""
import os

import pytest
import torch

from llmserve_b200 import LLM, SamplingParams
from llmserve_b200.engine.model_runner import GreedySampler
from llmserve_b200.models.synthetic import TINY, write_eagle3_checkpoint, write_qwen3_checkpoint


@pytest.fixture(scope="module")
def ckpts(tmp_path_factory):
    d = tmp_path_factory.mktemp("ckpt")
    tgt = write_qwen3_checkpoint(str(d / "target"), TINY, seed=0)
    draft = write_eagle3_checkpoint(str(d / "draft"), TINY, draft_vocab=512, seed=0)
    return tgt, draft


def _prompts(n=8, seed=0):
    g = torch.Generator().manual_seed(seed)
    lens = torch.randint(8, 65, (n,), generator=g).tolist()
    return [torch.randint(0, 1024, (L,), generator=g).tolist() for L in lens]


def _run(path, prompts, max_tokens=32, **kw):
    kw.setdefault("num_kvcache_blocks", 64)
    llm = LLM(path, device="cpu", enforce_eager=True, kvcache_block_size=16, max_model_len=256, **kw)
    llm.model_runner.sampler = GreedySampler()
    out = llm.generate(prompts, SamplingParams(temperature=0.5, max_tokens=max_tokens, ignore_eos=True),
                       use_tqdm=False)
    metrics = llm.get_metrics()
    llm.exit()
    return [o["token_ids"] for o in out], metrics


def test_speculative_equals_baseline_config0(ckpts):
    tgt, draft = ckpts
    prompts = _prompts()
    base, _ = _run(tgt, prompts)
    spec, m = _run(tgt, prompts, speculative_model=draft, speculative_gamma=3)
    assert base == spec
    s = m["summary"]["speculative"]
    assert s["steps"] > 0 and s["draft_tokens"] == 3 * s["steps"]
    assert all(len(t) == 32 for t in spec)


def test_chunked_prefill_and_small_budget_match(ckpts):
    tgt, _ = ckpts
    prompts = _prompts(6, seed=3)
    base, _ = _run(tgt, prompts, max_tokens=12)
    chunked, _ = _run(tgt, prompts, max_tokens=12, enable_chunked_prefill=True, max_num_batched_tokens=24)
    assert base == chunked


def test_chunked_prefill_with_speculation(ckpts):
    tgt, draft = ckpts
    prompts = _prompts(5, seed=4)
    base, _ = _run(tgt, prompts, max_tokens=16)
    spec, _ = _run(tgt, prompts, max_tokens=16, enable_chunked_prefill=True, max_num_batched_tokens=40,
                   speculative_model=draft)
    assert base == spec


def test_tree_speculation_equals_baseline(ckpts):
    tgt, draft = ckpts
    prompts = _prompts(1, seed=5)
    base, _ = _run(tgt, prompts, max_tokens=20)
    for nodes in (6, 10):
        tree, m = _run(tgt, prompts, max_tokens=20, speculative_model=draft, speculative_tree_nodes=nodes)
        assert base == tree
        assert m["summary"]["speculative"]["gamma_counts"] == {str(nodes): m["summary"]["speculative"]["steps"]}


def test_rejection_mode_runs_and_emits(ckpts):
    tgt, draft = ckpts
    llm = LLM(tgt, device="cpu", enforce_eager=True, kvcache_block_size=16, max_model_len=256, num_kvcache_blocks=64,
              speculative_model=draft, speculative_accept_mode="rejection", speculative_trace=True)
    out = llm.generate(_prompts(3, seed=6), SamplingParams(temperature=0.8, max_tokens=10, ignore_eos=True),
                       use_tqdm=False)
    req = llm.get_metrics()["requests"]
    llm.exit()
    assert all(len(o["token_ids"]) == 10 for o in out)
    assert any(r["speculative_trace"] for r in req)


def test_prefix_cache_hit_gives_same_tokens(ckpts):
    tgt, _ = ckpts
    shared = list(range(5, 5 + 48))
    prompts = [shared + [7, 8], shared + [9]]
    llm = LLM(tgt, device="cpu", enforce_eager=True, kvcache_block_size=16, max_model_len=256, num_kvcache_blocks=64)
    llm.model_runner.sampler = GreedySampler()
    sp = SamplingParams(max_tokens=6, ignore_eos=True)
    first = llm.generate([prompts[0]], sp, use_tqdm=False)[0]["token_ids"]
    second = llm.generate([prompts[1]], sp, use_tqdm=False)[0]["token_ids"]
    llm.exit()
    fresh, _ = _run(tgt, [prompts[1]], max_tokens=6)
    assert second == fresh[0]
    assert len(first) == 6


def test_metrics_schema_keys(ckpts):
    tgt, _ = ckpts
    _, m = _run(tgt, _prompts(2, seed=8), max_tokens=4)
    s = m["summary"]
    for key in ("num_requests", "num_finished", "num_failed", "total_output_tokens", "wall_time", "throughput",
                "ttft", "burst_itl", "itl", "output_event_latency", "speculative_step_latency", "tpot",
                "request_latency", "speculative", "kv_cache"):
        assert key in s
    for key in ("total_blocks", "used_blocks", "free_blocks", "reserved_blocks", "preemptions",
                "model_runtime_bytes", "kv_cache_bytes"):
        assert key in s["kv_cache"]
    r = m["requests"][0]
    for key in ("seq_id", "prompt_tokens", "output_tokens", "success", "arrival_time", "first_token_time",
                "token_times", "finish_time", "ttft", "burst_itl", "output_event_latency", "latency"):
        assert key in r
    assert s["num_finished"] == 2 and s["tpot"]["p99"] is not None


def test_string_prompt_without_tokenizer_files(ckpts):
    tgt, _ = ckpts
    llm = LLM(tgt, device="cpu", enforce_eager=True, kvcache_block_size=16, max_model_len=256, num_kvcache_blocks=32)
    out = llm.generate(["hello"], SamplingParams(max_tokens=3, ignore_eos=True), use_tqdm=False)
    llm.exit()
    assert len(out[0]["token_ids"]) == 3 and isinstance(out[0]["text"], str)


def test_dummy_load_format_and_reset_metrics(tmp_path):
    from llmserve_b200.models.synthetic import write_config_only
    path = write_config_only(str(tmp_path / "cfg"), TINY)
    llm = LLM(path, device="cpu", load_format="dummy", enforce_eager=True, kvcache_block_size=16, max_model_len=128,
              num_kvcache_blocks=16)
    llm.generate([[1, 2, 3]], SamplingParams(max_tokens=2, ignore_eos=True), use_tqdm=False)
    llm.reset_metrics()
    assert llm.get_metrics()["summary"]["num_requests"] == 0
    llm.exit()


def _run_overlap(path, prompts, overlap, eos=None, max_tokens=(20,), **kw):
    llm = LLM(path, device="cpu", enforce_eager=True, kvcache_block_size=16, max_model_len=256,
              num_kvcache_blocks=kw.pop("num_kvcache_blocks", 64), overlap_decode=overlap, **kw)
    llm.model_runner.sampler = GreedySampler()
    if eos is not None:
        llm.scheduler.eos = eos
    ids = [llm.add_request(p, SamplingParams(temperature=0.5, max_tokens=max_tokens[i % len(max_tokens)],
                                             ignore_eos=eos is None)) for i, p in enumerate(prompts)]
    outs, steps, launched = {}, 0, 0
    while not llm.is_finished():
        done, n = llm.step()
        steps += 1
        outs.update(dict(done))
    m = llm.get_metrics()["summary"]
    llm.exit()
    return [outs[i] for i in ids], m, llm.overlapped_launches


def test_overlapped_decode_matches_synchronous(ckpts):
    """The one-step-ahead decode loop (input ids fed from the device, host work overlapped) emits
    exactly the synchronous loop's tokens: mixed max_tokens, block boundaries (block 16), EOS
    stops found one step late, and a pool small enough that the pipeline has to drain."""
    tgt, _ = ckpts
    prompts = _prompts(6, seed=3)
    base, mb, n0 = _run_overlap(tgt, prompts, False, max_tokens=(20, 7, 33))
    over, mo, n1 = _run_overlap(tgt, prompts, True, max_tokens=(20, 7, 33))
    assert n0 == 0 and n1 > 20
    assert over == base
    assert mo["total_output_tokens"] == mb["total_output_tokens"] and mo["num_finished"] == 6
    # EOS: stop on a token that the synchronous run emits mid-sequence
    eos = base[0][4]
    b2, _, _ = _run_overlap(tgt, prompts, False, eos=eos, max_tokens=(30,))
    o2, m2, _ = _run_overlap(tgt, prompts, True, eos=eos, max_tokens=(30,))
    assert o2 == b2 and len(o2[0]) == 5 and o2[0][-1] == eos
    # tight pool: preemption / drain path
    b3, _, _ = _run_overlap(tgt, prompts, False, max_tokens=(40,), num_kvcache_blocks=14)
    o3, _, n3 = _run_overlap(tgt, prompts, True, max_tokens=(40,), num_kvcache_blocks=14)
    assert o3 == b3 and n3 > 0


def test_pd_disaggregation_matches_single_engine(ckpts):
    """Prefill on one engine, decode on another (both on the CPU tier here), KV blocks pushed
    between their pools: the tokens equal a single engine's; prefix hits in the decode pool are
    reused instead of copied; a small decode pool makes requests wait (parked) without loss."""
    tgt, _ = ckpts
    prompts = _prompts(6, seed=5)
    prompts.append(list(prompts[0]))          # identical prompt: decode-side prefix hit
    base, _ = _run(tgt, prompts, max_tokens=24)
    for blocks in (64, 14):
        llm = LLM(tgt, device="cpu", enforce_eager=True, kvcache_block_size=16, max_model_len=256,
                  num_kvcache_blocks=blocks, pd_disaggregation=True, pd_prefill_devices=(0,), pd_decode_devices=(0,))
        llm.model_runner.sampler = GreedySampler()
        assert llm.prefill.model_runner.sampler.is_greedy
        out = llm.generate(prompts, SamplingParams(temperature=0.5, max_tokens=24, ignore_eos=True))
        m = llm.get_metrics()["summary"]
        llm.exit()
        assert [o["token_ids"] for o in out] == base
        assert m["pd"]["handoffs"] == 7 and m["pd"]["blocks_pushed"] > 0 and m["num_finished"] == 7
        if blocks == 64:
            assert m["pd"]["blocks_reused"] >= 1


def test_debug_bounds_checks_catch_bad_metadata(ckpts):
    """``debug_bounds_checks``: a block id outside the pool or a slot that disagrees with the
    block table is reported on the host before any kernel runs; the same run without corruption
    passes the checks and matches the unchecked run."""
    tgt, _ = ckpts
    prompts = _prompts(3, seed=9)
    base, _ = _run(tgt, prompts, max_tokens=10)
    checked, _ = _run(tgt, prompts, max_tokens=10, debug_bounds_checks=True)
    assert checked == base
    llm = LLM(tgt, device="cpu", enforce_eager=True, kvcache_block_size=16, max_model_len=256, num_kvcache_blocks=64,
              debug_bounds_checks=True)
    llm.model_runner.sampler = GreedySampler()
    llm.add_request(prompts[0], SamplingParams(max_tokens=10, ignore_eos=True))
    llm.step()                                   # prefill
    seq = llm.scheduler.running[0]
    seq.block_table[0] = 64                      # one past the pool
    with pytest.raises(ValueError, match="outside"):
        llm.step()
    seq.block_table[0] = 0
    r = llm.model_runner
    with pytest.raises(ValueError, match="maps to slot"):
        r.check_bounds([seq], [len(seq) - 1], [5])
    llm.exit()


def test_speculative_graph_step_layout_equals_eager_and_baseline(ckpts):
    """The static-buffer step of the EAGLE3 graphs (run as its host emulation here): the same
    tokens as the eager speculative step and as plain decoding, with batches that leave padded
    rows in their bucket and sequences that cross block boundaries."""
    tgt, draft = ckpts
    prompts = _prompts(5, seed=8)
    base, _ = _run(tgt, prompts, max_tokens=40)
    eager, _ = _run(tgt, prompts, max_tokens=40, speculative_model=draft)
    llm = LLM(tgt, device="cpu", enforce_eager=True, kvcache_block_size=16, max_model_len=256, num_kvcache_blocks=64,
              speculative_model=draft, speculative_cuda_graphs=True, debug_bounds_checks=True)
    llm.model_runner.sampler = GreedySampler()
    out = llm.generate(prompts, SamplingParams(temperature=0.5, max_tokens=40, ignore_eos=True), use_tqdm=False)
    sg = llm.model_runner.spec.graphs
    assert sg is not None and sg.steps > 0
    llm.exit()
    graphed = [o["token_ids"] for o in out]
    assert graphed == eager == base


def test_get_metrics_equals_the_reference_summary_of_the_same_run(ckpts):
    """The reference engine's own ``get_metrics`` applied to this engine's request records,
    scheduler and runner (speculation and capacity admission on) returns exactly our metrics."""
    from tests.support import reference_module
    ref_engine = reference_module("llmserve.engine.llm_engine")
    tgt, draft = ckpts
    llm = LLM(tgt, device="cpu", enforce_eager=True, kvcache_block_size=16, max_model_len=256, num_kvcache_blocks=64,
              speculative_model=draft, enable_kv_capacity_admission=True)
    llm.model_runner.sampler = GreedySampler()
    llm.generate(_prompts(3, seed=2), SamplingParams(max_tokens=12, ignore_eos=True), use_tqdm=False)
    ours = llm.get_metrics()
    proxy = ref_engine.LLMEngine.__new__(ref_engine.LLMEngine)
    for k in ("request_metrics", "scheduler", "model_runner", "speculative_batch_calls",
              "speculative_batch_sequences", "speculative_max_batch_size", "last_step_events"):
        object.__setattr__(proxy, k, getattr(llm, k))
    theirs = ref_engine.LLMEngine.get_metrics(proxy)
    llm.exit()
    assert ours["summary"]["speculative"]["steps"] > 0
    assert ours == theirs


@pytest.mark.parametrize("speculative", [False, True, "tree"])
def test_step_is_lockstep_with_the_reference_engine_step(ckpts, speculative):
    """Two engines with the same requests: one steps with ``LLMEngine.step``, the other with the
    reference engine's ``step`` driving its scheduler and runner.  Every step returns the same
    outputs and the same events (timestamps aside), and the request records end identical."""
    from tests.support import reference_module
    ref_engine = reference_module("llmserve.engine.llm_engine")
    tgt, draft = ckpts
    kw = dict(device="cpu", enforce_eager=True, kvcache_block_size=16, max_model_len=256, num_kvcache_blocks=64,
              enable_chunked_prefill=True, max_num_batched_tokens=40, overlap_decode=False,
              speculative_model=draft if speculative else None,
              speculative_tree_nodes=10 if speculative == "tree" else 0)
    ours, driven = LLM(tgt, **kw), LLM(tgt, **kw)
    for e in (ours, driven):
        e.model_runner.sampler = GreedySampler()
    proxy = ref_engine.LLMEngine.__new__(ref_engine.LLMEngine)
    for k in ("request_metrics", "scheduler", "model_runner", "last_step_events"):
        object.__setattr__(proxy, k, getattr(driven, k))
    for k in ("speculative_batch_calls", "speculative_batch_sequences", "speculative_max_batch_size"):
        object.__setattr__(proxy, k, 0)
    sp = SamplingParams(max_tokens=10, ignore_eos=True)
    for p in _prompts(1 if speculative == "tree" else 4, seed=5):
        ours.add_request(p, sp)
        driven.add_request(p, sp)
    # sequence ids come from one process-wide counter: compare them by arrival order
    order_ours = {sid: i for i, sid in enumerate(ours.request_metrics)}
    order_driven = {sid: i for i, sid in enumerate(driven.request_metrics)}

    def norm(events, order):
        return {k: ([order[x] for x in v] if k.endswith("seq_ids") else v) for k, v in events.items()
                if k not in ("step_start", "step_end", "speculative_debug", "speculative_debug_by_seq")}

    steps = 0
    while not ours.is_finished():
        a, b = ours.step(), ref_engine.LLMEngine.step(proxy)
        assert a[1] == b[1] and [t for _, t in a[0]] == [t for _, t in b[0]], steps
        assert norm(ours.last_step_events, order_ours) == norm(proxy.last_step_events, order_driven), steps
        steps += 1
    assert driven.is_finished() and steps > 3
    fields = ("output_tokens", "prompt_tokens", "success", "speculative_steps", "speculative_draft_tokens",
              "speculative_accepted_tokens", "speculative_emitted_tokens", "speculative_accept_all_count",
              "speculative_gamma_counts")
    rec = [[m[f] for f in fields] + [len(m["token_times"]), len(m["output_event_times"])]
           for m in ours.request_metrics.values()]
    assert rec == [[m[f] for f in fields] + [len(m["token_times"]), len(m["output_event_times"])]
                   for m in driven.request_metrics.values()]
    assert ours.speculative_batch_calls == proxy.speculative_batch_calls
    ours.exit()
    driven.exit()


def test_pd_disaggregation_with_eagle3_keeps_the_draft_state(ckpts):
    """Prefill/decode disaggregation with an EAGLE3 draft: the draft's prompt K/V and its length move
    with each sequence, so the decode side drafts exactly what a single speculative engine drafts
    (same draft tokens step by step) and the output equals plain decoding."""
    tgt, draft = ckpts
    prompts = _prompts(4, seed=9)
    base, _ = _run(tgt, prompts, max_tokens=16)
    kw = dict(device="cpu", enforce_eager=True, kvcache_block_size=16, max_model_len=256, num_kvcache_blocks=64,
              speculative_model=draft, speculative_trace=True)
    runs = []
    for pd in (False, True):
        extra = dict(pd_disaggregation=True, pd_prefill_devices=(0,), pd_decode_devices=(0,)) if pd else {}
        llm = LLM(tgt, **kw, **extra)
        llm.model_runner.sampler = GreedySampler()
        out = llm.generate(prompts, SamplingParams(temperature=0.5, max_tokens=16, ignore_eos=True), use_tqdm=False)
        m = llm.get_metrics()
        llm.exit()
        drafts = [[e["draft_token_ids"] for e in r["speculative_trace"]] for r in m["requests"]]
        runs.append(([o["token_ids"] for o in out], drafts, m["summary"]))
    (single, d_single, _), (pd_out, d_pd, summary) = runs
    assert single == base and pd_out == base
    assert d_pd == d_single and any(d_single)
    assert summary["pd"]["handoffs"] == 4 and summary["speculative"]["steps"] > 0


def test_awq_target_with_eagle3_equals_awq_plain_decoding(tmp_path, ckpts):
    """An AutoAWQ W4A16 target with an EAGLE3 draft (the reference runs AWQ eager, TP 1, and its
    speculation separately): speculative output equals the AWQ target's plain decoding."""
    from llmserve_b200.models.synthetic import write_awq_checkpoint
    _, draft = ckpts
    awq = write_awq_checkpoint(str(tmp_path / "awq"), TINY, seed=3)
    prompts = _prompts(3, seed=1)
    base, _ = _run(awq, prompts, max_tokens=12)
    spec, m = _run(awq, prompts, max_tokens=12, speculative_model=draft)
    assert spec == base and m["summary"]["speculative"]["steps"] > 0


def test_host_engine_logits_equal_fp32_transformers_forward(tmp_path):
    """The host (fp32) engine's logits at every step -- prefill over the paged pool, then decode
    steps crossing block boundaries -- equal transformers' Qwen3 forward of the same weights,
    teacher-forced on the engine's tokens (an implementation independent of this one)."""
    import glob

    from safetensors.torch import load_file
    from transformers import Qwen3Config, Qwen3ForCausalLM

    from tests.support import RecordingSampler, compare_logits
    cfg = dict(TINY, torch_dtype="bfloat16", num_hidden_layers=2)
    path = write_qwen3_checkpoint(str(tmp_path / "m"), cfg)
    g = torch.Generator().manual_seed(11)
    prompts = [torch.randint(0, cfg["vocab_size"], (int(n),), generator=g).tolist() for n in (33, 7, 40)]
    n_out = 12
    llm = LLM(path, device="cpu", enforce_eager=True, max_model_len=256, max_num_batched_tokens=1024, max_num_seqs=4,
              kvcache_block_size=16, num_kvcache_blocks=64)
    rec = RecordingSampler()
    llm.model_runner.sampler = rec
    out = [o["token_ids"] for o in llm.generate(prompts, SamplingParams(max_tokens=n_out, ignore_eos=True),
                                                use_tqdm=False)]
    llm.exit()
    sd = {}
    for f in glob.glob(f"{path}/*.safetensors"):
        sd.update(load_file(f))
    model = Qwen3ForCausalLM(Qwen3Config(**{k: v for k, v in cfg.items() if k not in ("architectures", "torch_dtype")}))
    model.float().eval().load_state_dict({k: v.float() for k, v in sd.items()}, strict=True)
    ref = [torch.empty_like(x) for x in rec.logits]
    with torch.no_grad():
        for i, (p, toks) in enumerate(zip(prompts, out)):
            full = model(torch.tensor([p + toks[:-1]])).logits[0]
            for j in range(n_out):
                ref[j][i] = full[len(p) - 1 + j]
    worst, _ = compare_logits(rec.logits, ref, 1e-4)
    assert worst < 1e-5
