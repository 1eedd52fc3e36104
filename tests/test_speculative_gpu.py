"""EAGLE3 speculative decoding on one B200 (bf16 kernels, random target and speculator).

Greedy verification makes speculative output a function of the target model alone, so it must
equal plain greedy decoding.  On the GPU the verify pass (packed gamma + 1 tokens per sequence,
prefill attention) and the plain decode pass (one token, decode attention) round differently in
bf16, so a token may legitimately differ where the target's top two logits are a near-tie.  The
checks:

* eager and CUDA-graphed speculative steps emit identical tokens (same kernels, same shapes);
* speculative output equals plain decoding; where they differ, both must be greedy decodings of
  the target: every token of each is the argmax of an fp32 Hugging Face forward of the same
  weights over its own prefix, or within a small band of it (a bf16 near-tie);
* the speculative counters show the draft ran (gamma drafts per step).
"""
import pytest
import torch

pytestmark = pytest.mark.gpu

GAMMA = 3


@pytest.fixture(scope="module")
def ckpts(tmp_path_factory):
    from safetensors.torch import save_file

    from llmserve_b200.models.synthetic import TINY, qwen3_state_dict, write_config_only, write_eagle3_checkpoint
    d = tmp_path_factory.mktemp("spec")
    cfg = dict(TINY, torch_dtype="bfloat16", num_hidden_layers=4)
    tgt = write_config_only(str(d / "target"), cfg)
    # std 0.05: varied greedy continuations that depend on attention (0.02 mostly repeats a token)
    save_file(qwen3_state_dict(cfg, seed=1, std=0.05), str(d / "target" / "model.safetensors"))
    draft = write_eagle3_checkpoint(str(d / "draft"), cfg, draft_vocab=512, seed=1)
    return tgt, draft


def _prompts(n=6, seed=0):
    g = torch.Generator().manual_seed(seed)
    return [torch.randint(0, 1024, (int(L),), generator=g).tolist() for L in torch.randint(8, 90, (n,), generator=g)]


def _generate(path, prompts, max_tokens, **kw):
    from llmserve_b200 import LLM, SamplingParams
    from llmserve_b200.engine.model_runner import GreedySampler
    llm = LLM(path, enforce_eager=False, max_model_len=512, max_num_batched_tokens=2048, max_num_seqs=16,
              kvcache_block_size=16, gpu_memory_utilization=0.3, num_kvcache_blocks=256, **kw)
    llm.model_runner.sampler = GreedySampler()
    out = [o["token_ids"] for o in llm.generate(prompts, SamplingParams(max_tokens=max_tokens, ignore_eos=True),
                                                 use_tqdm=False)]
    spec = llm.get_metrics()["summary"]["speculative"]
    llm.exit()
    return out, spec


_HF = {}


def _hf_logits(path, ids):
    """Last-position logits of an fp32 Hugging Face Qwen3 forward (CPU) over the same weights."""
    import glob
    import os

    from safetensors.torch import load_file
    from transformers import Qwen3Config, Qwen3ForCausalLM
    if path not in _HF:
        model = Qwen3ForCausalLM(Qwen3Config.from_pretrained(path)).float().eval()
        sd = {}
        for f in sorted(glob.glob(os.path.join(path, "*.safetensors"))):
            sd.update(load_file(f))
        missing, unexpected = model.load_state_dict({k: v.float() for k, v in sd.items()}, strict=False)
        assert not unexpected and all("rotary" in k for k in missing), (missing, unexpected)
        _HF[path] = model
    with torch.no_grad():
        return _HF[path](torch.tensor([ids])).logits[0, -1].float()


def _hf_all_logits(path, ids):
    _hf_logits(path, ids[:1])                    # builds and caches the model
    with torch.no_grad():
        return _HF[path](torch.tensor([ids])).logits[0].float()


def _check_greedy_against_fp32(path, prompts, outputs, band=0.15):
    """Every emitted token must be the fp32 argmax of the target given the sequence's own prefix,
    or within ``band`` logit standard deviations of it (a bf16 near-tie).  One causal forward per
    sequence yields the logits at every position."""
    for p, out in zip(prompts, outputs):
        logits = _hf_all_logits(path, p + out)
        for j, tok in enumerate(out):
            row = logits[len(p) + j - 1]
            gap = float(row.max() - row[tok])
            assert gap <= band * float(row.std()), (
                f"token {j} = {tok} is {gap:.4f} below the fp32 maximum (logit std {float(row.std()):.4f}): "
                "not greedy decoding of the target")


def _check_equal_or_near_tie(path, prompts, plain, spec, band=0.15):
    """Speculative output against plain decoding: identical, or both are greedy decodings of the
    target that part at a near-tie (each checked token by token against the fp32 forward)."""
    assert [len(a) for a in plain] == [len(b) for b in spec]
    if plain != spec:
        _check_greedy_against_fp32(path, prompts, plain, band)
        _check_greedy_against_fp32(path, prompts, spec, band)


@pytest.mark.timeout(900)
def test_eagle3_eager_and_graphed_equal_plain_decoding(ckpts):
    tgt, draft = ckpts
    prompts = _prompts()
    plain, _ = _generate(tgt, prompts, 48)
    eager, s_eager = _generate(tgt, prompts, 48, speculative_model=draft, speculative_gamma=GAMMA)
    graphed, s_graph = _generate(tgt, prompts, 48, speculative_model=draft, speculative_gamma=GAMMA,
                                 speculative_cuda_graphs=True)
    assert graphed == eager
    for s in (s_eager, s_graph):
        assert s["steps"] > 0 and s["draft_tokens"] == GAMMA * s["steps"]
    _check_equal_or_near_tie(tgt, prompts, plain, eager)


@pytest.mark.timeout(900)
def test_eagle3_tree_equals_plain_decoding(ckpts):
    tgt, draft = ckpts
    prompts = _prompts(1, seed=4)
    plain, _ = _generate(tgt, prompts, 40)
    tree, s = _generate(tgt, prompts, 40, speculative_model=draft, speculative_tree_nodes=10)
    assert s["steps"] > 0
    _check_equal_or_near_tie(tgt, prompts, plain, tree)
