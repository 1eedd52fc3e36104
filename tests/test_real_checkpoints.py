"""Real-checkpoint integration, skipped unless the checkpoints are named in the environment:

* ``LLMSERVE_TEST_TARGET_MODEL``       an HF Qwen3 directory (e.g. Qwen3-8B);
* ``LLMSERVE_TEST_SPECULATIVE_MODEL``  an EAGLE3 speculator for it (RedHat or SpecForge layout);
* ``LLMSERVE_TEST_AWQ_MODEL``          an AutoAWQ GEMM group-128 Qwen3 checkpoint.

The same variable names as the reference's tier of real-checkpoint tests, so one environment
drives both suites.
"""
import os

import pytest
import torch

TARGET = os.environ.get("LLMSERVE_TEST_TARGET_MODEL")
DRAFT = os.environ.get("LLMSERVE_TEST_SPECULATIVE_MODEL")
AWQ = os.environ.get("LLMSERVE_TEST_AWQ_MODEL")

needs_eagle3 = pytest.mark.skipif(not (TARGET and DRAFT and os.path.isdir(TARGET) and os.path.isdir(DRAFT)),
                                  reason="set LLMSERVE_TEST_TARGET_MODEL and LLMSERVE_TEST_SPECULATIVE_MODEL")
needs_awq = pytest.mark.skipif(not (AWQ and os.path.isdir(AWQ)), reason="set LLMSERVE_TEST_AWQ_MODEL")


@needs_eagle3
def test_real_speculator_loads_and_runs_a_three_step_cycle():
    """The speculator with the target's embedding: three greedy drafts from the chat start token,
    accepted against verify logits that force the end-of-turn token after them."""
    from llmserve_b200.models.eagle3 import Eagle3Speculator
    from llmserve_b200.speculative.draft import run_eagle3_speculative_cycle
    draft = Eagle3Speculator.from_pretrained(DRAFT, target_model_path=TARGET).float().eval()
    draft.prepare()
    logits = torch.zeros(4, draft.target_vocab_size)
    logits[-1].fill_(float("-inf"))
    logits[-1, 151645] = 0.0
    torch.manual_seed(0)
    res = run_eagle3_speculative_cycle(draft, 151644, torch.zeros(1, 1, 3 * draft.target_hidden_size), 0, logits,
                                       3, 1.0, random_values=torch.zeros(3))
    assert len(res.draft_token_ids) == 3
    assert all(0 <= t < draft.target_vocab_size for t in res.draft_token_ids)
    assert res.sample_result.accepted_all and res.sample_result.token_ids[-1] == 151645


@pytest.mark.gpu
@needs_eagle3
def test_real_models_speculative_tokens_equal_plain_decoding():
    from llmserve_b200 import LLM, SamplingParams
    from llmserve_b200.engine.model_runner import GreedySampler
    prompts = ["The capital of France is", "Explain the KV cache of a transformer in one sentence:"]
    outs = []
    for draft in (None, DRAFT):
        llm = LLM(TARGET, speculative_model=draft, max_model_len=1024, gpu_memory_utilization=0.6)
        llm.model_runner.sampler = GreedySampler()
        outs.append([o["token_ids"] for o in llm.generate(prompts, SamplingParams(max_tokens=48), use_tqdm=False)])
        llm.exit()
    assert outs[0] == outs[1]


@pytest.mark.gpu
@needs_awq
def test_real_awq_checkpoint_generates_with_the_w4a16_kernel():
    from llmserve_b200 import LLM, SamplingParams
    from llmserve_b200.ops._ext import check_status
    llm = LLM(AWQ, max_model_len=512, gpu_memory_utilization=0.5)
    out = llm.generate(["Hello, my name is"], SamplingParams(temperature=0.6, max_tokens=16), use_tqdm=False)
    check_status(torch.device("cuda", 0))
    llm.exit()
    assert len(out[0]["token_ids"]) >= 1
