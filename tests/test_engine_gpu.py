"""The engine on one B200: CUDA-graph decode with the overlapped loop (ids fed from the device)
emits exactly the synchronous loop's tokens, including EOS stops found one step late and block
boundaries; and a speculative engine runs through the same graphs' model."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _run(path, overlap, eos=None, **kw):
    from llmserve_b200 import LLM, SamplingParams
    from llmserve_b200.engine.model_runner import GreedySampler
    llm = LLM(path, enforce_eager=False, max_model_len=512, max_num_batched_tokens=2048, max_num_seqs=16,
              kvcache_block_size=16, gpu_memory_utilization=0.3, num_kvcache_blocks=256, overlap_decode=overlap, **kw)
    llm.model_runner.sampler = GreedySampler()
    if eos is not None:
        llm.scheduler.eos = eos
    g = torch.Generator().manual_seed(3)
    prompts = [torch.randint(0, 1024, (int(n),), generator=g).tolist() for n in (33, 7, 100, 16, 64)]
    sps = [SamplingParams(max_tokens=n, ignore_eos=eos is None) for n in (40, 23, 31, 17, 40)]
    out = [o["token_ids"] for o in llm.generate(prompts, sps, use_tqdm=False)]
    n = llm.overlapped_launches
    llm.exit()
    return out, n


@pytest.mark.timeout(600)
def test_overlapped_graph_decode_matches_synchronous(tmp_path):
    from llmserve_b200.models.synthetic import TINY, write_qwen3_checkpoint
    path = write_qwen3_checkpoint(str(tmp_path / "m"), dict(TINY, torch_dtype="bfloat16", num_hidden_layers=4))
    sync, n0 = _run(path, False)
    over, n1 = _run(path, True)
    assert n0 == 0 and n1 > 10
    assert over == sync
    eos = sync[2][5]
    s2, _ = _run(path, False, eos=eos)
    o2, _ = _run(path, True, eos=eos)
    assert o2 == s2 and s2[2][-1] == eos
