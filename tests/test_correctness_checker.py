"""``check_speculative_correctness.py`` end to end on the CPU fp32 engine (tiny Qwen3 + EAGLE3 draft,
the BASELINE config-0 shapes) and its check logic with hand-made results (reference tests:
``tests/test_check_speculative_correctness.py``)."""
import json

import pytest

import check_speculative_correctness as csc
from llmserve_b200.models.synthetic import TINY, write_eagle3_checkpoint, write_qwen3_checkpoint


@pytest.fixture(scope="module")
def ckpts(tmp_path_factory):
    d = tmp_path_factory.mktemp("csc")
    return (write_qwen3_checkpoint(str(d / "target"), TINY, seed=0),
            write_eagle3_checkpoint(str(d / "draft"), TINY, draft_vocab=512, seed=0))


def _factory(model, **kw):
    from llmserve_b200 import LLM
    return LLM(model, kvcache_block_size=16, num_kvcache_blocks=64, **kw)


def test_single_prompt_tokens_match_on_cpu(ckpts, tmp_path):
    tgt, draft = ckpts
    out = tmp_path / "r.json"
    rc = csc.main(["--model", tgt, "--speculative-model", draft, "--device", "cpu", "--argmax-sampler",
                   "--prompt-token-ids", "5,17,300,41,9,77", "--output-len", "12", "--max-model-len", "128",
                   "--require-token-match", "--output-json", str(out)], engine_factory=_factory)
    report = json.loads(out.read_text())
    assert rc == 0, report["checks"]
    assert report["checks"]["token_ids_match"] and len(report["baseline"]["token_ids"]) == 12
    assert report["speculative"]["metrics"]["summary"]["speculative"]["steps"] > 0


def test_batch_consistency_on_cpu(ckpts):
    tgt, draft = ckpts
    args = csc.build_parser().parse_args(["--model", tgt, "--speculative-model", draft, "--device", "cpu",
                                          "--batch-consistency", "--batch-sizes", "2,3", "--output-len", "8",
                                          "--max-model-len", "128", "--max-num-batched-tokens", "256"])
    report = csc.run_batch_consistency(args, engine_factory=_factory)
    assert report["required_checks_pass"], [b["checks"] for b in report["batches"]]
    assert [b["batch_size"] for b in report["batches"]] == [2, 3]


def test_check_logic_flags_bad_metrics():
    good = {"summary": {"num_finished": 1, "num_failed": 0, "total_output_tokens": 3,
                        "speculative": {"steps": 1, "draft_tokens": 3, "accepted_tokens": 2, "emitted_tokens": 3,
                                        "acceptance_rate": 2 / 3}}}
    base = csc.RunResult([1, 2, 3], {"summary": dict(good["summary"], speculative={})}, [])
    spec = csc.RunResult([1, 2, 4], good, [])
    c = csc.build_checks(base, spec, 3)
    assert c["required_checks_pass"] and not c["token_ids_match"]
    bad = json.loads(json.dumps(good))
    bad["summary"]["speculative"]["accepted_tokens"] = 5
    assert not csc.build_checks(base, csc.RunResult([1, 2, 3], bad, []), 3)["required_checks_pass"]
    assert csc.parse_batch_sizes("4,2,2") == [2, 4]
    with pytest.raises(ValueError):
        csc.parse_token_ids(" , ")


def test_graphed_speculative_step_tokens_match_on_cpu(ckpts, tmp_path):
    """``--speculative-cuda-graphs``: the speculative engine takes the graphed chain step (its
    static-buffer emulation on the CPU tier) and still matches plain decoding token for token."""
    tgt, draft = ckpts
    out = tmp_path / "g.json"
    rc = csc.main(["--model", tgt, "--speculative-model", draft, "--device", "cpu", "--argmax-sampler",
                   "--speculative-cuda-graphs", "--prompt-token-ids", "8,19,301,44,2,70,5", "--output-len", "14",
                   "--max-model-len", "128", "--require-token-match", "--output-json", str(out)],
                  engine_factory=_factory)
    report = json.loads(out.read_text())
    assert rc == 0, report["checks"]
    assert report["checks"]["token_ids_match"] and len(report["baseline"]["token_ids"]) == 14
