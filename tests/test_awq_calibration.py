"""Offline AWQ: quantiser, scale / clip search, scale folding, per-layer Qwen3 calibration, the
quantizer CLI (export + resume) and the quality evaluator -- on CPU, against the reference's
functions where importable (reference tests: ``tests/test_awq_quantizer.py``,
``tests/test_qwen3_awq_calibration.py``, ``tests/test_quantize_qwen3_awq_cli.py``,
``tests/test_awq_quality.py``)."""
import copy
import json
import random
from argparse import Namespace
from pathlib import Path

import pytest
import torch
from torch import nn

from llmserve_b200.quantization.awq import dequantize_awq_gemm
from llmserve_b200.quantization.awq_calibration import (apply_awq_clip, fake_quantize_awq_weight, fold_linear_scale,
                                                         fold_rmsnorm_scale, quantize_awq_weight, search_awq_clip,
                                                         search_awq_scale)
from tests.support import reference_module


def _outlier_inputs(t, c, seed=0):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(t, c, generator=g)
    x[:, :: max(1, c // 16)] *= 20.0              # a few salient channels, as AWQ assumes
    return x


def test_quantizer_matches_reference_bitwise():
    ref = reference_module("llmserve.quantization.awq_calibration")
    w = torch.randn(64, 384, generator=torch.Generator().manual_seed(1))
    ours, theirs = quantize_awq_weight(w), ref.quantize_awq_weight(w)
    assert torch.equal(ours.qweight, theirs.qweight)
    assert torch.equal(ours.qzeros, theirs.qzeros)
    torch.testing.assert_close(ours.scales, theirs.scales)
    torch.testing.assert_close(fake_quantize_awq_weight(w), ref.fake_quantize_awq_weight(w))
    deq = dequantize_awq_gemm(ours.qweight, ours.qzeros, ours.scales, group_size=128).t()
    torch.testing.assert_close(deq, fake_quantize_awq_weight(w), rtol=0, atol=1e-6)


def test_scale_search_matches_reference_and_reduces_error():
    ref = reference_module("llmserve.quantization.awq_calibration")
    x = _outlier_inputs(200, 256)
    g = torch.Generator().manual_seed(2)
    ws = [torch.randn(128, 256, generator=g) * 0.02, torch.randn(64, 256, generator=g) * 0.02]
    ours = search_awq_scale(x, ws, n_grid=10)
    theirs = ref.search_awq_scale(x, ws, n_grid=10)
    torch.testing.assert_close(ours, theirs, rtol=1e-4, atol=1e-5)

    def err(s):
        return sum(float((x @ w.t() - x @ (fake_quantize_awq_weight(w * s) / s).t()).pow(2).mean()) for w in ws)
    assert err(ours) < err(torch.ones(256))


def test_clip_search_matches_reference():
    ref = reference_module("llmserve.quantization.awq_calibration")
    x = _outlier_inputs(96, 256, seed=3)
    w = torch.randn(40, 256, generator=torch.Generator().manual_seed(4)) * 0.02
    w[:, 7] *= 8.0                                   # outlier weights make clipping worthwhile
    ours = search_awq_clip(w, x, n_grid=10, output_chunk_size=16)
    theirs = ref.search_awq_clip(w, x, n_grid=10, output_chunk_size=16)
    torch.testing.assert_close(ours, theirs, rtol=1e-5, atol=1e-6)
    assert bool((ours < w.reshape(40, 2, 128).abs().amax(-1, keepdim=True)).any())
    clipped = w.clone()
    apply_awq_clip(clipped, ours)
    assert float(clipped.abs().max()) <= float(ours.max()) + 1e-7


def test_scale_folding_preserves_the_function():
    torch.manual_seed(5)
    norm, a, b, down = nn.RMSNorm(256), nn.Linear(256, 128, bias=False), nn.Linear(256, 64, bias=False), \
        nn.Linear(128, 32, bias=False)
    with torch.no_grad():
        norm.weight.uniform_(0.5, 1.5)
    x = torch.randn(10, 256)
    before = (a(norm(x)), b(norm(x)), down(a(norm(x))))
    s = torch.rand(256) + 0.5
    fold_rmsnorm_scale(norm, [a, b], s)
    fold_linear_scale(a, [down], torch.rand(128) + 0.5)
    after = (a(norm(x)), b(norm(x)), down(a(norm(x))))
    torch.testing.assert_close(after[1], before[1], rtol=1e-4, atol=1e-5)
    torch.testing.assert_close(after[2], before[2], rtol=1e-4, atol=1e-5)


def _tiny_hf_config(layers=2):
    from transformers import Qwen3Config
    return Qwen3Config(vocab_size=512, hidden_size=256, intermediate_size=512, num_hidden_layers=layers,
                       num_attention_heads=4, num_key_value_heads=2, head_dim=64, max_position_embeddings=512,
                       rms_norm_eps=1e-6, rope_theta=1e6, tie_word_embeddings=False, eos_token_id=2)


def test_calibrate_hf_qwen3_layer_writes_quantized_weights():
    from transformers import Qwen3ForCausalLM

    from llmserve_b200.quantization.qwen3_awq import QWEN3_QUANTIZED_LINEAR_NAMES, calibrate_qwen3_layer
    from llmserve_b200.quantization.quantize_qwen3 import capture_first_layer_input
    torch.manual_seed(6)
    model = Qwen3ForCausalLM(_tiny_hf_config()).eval()
    enc = {"input_ids": torch.randint(0, 512, (2, 24)), "attention_mask": torch.ones(2, 24, dtype=torch.long)}
    hidden, kwargs = capture_first_layer_input(model, enc, torch.device("cpu"))
    assert hidden.shape == (2, 24, 256) and "position_embeddings" in kwargs
    layer = model.model.layers[0]
    rtn = copy.deepcopy(layer)
    with torch.no_grad():
        dense_out = layer(hidden, **kwargs)
        for name in QWEN3_QUANTIZED_LINEAR_NAMES:        # round-to-nearest without the AWQ searches
            m = rtn.get_submodule(name)
            m.weight.copy_(fake_quantize_awq_weight(m.weight))
        rtn_out = rtn(hidden, **kwargs)
    res = calibrate_qwen3_layer(layer, hidden, forward_kwargs=kwargs, n_grid=4, max_tokens=32)
    assert set(res.packed_weights) == set(QWEN3_QUANTIZED_LINEAR_NAMES)
    for name, p in res.packed_weights.items():
        w = layer.get_submodule(name).weight
        assert p.qweight.shape == (w.shape[1], w.shape[0] // 8)
        deq = dequantize_awq_gemm(p.qweight, p.qzeros, p.scales, group_size=128).t()
        torch.testing.assert_close(w, deq)
    assert res.evaluated_clip_group_count > 0
    # AWQ's error on the layer's residual update is below plain round-to-nearest's
    upd = (dense_out - hidden).norm()
    awq_err, rtn_err = float((res.hidden_states - dense_out).norm() / upd), float((rtn_out - dense_out).norm() / upd)
    assert awq_err < rtn_err < 0.5, (awq_err, rtn_err)


def _write_hf_checkpoint(path: Path, layers=2):
    from transformers import Qwen3ForCausalLM

    from llmserve_b200.models.synthetic import write_word_tokenizer
    torch.manual_seed(7)
    cfg = _tiny_hf_config(layers)
    model = Qwen3ForCausalLM(cfg).to(torch.bfloat16)
    model.save_pretrained(path)
    write_word_tokenizer(str(path), cfg.vocab_size, 2)
    return path


def _text(path: Path, lines=6, words=40, seed=0):
    rng = random.Random(seed)
    path.write_text("\n".join(" ".join(f"t{rng.randrange(3, 512)}" for _ in range(words)) for _ in range(lines)))
    return path


def test_quantizer_cli_exports_autoawq_and_resumes(tmp_path):
    from llmserve_b200.quantization import quantize_qwen3
    src = _write_hf_checkpoint(tmp_path / "bf16")
    calib = _text(tmp_path / "calib.txt")
    args = quantize_qwen3.build_parser().parse_args(
        ["--model", str(src), "--output", str(tmp_path / "awq"), "--calib-file", str(calib), "--device", "cpu",
         "--n-grid", "4", "--search-tokens", "64", "--max-seq-len", "32"])
    assert args.group_size == 128 and not args.no_clip
    first = quantize_qwen3.run(args)
    assert first["status"] == "complete" and first["completed_layers"] == 2
    cfg = json.loads((tmp_path / "awq" / "config.json").read_text())
    assert cfg["quantization_config"] == {"backend": "autoawq", "bits": 4, "do_fuse": False, "group_size": 128,
                                          "quant_method": "awq", "version": "gemm", "zero_point": True}
    manifest = json.loads((tmp_path / "awq" / "quantization_manifest.json").read_text())
    assert manifest["num_layers"] == 2 and manifest["format"] == "autoawq-gemm"
    from safetensors.torch import load_file
    sd = load_file(str(tmp_path / "awq" / "model.safetensors"))
    assert sd["model.layers.1.mlp.down_proj.qweight"].shape == (512, 256 // 8)
    assert "model.layers.0.self_attn.q_proj.weight" not in sd
    second = quantize_qwen3.run(args)          # everything comes from the layer cache
    assert [second["layers"][str(i)]["status"] for i in range(2)] == ["resumed", "resumed"]
    sd2 = load_file(str(tmp_path / "awq" / "model.safetensors"))
    assert all(torch.equal(sd[k], sd2[k]) for k in sd)
    other = Namespace(**dict(vars(args), n_grid=5))
    with pytest.raises(RuntimeError, match="differ"):
        quantize_qwen3.run(other)

    # the exported checkpoint: quality evaluator (HF + reference W4A16 linears) and our engine
    from llmserve_b200.quantization import awq_quality
    q_args = awq_quality.build_parser().parse_args(
        ["--model", str(tmp_path / "awq"), "--eval-file", str(calib), "--output", str(tmp_path / "q.json"),
         "--device", "cpu", "--sequence-length", "32", "--max-eval-tokens", "96", "--max-new-tokens", "4"])
    res = awq_quality.run(q_args)
    assert res["mode"] == "awq-reference" and res["perplexity"]["tokens"] == 96
    assert 1.0 < res["perplexity"]["perplexity"] < 1e4 and len(res["generations"]) == 2
    b_args = Namespace(**dict(vars(q_args), model=src, output=tmp_path / "b.json"))
    base = awq_quality.run(b_args)
    assert base["mode"] == "bf16"
    # quantisation error on a random model is small: mean NLL within 2% of the bf16 model
    assert abs(res["perplexity"]["mean_nll"] - base["perplexity"]["mean_nll"]) < 0.02 * base["perplexity"]["mean_nll"]

    # the reference runtime accepts the export and dequantises it to the same weights
    ref_awq = reference_module("llmserve.layers.quantization.awq")
    from transformers import AutoConfig
    ref_awq.AWQRuntimeConfig.from_hf_config(AutoConfig.from_pretrained(str(tmp_path / "awq")))
    base_name = "model.layers.1.self_attn.o_proj"
    tensors = [sd[f"{base_name}.{t}"] for t in ("qweight", "qzeros", "scales")]
    torch.testing.assert_close(ref_awq.dequantize_awq_gemm(*tensors, group_size=128),
                               dequantize_awq_gemm(*tensors, group_size=128), rtol=0, atol=0)


def test_layer_calibration_is_as_accurate_as_the_reference_pipeline():
    """The same HF Qwen3 layer and calibration activations through both pipelines: the error of the
    quantised layer's output (relative to its residual update) is within 2% of the reference's
    (this pipeline evaluates its searches in fp32 on an evenly spaced token subsample)."""
    from transformers import Qwen3ForCausalLM

    from llmserve_b200.quantization.qwen3_awq import calibrate_qwen3_layer
    from llmserve_b200.quantization.quantize_qwen3 import capture_first_layer_input
    ref = reference_module("llmserve.quantization.qwen3_awq")
    torch.manual_seed(1)
    model = Qwen3ForCausalLM(_tiny_hf_config()).eval()
    enc = {"input_ids": torch.randint(0, 512, (2, 64)), "attention_mask": torch.ones(2, 64, dtype=torch.long)}
    hidden, kwargs = capture_first_layer_input(model, enc, torch.device("cpu"))
    layer = model.model.layers[0]
    with torch.no_grad():
        dense = layer(hidden, **kwargs)
        dense = dense[0] if isinstance(dense, tuple) else dense
    ours = calibrate_qwen3_layer(copy.deepcopy(layer), hidden, forward_kwargs=kwargs, n_grid=10, max_tokens=128)
    theirs = ref.calibrate_qwen3_layer(copy.deepcopy(layer), hidden, forward_kwargs=kwargs, n_grid=10, max_tokens=128)
    upd = (dense - hidden).norm()
    err_ours = float((ours.hidden_states - dense).norm() / upd)
    err_ref = float((theirs.hidden_states - dense).norm() / upd)
    assert err_ours <= 1.02 * err_ref, (err_ours, err_ref)
