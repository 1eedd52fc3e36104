"""Synthetic checkpoints with the real tensor names, shapes and formats.

There is no network for downloading Qwen3 / EAGLE3 / AWQ checkpoints, so tests and benchmarks
write random-init ones: HF Qwen3 safetensors (``model.layers.N.self_attn.q_proj.weight`` ...),
a RedHat-style nested EAGLE3 speculator directory (``layers.0.*`` names, ``d2t``/``t2d``), and
AutoAWQ GEMM group-128 tensors.  ``write_config_only`` produces a directory with just
``config.json`` for ``load_format="dummy"`` (weights drawn on the device).
"""
import json
import os

import torch
from safetensors.torch import save_file

from llmserve_b200.quantization.awq import pack_awq_int4

QWEN3_8B = dict(
    architectures=["Qwen3ForCausalLM"], model_type="qwen3", hidden_size=4096, intermediate_size=12288,
    num_hidden_layers=36, num_attention_heads=32, num_key_value_heads=8, head_dim=128, vocab_size=151936,
    max_position_embeddings=40960, rope_theta=1000000.0, rms_norm_eps=1e-6, hidden_act="silu",
    attention_bias=False, tie_word_embeddings=False, torch_dtype="bfloat16", bos_token_id=151643,
    eos_token_id=151645,
)

TINY = dict(
    architectures=["Qwen3ForCausalLM"], model_type="qwen3", hidden_size=256, intermediate_size=512,
    num_hidden_layers=2, num_attention_heads=4, num_key_value_heads=2, head_dim=64, vocab_size=1024,
    max_position_embeddings=4096, rope_theta=1000000.0, rms_norm_eps=1e-6, hidden_act="silu",
    attention_bias=False, tie_word_embeddings=False, torch_dtype="float32", bos_token_id=1, eos_token_id=2,
)

EAGLE3_8B = dict(
    draft_vocab_size=32000, target_hidden_size=4096, norm_before_residual=False,
    transformer_layer_config=dict(hidden_size=4096, intermediate_size=12288, num_attention_heads=32,
                                  num_key_value_heads=8, head_dim=128, vocab_size=151936,
                                  max_position_embeddings=40960, rope_theta=1000000.0, rms_norm_eps=1e-6),
)

_DT = {"float32": torch.float32, "bfloat16": torch.bfloat16}


def write_config_only(path: str, config: dict):
    os.makedirs(path, exist_ok=True)
    with open(os.path.join(path, "config.json"), "w") as f:
        json.dump(config, f, indent=2)
    return path


def qwen3_state_dict(config: dict, seed: int = 0, std: float = 0.02, dtype=None) -> dict:
    g = torch.Generator().manual_seed(seed)
    dtype = dtype or _DT[config["torch_dtype"]]
    H, I, V = config["hidden_size"], config["intermediate_size"], config["vocab_size"]
    nh, nkv, hd = config["num_attention_heads"], config["num_key_value_heads"], config["head_dim"]

    def rnd(*shape):
        return (torch.randn(*shape, generator=g) * std).to(dtype)

    def near_one(n):
        return (1 + 0.1 * torch.randn(n, generator=g)).to(dtype)

    sd = {"model.embed_tokens.weight": rnd(V, H), "model.norm.weight": near_one(H)}
    if not config.get("tie_word_embeddings"):
        sd["lm_head.weight"] = rnd(V, H)
    for i in range(config["num_hidden_layers"]):
        p = f"model.layers.{i}."
        sd[p + "self_attn.q_proj.weight"] = rnd(nh * hd, H)
        sd[p + "self_attn.k_proj.weight"] = rnd(nkv * hd, H)
        sd[p + "self_attn.v_proj.weight"] = rnd(nkv * hd, H)
        sd[p + "self_attn.o_proj.weight"] = rnd(H, nh * hd)
        sd[p + "self_attn.q_norm.weight"] = near_one(hd)
        sd[p + "self_attn.k_norm.weight"] = near_one(hd)
        sd[p + "mlp.gate_proj.weight"] = rnd(I, H)
        sd[p + "mlp.up_proj.weight"] = rnd(I, H)
        sd[p + "mlp.down_proj.weight"] = rnd(H, I)
        sd[p + "input_layernorm.weight"] = near_one(H)
        sd[p + "post_attention_layernorm.weight"] = near_one(H)
    return sd


def write_qwen3_checkpoint(path: str, config: dict, seed: int = 0, shards: int = 1) -> str:
    write_config_only(path, config)
    sd = qwen3_state_dict(config, seed)
    names = sorted(sd)
    for k in range(shards):
        part = {n: sd[n].contiguous() for n in names[k::shards]}
        save_file(part, os.path.join(path, f"model-{k + 1:05d}-of-{shards:05d}.safetensors"))
    return path


def awq_quantize_dense(w_out_in: torch.Tensor, group: int = 128):
    """Round-to-nearest asymmetric int4 per (group of K, output column) -> AutoAWQ tensors."""
    w = w_out_in.float().t().contiguous()
    K, N = w.shape
    wg = w.view(K // group, group, N)
    lo, hi = wg.amin(1), wg.amax(1)
    scale = ((hi - lo) / 15).clamp_min(1e-8)
    zero = (-lo / scale).round().clamp(0, 15)
    q = (wg / scale.unsqueeze(1) + zero.unsqueeze(1)).round().clamp(0, 15).view(K, N).to(torch.int32)
    return pack_awq_int4(q), pack_awq_int4(zero.to(torch.int32)), scale.to(torch.bfloat16)


AWQ_QUANT_CONFIG = dict(quant_method="awq", backend="autoawq", bits=4, group_size=128, version="gemm",
                        zero_point=True)


def write_awq_checkpoint(path: str, config: dict, seed: int = 0, random_codes: bool = False) -> str:
    """AutoAWQ GEMM g128 checkpoint.  ``random_codes`` draws codes/zeros uniform 0..15 and scales
    |N(0,1)|*0.01 (the benchmark spec); otherwise a dense random model is RTN-quantised."""
    cfg = dict(config, torch_dtype="bfloat16", quantization_config=dict(AWQ_QUANT_CONFIG))
    write_config_only(path, cfg)
    sd = qwen3_state_dict(dict(config, torch_dtype="bfloat16"), seed)
    g = torch.Generator().manual_seed(seed + 1)
    out = {}
    for name, t in sd.items():
        if name.startswith("model.layers.") and name.endswith("_proj.weight"):
            base = name[: -len(".weight")]
            if random_codes:
                N, K = t.shape
                q = torch.randint(0, 16, (K, N), generator=g, dtype=torch.int32)
                z = torch.randint(0, 16, (K // 128, N), generator=g, dtype=torch.int32)
                out[base + ".qweight"] = pack_awq_int4(q)
                out[base + ".qzeros"] = pack_awq_int4(z)
                out[base + ".scales"] = (torch.randn(K // 128, N, generator=g).abs() * 0.01).to(torch.bfloat16)
            else:
                out[base + ".qweight"], out[base + ".qzeros"], out[base + ".scales"] = awq_quantize_dense(t)
        else:
            out[name] = t
    save_file(out, os.path.join(path, "model.safetensors"))
    return path


def write_eagle3_checkpoint(path: str, target_config: dict, draft_vocab: int, seed: int = 0,
                            nested: bool = True, include_embedding: bool = False, std: float = 0.02) -> str:
    H = target_config["hidden_size"]
    layer = dict(hidden_size=H, intermediate_size=target_config["intermediate_size"],
                 num_attention_heads=target_config["num_attention_heads"],
                 num_key_value_heads=target_config["num_key_value_heads"], head_dim=target_config["head_dim"],
                 vocab_size=target_config["vocab_size"],
                 max_position_embeddings=target_config["max_position_embeddings"],
                 rope_theta=target_config["rope_theta"], rms_norm_eps=target_config["rms_norm_eps"])
    if nested:
        cfg = dict(draft_vocab_size=draft_vocab, target_hidden_size=H, norm_before_residual=False,
                   transformer_layer_config=layer)
    else:
        cfg = dict(layer, draft_vocab_size=draft_vocab, target_hidden_size=H)
    write_config_only(path, cfg)
    dtype = _DT[target_config["torch_dtype"]]
    g = torch.Generator().manual_seed(seed + 100)
    nh, nkv, hd, I, V = (layer["num_attention_heads"], layer["num_key_value_heads"], layer["head_dim"],
                         layer["intermediate_size"], layer["vocab_size"])

    def rnd(*shape):
        return (torch.randn(*shape, generator=g) * std).to(dtype)

    prefix = "layers.0." if nested else "midlayer."
    sd = {
        "fc.weight": rnd(H, 3 * H), "norm.weight": torch.ones(H, dtype=dtype), "lm_head.weight": rnd(draft_vocab, H),
        prefix + "input_layernorm.weight": torch.ones(H, dtype=dtype),
        prefix + "hidden_norm.weight": torch.ones(H, dtype=dtype),
        prefix + "post_attention_layernorm.weight": torch.ones(H, dtype=dtype),
        prefix + "self_attn.q_proj.weight": rnd(nh * hd, 2 * H),
        prefix + "self_attn.k_proj.weight": rnd(nkv * hd, 2 * H),
        prefix + "self_attn.v_proj.weight": rnd(nkv * hd, 2 * H),
        prefix + "self_attn.o_proj.weight": rnd(H, nh * hd),
        prefix + "mlp.gate_proj.weight": rnd(I, H), prefix + "mlp.up_proj.weight": rnd(I, H),
        prefix + "mlp.down_proj.weight": rnd(H, I),
    }
    ids = torch.randperm(V, generator=g)[:draft_vocab].sort().values
    sd["d2t"] = ids - torch.arange(draft_vocab)
    t2d = torch.zeros(V, dtype=torch.bool)
    t2d[ids] = True
    sd["t2d"] = t2d
    if include_embedding:
        sd["embed_tokens.weight"] = rnd(V, H)
    save_file(sd, os.path.join(path, "model.safetensors"))
    return path


def write_word_tokenizer(path: str, vocab_size: int, eos_token_id: int) -> str:
    """A word-level HF fast tokenizer whose words are ``t0 .. t{vocab-1}`` (``t{i}`` -> id ``i``);
    calibration and evaluation text for synthetic checkpoints is written in those words."""
    from tokenizers import Tokenizer, models, pre_tokenizers
    os.makedirs(path, exist_ok=True)
    tok = Tokenizer(models.WordLevel(vocab={f"t{i}": i for i in range(vocab_size)}, unk_token="t0"))
    tok.pre_tokenizer = pre_tokenizers.Whitespace()
    tok.save(os.path.join(path, "tokenizer.json"))
    with open(os.path.join(path, "tokenizer_config.json"), "w") as f:
        json.dump({"tokenizer_class": "PreTrainedTokenizerFast", "eos_token": f"t{eos_token_id}",
                   "unk_token": "t0", "model_max_length": 1 << 20}, f)
    return path
