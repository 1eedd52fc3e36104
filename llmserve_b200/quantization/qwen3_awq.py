"""Per-layer AWQ calibration of Hugging Face Qwen3 decoder layers and AutoAWQ GEMM export.

Behaviour parity with ``llmserve/quantization/qwen3_awq.py`` of the reference
(``calibrate_qwen3_layer`` :83-186, layer cache save/load/apply :204-254,
``export_qwen3_awq_checkpoint`` :297-370).  One decoder layer at a time:

1. run the layer once with forward pre-hooks on q_proj, o_proj, gate_proj and down_proj to record
   the inputs of its four linear groups;
2. search scales for {q, k, v} (folded into ``input_layernorm``), {gate, up} (folded into
   ``post_attention_layernorm``) and {down} (folded into ``up_proj``'s output rows);
3. optionally search clipping thresholds for v, o, gate, up and down on the scaled inputs;
4. quantise all seven projections, write the dequantised weights back into the layer, and run
   the layer again so the next layer calibrates on the quantised network's activations.

The layer cache (one safetensors file per layer: packed tensors plus the two folded norm weights)
makes the CLI resumable; the export writes AutoAWQ GEMM tensors (``qweight``/``qzeros``/
``scales``) under the HF names, the AutoAWQ ``quantization_config``, sharded safetensors with an
HF index, and a ``quantization_manifest.json``.
"""
import json
import shutil
from dataclasses import dataclass
from pathlib import Path

import torch
from safetensors.torch import load_file, save_file
from torch import nn

from llmserve_b200.quantization.awq import dequantize_awq_gemm
from llmserve_b200.quantization.awq_calibration import (PackedAWQWeight, apply_awq_clip, fold_linear_scale,
                                                         fold_rmsnorm_scale, quantize_awq_weight, search_awq_clip,
                                                         search_awq_scale)

QWEN3_QUANTIZED_LINEAR_NAMES = ("self_attn.q_proj", "self_attn.k_proj", "self_attn.v_proj", "self_attn.o_proj",
                                "mlp.gate_proj", "mlp.up_proj", "mlp.down_proj")
_PROBED = ("self_attn.q_proj", "self_attn.o_proj", "mlp.gate_proj", "mlp.down_proj")
CACHE_FORMAT = "llmserve-qwen3-awq-layer-v1"
AUTOAWQ_GEMM_CONFIG = {"backend": "autoawq", "bits": 4, "do_fuse": False, "quant_method": "awq", "version": "gemm",
                       "zero_point": True}


@dataclass(frozen=True)
class Qwen3LayerCalibrationResult:
    hidden_states: torch.Tensor
    packed_weights: dict
    clipped_group_count: int
    evaluated_clip_group_count: int


def _forward(layer: nn.Module, hidden_states: torch.Tensor, kwargs: dict) -> torch.Tensor:
    out = layer(hidden_states, **kwargs)
    return out[0] if isinstance(out, tuple) else out


@torch.no_grad()
def _record_linear_inputs(layer: nn.Module, hidden_states: torch.Tensor, kwargs: dict) -> dict:
    seen = {}
    hooks = [layer.get_submodule(name).register_forward_pre_hook(
        lambda _m, args, _n=name: seen.__setitem__(_n, args[0].detach())) for name in _PROBED]
    try:
        _forward(layer, hidden_states, kwargs)
    finally:
        for h in hooks:
            h.remove()
    missing = [n for n in _PROBED if n not in seen]
    if missing:
        raise RuntimeError(f"Qwen3 calibration did not observe inputs for: {missing}")
    return seen


@torch.no_grad()
def _write_dequantized(module: nn.Module, packed: PackedAWQWeight, group_size: int):
    w = dequantize_awq_gemm(packed.qweight, packed.qzeros, packed.scales, group_size=group_size)
    module.weight.copy_(w.t())


@torch.no_grad()
def calibrate_qwen3_layer(layer: nn.Module, hidden_states: torch.Tensor, *, forward_kwargs: dict | None = None,
                          group_size: int = 128, n_grid: int = 20, max_tokens: int = 512,
                          apply_clip: bool = True) -> Qwen3LayerCalibrationResult:
    kwargs = forward_kwargs or {}
    x = _record_linear_inputs(layer, hidden_states, kwargs)
    attn, mlp = layer.self_attn, layer.mlp
    search = dict(group_size=group_size, n_grid=n_grid, max_tokens=max_tokens)

    s_qkv = search_awq_scale(x["self_attn.q_proj"], [attn.q_proj.weight, attn.k_proj.weight, attn.v_proj.weight],
                             **search)
    fold_rmsnorm_scale(layer.input_layernorm, [attn.q_proj, attn.k_proj, attn.v_proj], s_qkv)
    s_gu = search_awq_scale(x["mlp.gate_proj"], [mlp.gate_proj.weight, mlp.up_proj.weight], **search)
    fold_rmsnorm_scale(layer.post_attention_layernorm, [mlp.gate_proj, mlp.up_proj], s_gu)
    s_down = search_awq_scale(x["mlp.down_proj"], [mlp.down_proj.weight], **search)
    fold_linear_scale(mlp.up_proj, [mlp.down_proj], s_down)

    clipped = evaluated = 0
    if apply_clip:
        # inputs as the scaled layer sees them: x / s where the scale was folded in front
        clip_inputs = {"self_attn.v_proj": x["self_attn.q_proj"] / s_qkv,
                       "self_attn.o_proj": x["self_attn.o_proj"],
                       "mlp.gate_proj": x["mlp.gate_proj"] / s_gu,
                       "mlp.up_proj": x["mlp.gate_proj"] / s_gu,
                       "mlp.down_proj": x["mlp.down_proj"] / s_down}
        for name, inp in clip_inputs.items():
            w = layer.get_submodule(name).weight
            before = w.reshape(w.shape[0], -1, group_size).abs().amax(dim=-1, keepdim=True)
            limits = search_awq_clip(w, inp, **search)
            evaluated += limits.numel()
            clipped += int((limits < before).sum())
            apply_awq_clip(w, limits, group_size=group_size)

    packed = {}
    for name in QWEN3_QUANTIZED_LINEAR_NAMES:
        module = layer.get_submodule(name)
        packed[name] = quantize_awq_weight(module.weight, group_size=group_size)
        _write_dequantized(module, packed[name], group_size)
    return Qwen3LayerCalibrationResult(hidden_states=_forward(layer, hidden_states, kwargs), packed_weights=packed,
                                       clipped_group_count=clipped, evaluated_clip_group_count=evaluated)


def _layer_cache_tensors(layer: nn.Module, packed: dict) -> dict:
    t = {"input_layernorm.weight": layer.input_layernorm.weight.detach(),
         "post_attention_layernorm.weight": layer.post_attention_layernorm.weight.detach()}
    for name, p in packed.items():
        t[f"{name}.qweight"], t[f"{name}.qzeros"], t[f"{name}.scales"] = p.qweight, p.qzeros, p.scales
    return {k: v.detach().cpu().contiguous() for k, v in t.items()}


def save_qwen3_layer_cache(layer: nn.Module, packed_weights: dict, path) -> None:
    path = Path(path)
    path.parent.mkdir(parents=True, exist_ok=True)
    tmp = path.with_suffix(path.suffix + ".tmp")
    save_file(_layer_cache_tensors(layer, packed_weights), str(tmp), metadata={"format": CACHE_FORMAT})
    tmp.replace(path)    # a killed run never leaves a half-written cache that a resume would trust


def load_qwen3_layer_cache(path) -> dict:
    return load_file(str(path), device="cpu")


@torch.no_grad()
def apply_qwen3_layer_cache(layer: nn.Module, tensors: dict, *, group_size: int = 128) -> dict:
    """Put a cached layer's folded norms and dequantised projections into ``layer``."""
    for norm in ("input_layernorm", "post_attention_layernorm"):
        w = layer.get_submodule(norm).weight
        w.copy_(tensors[f"{norm}.weight"].to(device=w.device, dtype=w.dtype))
    packed = {}
    for name in QWEN3_QUANTIZED_LINEAR_NAMES:
        module = layer.get_submodule(name)
        dev = module.weight.device
        packed[name] = PackedAWQWeight(qweight=tensors[f"{name}.qweight"].to(dev),
                                       qzeros=tensors[f"{name}.qzeros"].to(dev),
                                       scales=tensors[f"{name}.scales"].to(device=dev, dtype=module.weight.dtype))
        _write_dequantized(module, packed[name], group_size)
    return packed


def _parse_size(size) -> int:
    if isinstance(size, int):
        return size
    s = str(size).strip().upper()
    for unit, mult in (("GIB", 1 << 30), ("MIB", 1 << 20), ("KIB", 1 << 10), ("GB", 10**9), ("MB", 10**6),
                       ("KB", 10**3), ("B", 1)):
        if s.endswith(unit):
            return int(float(s[: -len(unit)]) * mult)
    return int(s)


def _shard(state_dict: dict, max_bytes: int) -> list:
    """Greedy shards in name order, each at most ``max_bytes`` unless one tensor is larger."""
    shards, cur, cur_bytes = [], [], 0
    for name in sorted(state_dict):
        n = state_dict[name].numel() * state_dict[name].element_size()
        if cur and cur_bytes + n > max_bytes:
            shards.append(cur)
            cur, cur_bytes = [], 0
        cur.append(name)
        cur_bytes += n
    if cur:
        shards.append(cur)
    return shards


def _awq_state_dict(model: nn.Module, layer_cache_paths: list) -> dict:
    replaced = {f"model.layers.{i}.{n}.weight" for i in range(len(layer_cache_paths))
                for n in QWEN3_QUANTIZED_LINEAR_NAMES}
    sd = {k: v.detach().cpu().contiguous() for k, v in model.state_dict().items() if k not in replaced}
    for i, path in enumerate(layer_cache_paths):
        cached = load_qwen3_layer_cache(path)
        for n in QWEN3_QUANTIZED_LINEAR_NAMES:
            for part in ("qweight", "qzeros", "scales"):
                sd[f"model.layers.{i}.{n}.{part}"] = cached[f"{n}.{part}"].contiguous()
    return sd


def export_qwen3_awq_checkpoint(model: nn.Module, layer_cache_paths: list, source_model_dir, output_dir, *,
                                calibration_metadata: dict, group_size: int = 128,
                                max_shard_size="4GB") -> None:
    src, out = Path(source_model_dir), Path(output_dir)
    if not (src / "config.json").is_file():
        raise FileNotFoundError(f"missing source config: {src / 'config.json'}")
    if len(layer_cache_paths) != len(model.model.layers):
        raise ValueError("one AWQ cache is required for every Qwen3 decoder layer")
    out.mkdir(parents=True, exist_ok=True)
    for f in src.iterdir():      # tokenizer, generation config, ... (not the weights or the config)
        weights = f.name.startswith("model") and (f.suffix == ".safetensors" or f.name.endswith(".index.json"))
        if f.is_file() and f.name != "config.json" and not weights:
            shutil.copy2(f, out / f.name)
    config = json.loads((src / "config.json").read_text(encoding="utf-8"))
    config["quantization_config"] = dict(AUTOAWQ_GEMM_CONFIG, group_size=group_size)
    (out / "config.json").write_text(json.dumps(config, indent=2, ensure_ascii=False) + "\n", encoding="utf-8")

    sd = _awq_state_dict(model, layer_cache_paths)
    for old in out.glob("model*.safetensors"):
        old.unlink()
    index = out / "model.safetensors.index.json"
    if index.exists():
        index.unlink()
    shards = _shard(sd, _parse_size(max_shard_size))
    total = sum(t.numel() * t.element_size() for t in sd.values())
    names = (["model.safetensors"] if len(shards) == 1 else
             [f"model-{i + 1:05d}-of-{len(shards):05d}.safetensors" for i in range(len(shards))])
    weight_map = {}
    for fname, keys in zip(names, shards):
        save_file({k: sd[k] for k in keys}, str(out / fname), metadata={"format": "pt"})
        weight_map.update({k: fname for k in keys})
    if len(shards) > 1:
        index.write_text(json.dumps({"metadata": {"total_size": total}, "weight_map": weight_map}, indent=2,
                                    sort_keys=True) + "\n", encoding="utf-8")
    manifest = {"format": "autoawq-gemm", "quant_method": "activation-aware-w4a16", "bits": 4,
                "group_size": group_size, "zero_point": True, "source_model": str(src.resolve()),
                "num_layers": len(layer_cache_paths), "calibration": calibration_metadata, "checkpoint_bytes": total}
    (out / "quantization_manifest.json").write_text(
        json.dumps(manifest, indent=2, ensure_ascii=False, sort_keys=True) + "\n", encoding="utf-8")
