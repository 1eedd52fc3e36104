"""CLI: calibrate a BF16 Hugging Face Qwen3 checkpoint with AWQ and export AutoAWQ GEMM W4A16.

``python -m llmserve_b200.quantization.quantize_qwen3 --model BF16_DIR --output AWQ_DIR --calib-file TEXT``

Behaviour parity with ``llmserve/quantization/quantize_qwen3.py`` of the reference (arguments
:37-52, ``run`` :156-296): calibration text one sample per line; the first decoder layer's input
and keyword arguments are recorded by a forward pre-hook that stops the model there; the layers
are then calibrated one at a time on the device (the rest of the model stays on the host); each
layer's result is cached (``layer-NN.safetensors``) and ``calibration_progress.json`` is written
atomically after every layer, so an interrupted run resumes from the cache.  A cache made with
different settings (the signature: source, calibration file hash, sample and token counts, search
sizes, group size, clipping) is refused.

Unlike the reference, ``--device cpu`` is accepted (small models, tests); the default is
``cuda:0``.
"""
import argparse
import hashlib
import itertools
import json
import os
import tempfile
import time
from pathlib import Path

import torch
from torch.utils._pytree import tree_map

from llmserve_b200.quantization.qwen3_awq import (apply_qwen3_layer_cache, calibrate_qwen3_layer,
                                                   export_qwen3_awq_checkpoint, load_qwen3_layer_cache,
                                                   save_qwen3_layer_cache)


class _StopAtFirstLayer(Exception):
    pass


def build_parser() -> argparse.ArgumentParser:
    p = argparse.ArgumentParser(description="Calibrate and export a Qwen3 checkpoint as runtime-native AWQ W4A16.")
    p.add_argument("--model", type=Path, required=True, help="BF16 Qwen3 model")
    p.add_argument("--output", type=Path, required=True, help="AWQ checkpoint directory")
    p.add_argument("--calib-file", type=Path, required=True, help="One sample per line")
    p.add_argument("--device", default="cuda:0")
    p.add_argument("--max-calib-samples", type=int, default=32)
    p.add_argument("--max-seq-len", type=int, default=512)
    p.add_argument("--search-tokens", type=int, default=512)
    p.add_argument("--n-grid", type=int, default=20)
    p.add_argument("--group-size", type=int, default=128)
    p.add_argument("--no-clip", action="store_true")
    p.add_argument("--cache-dir", type=Path)
    p.add_argument("--max-shard-size", default="4GB")
    return p


def load_calibration_texts(path: Path, *, max_samples: int) -> list:
    """The first ``max_samples`` non-blank lines of ``path`` (stripped), one calibration sample
    each."""
    if max_samples < 1:
        raise ValueError(f"max_samples={max_samples}: at least one calibration sample is needed")
    try:
        with open(path, encoding="utf-8") as f:
            samples = list(itertools.islice((ln.strip() for ln in f if ln.strip()), max_samples))
    except (FileNotFoundError, IsADirectoryError) as e:
        raise FileNotFoundError(f"no calibration text file at {path}") from e
    if not samples:
        raise ValueError(f"{path} holds only blank lines; nothing to calibrate on")
    return samples


def _sha256(path: Path) -> str:
    with open(path, "rb") as f:
        return hashlib.file_digest(f, "sha256").hexdigest()


def atomic_write_json(path: Path, payload: dict) -> None:
    """The progress record, sorted and UTF-8, replaced atomically (a resumed run never reads half a file)."""
    text = json.dumps(payload, indent=2, ensure_ascii=False, sort_keys=True) + "\n"
    path.parent.mkdir(parents=True, exist_ok=True)
    fd, tmp = tempfile.mkstemp(dir=path.parent, suffix=".partial")
    with os.fdopen(fd, "w", encoding="utf-8") as f:
        f.write(text)
    os.replace(tmp, path)


def _to(value, device):
    """Every tensor inside a (nested) argument structure moved to ``device``."""
    return tree_map(lambda v: v.to(device) if isinstance(v, torch.Tensor) else v, value)


def validate_args(args) -> None:
    problems = [f"--{n.replace('_', '-')} must be >= 1" for n in ("max_calib_samples", "max_seq_len", "search_tokens",
                                                                  "n_grid") if getattr(args, n) < 1]
    if args.group_size != 128:
        problems.append(f"--group-size {args.group_size}: the W4A16 kernels take groups of 128 only")
    if args.model.resolve() == args.output.resolve():
        problems.append("--output would overwrite the BF16 source checkpoint")
    if problems:
        raise ValueError("; ".join(problems))


@torch.no_grad()
def capture_first_layer_input(model, encoded: dict, device: torch.device):
    """Run embeddings (+ rotary tables) on ``device`` and stop at the first decoder layer."""
    base = model.model
    first = base.layers[0].to(device)
    base.embed_tokens.to(device)
    if hasattr(base, "rotary_emb"):
        base.rotary_emb.to(device)
    seen = {}

    def hook(_module, args, kwargs):
        seen["hidden"], seen["kwargs"] = args[0].detach(), dict(kwargs)
        raise _StopAtFirstLayer

    handle = first.register_forward_pre_hook(hook, with_kwargs=True)
    try:
        mask = encoded.get("attention_mask")
        base(input_ids=encoded["input_ids"].to(device), attention_mask=None if mask is None else mask.to(device),
             use_cache=False)
    except _StopAtFirstLayer:
        pass
    finally:
        handle.remove()
        base.embed_tokens.to("cpu")
        if hasattr(base, "rotary_emb"):
            base.rotary_emb.to("cpu")
    if "hidden" not in seen:
        raise RuntimeError("failed to capture the first Qwen3 decoder layer input")
    kwargs = seen["kwargs"]
    kwargs.pop("past_key_values", None)
    kwargs["use_cache"] = False
    return seen["hidden"], kwargs


def _layer_forward(layer, hidden, kwargs):
    out = layer(hidden, **kwargs)
    return out[0] if isinstance(out, tuple) else out


def run(args) -> dict:
    from transformers import AutoModelForCausalLM, AutoTokenizer

    validate_args(args)
    t_start = time.time()
    device = torch.device(args.device)
    if device.type == "cuda" and not torch.cuda.is_available():
        raise RuntimeError("Qwen3 AWQ calibration on a CUDA device needs CUDA")
    texts = load_calibration_texts(args.calib_file, max_samples=args.max_calib_samples)
    tok = AutoTokenizer.from_pretrained(args.model)
    if tok.pad_token_id is None:
        tok.pad_token = tok.eos_token
    encoded = tok(texts, return_tensors="pt", padding=True, truncation=True, max_length=args.max_seq_len)
    n_tokens = int(encoded["attention_mask"].sum())
    model = AutoModelForCausalLM.from_pretrained(args.model, dtype=torch.bfloat16, low_cpu_mem_usage=True,
                                                 attn_implementation="sdpa").eval()
    if getattr(model.config, "model_type", None) != "qwen3":
        raise ValueError("only Qwen3 checkpoints are supported")

    cache_dir = args.cache_dir or (args.output / ".calibration-cache")
    cache_dir.mkdir(parents=True, exist_ok=True)
    progress_path = cache_dir / "calibration_progress.json"
    signature = {"source_model": str(args.model.resolve()), "calibration_file": str(args.calib_file.resolve()),
                 "calibration_sha256": _sha256(args.calib_file), "samples": len(texts), "tokens": n_tokens,
                 "max_seq_len": args.max_seq_len, "search_tokens": args.search_tokens, "n_grid": args.n_grid,
                 "group_size": args.group_size, "apply_clip": not args.no_clip}
    progress = {"signature": signature, "layers": {}, "status": "calibrating"}
    if progress_path.exists():
        prev = json.loads(progress_path.read_text(encoding="utf-8"))
        if prev.get("signature") != signature:
            raise RuntimeError("calibration settings differ from the existing cache; use a new cache directory")
        progress = dict(prev, status="calibrating")

    if device.type == "cuda":
        torch.cuda.set_device(device)
        torch.cuda.reset_peak_memory_stats()
    hidden, kwargs = capture_first_layer_input(model, encoded, device)
    kwargs = _to(kwargs, device)
    cache_paths = []
    for i, layer in enumerate(model.model.layers):
        t_layer = time.time()
        layer.to(device)
        path = cache_dir / f"layer-{i:02d}.safetensors"
        cache_paths.append(path)
        if path.exists():
            apply_qwen3_layer_cache(layer, load_qwen3_layer_cache(path), group_size=args.group_size)
            hidden = _layer_forward(layer, hidden, kwargs)
            old = progress.get("layers", {}).get(str(i), {})
            status, clipped, evaluated = "resumed", old.get("clipped_groups"), old.get("evaluated_clip_groups")
        else:
            res = calibrate_qwen3_layer(layer, hidden, forward_kwargs=kwargs, group_size=args.group_size,
                                        n_grid=args.n_grid, max_tokens=args.search_tokens, apply_clip=not args.no_clip)
            hidden = res.hidden_states
            save_qwen3_layer_cache(layer, res.packed_weights, path)
            status, clipped, evaluated = "calibrated", res.clipped_group_count, res.evaluated_clip_group_count
        layer.to("cpu")
        if device.type == "cuda":
            torch.cuda.empty_cache()
        record = {"status": status, "cache": str(path), "elapsed_seconds": time.time() - t_layer,
                  "clipped_groups": clipped, "evaluated_clip_groups": evaluated}
        progress.setdefault("layers", {})[str(i)] = record
        progress["completed_layers"] = i + 1
        atomic_write_json(progress_path, progress)
        print(json.dumps({"layer": i, **record}, ensure_ascii=False), flush=True)

    del hidden, kwargs, encoded
    peak = None
    if device.type == "cuda":
        torch.cuda.empty_cache()
        peak = torch.cuda.max_memory_allocated(device)
    meta = {**signature, "layers": progress["layers"], "elapsed_seconds": time.time() - t_start,
            "peak_cuda_memory_bytes": peak}
    export_qwen3_awq_checkpoint(model, cache_paths, args.model, args.output, calibration_metadata=meta,
                                group_size=args.group_size, max_shard_size=args.max_shard_size)
    progress.update(status="complete", output=str(args.output.resolve()), elapsed_seconds=time.time() - t_start)
    atomic_write_json(progress_path, progress)
    return progress


def main() -> None:
    print(json.dumps(run(build_parser().parse_args()), indent=2, ensure_ascii=False), flush=True)


if __name__ == "__main__":
    main()
