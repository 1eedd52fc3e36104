"""CLI: quality of a BF16 or AWQ Qwen3 checkpoint on local text (perplexity + greedy samples).

``python -m llmserve_b200.quantization.awq_quality --model DIR --eval-file TEXT --output result.json``

Behaviour parity with ``llmserve/quantization/awq_quality.py`` of the reference (arguments
:82-96, ``ReferenceAWQLinear`` :15-60, ``_evaluate_perplexity`` :190-241, result schema in ``run``
:267-330): the text is tokenized sample by sample (EOS between samples) up to
``max_eval_tokens + 1`` ids, scored in non-overlapping blocks of ``sequence_length`` with the
summed token cross-entropy, and reported as mean NLL and perplexity with the first block's last
top-5; a few prompts are also decoded greedily.  ``--mode awq-reference`` runs the HF Qwen3
module tree with its seven projections per layer replaced by a dequantise-then-matmul W4A16
linear (the oracle of the serving kernel).

The reference builds the AWQ model through ``accelerate``'s empty-weight context; here it is built
on the meta device, materialised with ``to_empty`` on the target device and filled from the
safetensors shards directly (``accelerate`` is not needed).
"""
import argparse
import glob
import json
import math
import os
import time
from pathlib import Path

import torch
import torch.nn.functional as F
from torch import nn

from llmserve_b200.quantization.awq import awq_reference_linear
from llmserve_b200.quantization.qwen3_awq import QWEN3_QUANTIZED_LINEAR_NAMES


class ReferenceAWQLinear(nn.Module):
    """W4A16 linear over AutoAWQ GEMM buffers: dequantise, then matmul in fp32."""

    def __init__(self, input_size: int, output_size: int, *, group_size: int = 128, dtype=torch.bfloat16,
                 device=None):
        super().__init__()
        if input_size % group_size or output_size % 8:
            raise ValueError("AWQ linear shape is incompatible with packing")
        self.group_size, self.in_features, self.out_features = group_size, input_size, output_size
        self.register_buffer("qweight", torch.empty(input_size, output_size // 8, dtype=torch.int32, device=device))
        self.register_buffer("qzeros", torch.empty(input_size // group_size, output_size // 8, dtype=torch.int32,
                                                   device=device))
        self.register_buffer("scales", torch.empty(input_size // group_size, output_size, dtype=dtype,
                                                   device=device))

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return awq_reference_linear(x, self.qweight, self.qzeros, self.scales, group_size=self.group_size)


def build_parser() -> argparse.ArgumentParser:
    p = argparse.ArgumentParser(description="Evaluate BF16 or packed AWQ Qwen3 quality on fixed local text.")
    p.add_argument("--model", type=Path, required=True)
    p.add_argument("--eval-file", type=Path, required=True)
    p.add_argument("--output", type=Path, required=True)
    p.add_argument("--mode", choices=("auto", "bf16", "awq-reference"), default="auto")
    p.add_argument("--device", default="cuda:0")
    p.add_argument("--max-samples", type=int, default=32)
    p.add_argument("--sequence-length", type=int, default=128)
    p.add_argument("--max-eval-tokens", type=int, default=2048)
    p.add_argument("--generation-prompts", type=int, default=2)
    p.add_argument("--max-new-tokens", type=int, default=16)
    return p


def replace_qwen3_linears(model: nn.Module, group_size: int, dtype, device=None) -> None:
    suffixes = tuple("." + n for n in QWEN3_QUANTIZED_LINEAR_NAMES)
    for name, module in list(model.named_modules()):
        if not isinstance(module, nn.Linear) or not name.endswith(suffixes):
            continue
        if module.bias is not None:
            raise ValueError(f"AWQ reference loader does not support bias: {name}")
        parent, child = name.rsplit(".", 1)
        setattr(model.get_submodule(parent), child,
                ReferenceAWQLinear(module.in_features, module.out_features, group_size=group_size, dtype=dtype,
                                   device=device))


def _read_safetensors(path: Path, device) -> dict:
    from safetensors.torch import load_file
    files = sorted(glob.glob(os.path.join(str(path), "*.safetensors")))
    if not files:
        raise FileNotFoundError(f"no safetensors files under {path}")
    out = {}
    for f in files:
        out.update(load_file(f, device=str(device)))
    return out


def load_awq_reference_model(model_path: Path, device: torch.device):
    from transformers import AutoConfig
    from transformers.models.qwen3.modeling_qwen3 import Qwen3ForCausalLM, Qwen3RotaryEmbedding

    config = AutoConfig.from_pretrained(model_path)
    qc = getattr(config, "quantization_config", None)
    if not isinstance(qc, dict):
        raise ValueError("AWQ reference mode requires quantization_config")
    group_size = int(qc.get("group_size", 0))
    if qc.get("quant_method") != "awq" or group_size <= 0:
        raise ValueError("unsupported quantization_config")
    dtype = getattr(config, "dtype", None) or torch.bfloat16
    if isinstance(dtype, str):
        dtype = getattr(torch, dtype)
    with torch.device("meta"):
        model = Qwen3ForCausalLM(config)
        replace_qwen3_linears(model, group_size, dtype)
    model = model.to(dtype)               # norms, embeddings and head in the checkpoint's dtype
    model.to_empty(device=device)
    state = _read_safetensors(model_path, device)
    state = {k: (v.to(dtype) if v.is_floating_point() else v) for k, v in state.items()}
    if getattr(config, "tie_word_embeddings", False) and "lm_head.weight" not in state:
        state["lm_head.weight"] = state["model.embed_tokens.weight"]
    missing, _ = model.load_state_dict(state, strict=False)
    missing = [m for m in missing if not m.endswith("rotary_emb.inv_freq") and not m.endswith("original_inv_freq")]
    if missing:
        raise RuntimeError(f"checkpoint left uninitialized tensors: {missing[:8]}")
    model.model.rotary_emb = Qwen3RotaryEmbedding(config, device=device)
    return model.eval()


def load_model(model_path: Path, mode: str, device: torch.device):
    from transformers import AutoConfig, AutoModelForCausalLM
    config = AutoConfig.from_pretrained(model_path)
    is_awq = isinstance(getattr(config, "quantization_config", None), dict)
    if mode == "auto":
        mode = "awq-reference" if is_awq else "bf16"
    if mode == "awq-reference":
        return load_awq_reference_model(model_path, device), mode
    if is_awq:
        raise ValueError("BF16 mode cannot load a packed AWQ checkpoint")
    model = AutoModelForCausalLM.from_pretrained(model_path, dtype=torch.bfloat16, low_cpu_mem_usage=True)
    return model.to(device).eval(), mode


def read_texts(path: Path, max_samples: int) -> list:
    if max_samples <= 0:
        raise ValueError("max_samples must be positive")
    texts = []
    with path.open("r", encoding="utf-8") as f:
        for line in f:
            if line.strip():
                texts.append(line.strip())
                if len(texts) == max_samples:
                    break
    if not texts:
        raise ValueError("evaluation file contains no nonempty samples")
    return texts


@torch.inference_mode()
def evaluate_perplexity(model, tokenizer, texts, *, device, sequence_length: int, max_eval_tokens: int) -> dict:
    ids = []
    for text in texts:
        ids += tokenizer.encode(text, add_special_tokens=False)
        if tokenizer.eos_token_id is not None:
            ids.append(tokenizer.eos_token_id)
        if len(ids) > max_eval_tokens:
            break
    ids = ids[: max_eval_tokens + 1]
    if len(ids) < 2:
        raise ValueError("evaluation text produced fewer than two tokens")
    nll, count, top5 = 0.0, 0, None
    for start in range(0, len(ids) - 1, sequence_length):
        block = ids[start: start + sequence_length + 1]
        if len(block) < 2:
            continue
        logits = model(input_ids=torch.tensor([block[:-1]], device=device), use_cache=False).logits[0].float()
        target = torch.tensor(block[1:], device=device)
        nll += float(F.cross_entropy(logits, target, reduction="sum"))
        count += target.numel()
        if top5 is None:
            v, i = logits[-1].topk(5)
            top5 = {"token_ids": i.cpu().tolist(), "logits": v.cpu().tolist()}
    mean = nll / count
    return {"definition": "non-overlapping fixed-block causal perplexity", "tokens": count, "mean_nll": mean,
            "perplexity": math.exp(mean), "first_block_last_token_top5": top5}


@torch.inference_mode()
def generate_greedy(model, tokenizer, texts, device, max_new_tokens: int) -> list:
    if not texts:
        return []
    tokenizer.padding_side = "left"
    enc = {k: v.to(device) for k, v in tokenizer(texts, return_tensors="pt", padding=True).items()}
    out = model.generate(**enc, do_sample=False, max_new_tokens=max_new_tokens, pad_token_id=tokenizer.pad_token_id,
                         eos_token_id=tokenizer.eos_token_id)
    return [{"prompt": p, "output": tokenizer.decode(o, skip_special_tokens=True)} for p, o in zip(texts, out)]


def run(args) -> dict:
    from transformers import AutoTokenizer
    for name in ("max_samples", "sequence_length", "max_eval_tokens", "max_new_tokens"):
        if getattr(args, name) <= 0:
            raise ValueError(f"{name} must be positive")
    if args.generation_prompts < 0:
        raise ValueError("generation_prompts cannot be negative")
    device = torch.device(args.device)
    texts = read_texts(args.eval_file, args.max_samples)
    tok = AutoTokenizer.from_pretrained(args.model)
    if tok.pad_token_id is None:
        tok.pad_token = tok.eos_token
    t0 = time.time()
    if device.type == "cuda":
        torch.cuda.set_device(device)
        torch.cuda.reset_peak_memory_stats()
    model, mode = load_model(args.model, args.mode, device)
    ppl = evaluate_perplexity(model, tok, texts, device=device, sequence_length=args.sequence_length,
                              max_eval_tokens=args.max_eval_tokens)
    gens = generate_greedy(model, tok, texts[: args.generation_prompts], device, args.max_new_tokens)
    result = {"schema_version": 1, "model": args.model.name, "mode": mode, "evaluation_file": args.eval_file.name,
              "samples": len(texts), "sequence_length": args.sequence_length, "perplexity": ppl,
              "generations": gens, "elapsed_seconds": time.time() - t0,
              "peak_cuda_memory_bytes": torch.cuda.max_memory_allocated(device) if device.type == "cuda" else None}
    args.output.parent.mkdir(parents=True, exist_ok=True)
    tmp = args.output.with_suffix(args.output.suffix + ".tmp")
    tmp.write_text(json.dumps(result, indent=2, ensure_ascii=False, sort_keys=True) + "\n", encoding="utf-8")
    tmp.replace(args.output)
    return result


def main() -> None:
    print(json.dumps(run(build_parser().parse_args()), indent=2, ensure_ascii=False), flush=True)


if __name__ == "__main__":
    main()
