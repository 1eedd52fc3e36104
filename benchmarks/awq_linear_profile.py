"""One Qwen3 AWQ (W4A16, AutoAWQ GEMM g128) decoder layer's projections, timed with CUDA events.

``python -m benchmarks.awq_linear_profile --model AWQ_DIR [--layer-id 0] [--num-tokens 1,4,8,16]``
(``--model qwen3-8b-random`` draws the BASELINE's random codes / zeros / scales instead).

Behaviour parity with ``benchmarks/awq_linear_profile.py`` of the reference
(``merge_projection_tensors`` :67-90, ``load_layer_projections`` :93-147, stage summary :150-186,
``measure_projection_cuda`` :188-290): the q/k/v and gate/up checkpoint modules are merged into the
four projections and each is timed as its stages -- ``dequantize`` (AutoAWQ tensors -> dense bf16),
``matmul`` (dense bf16 GEMM), ``reference`` (the two together, the oracle) and ``cuda`` (the
serving kernel: here the sm_100a tcgen05 W4A16 kernel with in-shared-memory dequantisation and its
split-K reduction).  The reference's Triton stage has no counterpart (this project has no Triton
path).  As in ``benchmarks.linear_profile``, the packed weights rotate among enough copies to
exceed twice the L2, and each ``cuda`` measurement reports its payload bandwidth.
"""
import argparse
import json
from dataclasses import dataclass
from pathlib import Path

from benchmarks.environment import atomic_write_json, build_environment_metadata, discover_model_revision
from benchmarks.linear_profile import L2_BYTES, PROJECTION_NAMES, measured_hbm_gbs, parse_num_tokens

PROJECTION_COMPONENTS = {"qkv": ("q_proj", "k_proj", "v_proj"), "o": ("o_proj",), "gate_up": ("gate_proj", "up_proj"),
                         "down": ("down_proj",)}
AWQ_TENSOR_NAMES = ("qweight", "qzeros", "scales")
STAGES = ("dequantize", "matmul", "reference", "cuda")
RANDOM_MODEL = "qwen3-8b-random"


@dataclass(frozen=True)
class AWQProjectionTensors:
    name: str
    qweight: object
    qzeros: object
    scales: object

    @property
    def input_size(self) -> int:
        return self.qweight.shape[0]

    @property
    def output_size(self) -> int:
        return self.scales.shape[1]

    @property
    def payload_bytes(self) -> int:
        return sum(t.numel() * t.element_size() for t in (self.qweight, self.qzeros, self.scales))

    def to(self, device) -> "AWQProjectionTensors":
        return AWQProjectionTensors(self.name, self.qweight.to(device), self.qzeros.to(device), self.scales.to(device))


def merge_projection_tensors(name: str, parts: list) -> AWQProjectionTensors:
    import torch
    if not parts:
        raise ValueError("projection must contain at least one checkpoint module")
    if len({(q.shape[0], z.shape[0], s.shape[0]) for q, z, s in parts}) != 1:
        raise ValueError("projection parts must share input/group dimensions")
    p = AWQProjectionTensors(name, torch.cat([x[0] for x in parts], 1), torch.cat([x[1] for x in parts], 1),
                             torch.cat([x[2] for x in parts], 1))
    if p.qweight.shape[1] * 8 != p.output_size:
        raise ValueError("qweight packed output does not match scales")
    if p.qzeros.shape[1] * 8 != p.output_size:
        raise ValueError("qzeros packed output does not match scales")
    return p


def _module_prefix(layer_id: int, component: str) -> str:
    block = "self_attn" if component in ("q_proj", "k_proj", "v_proj", "o_proj") else "mlp"
    return f"model.layers.{layer_id}.{block}.{component}"


def load_layer_projections(model_path, *, layer_id: int) -> tuple:
    """The four merged projections of one layer from an AutoAWQ checkpoint (sharded with an HF
    index, or a single ``model.safetensors``)."""
    from safetensors import safe_open
    model_path = Path(model_path)
    index = model_path / "model.safetensors.index.json"
    keys = [f"{_module_prefix(layer_id, c)}.{t}" for comps in PROJECTION_COMPONENTS.values() for c in comps
            for t in AWQ_TENSOR_NAMES]
    if index.is_file():
        weight_map = json.loads(index.read_text(encoding="utf-8")).get("weight_map", {})
    elif (model_path / "model.safetensors").is_file():
        with safe_open(model_path / "model.safetensors", framework="pt", device="cpu") as f:
            weight_map = {k: "model.safetensors" for k in f.keys()}
    else:
        raise ValueError("AWQ profiler needs model.safetensors or model.safetensors.index.json")
    missing = [k for k in keys if k not in weight_map]
    if missing:
        raise ValueError(f"checkpoint index is missing AWQ tensors: {missing}")
    tensors, by_file = {}, {}
    for k in keys:
        by_file.setdefault(weight_map[k], []).append(k)
    for fname, ks in by_file.items():
        with safe_open(model_path / fname, framework="pt", device="cpu") as f:
            for k in ks:
                tensors[k] = f.get_tensor(k)
    return tuple(merge_projection_tensors(
        name, [tuple(tensors[f"{_module_prefix(layer_id, c)}.{t}"] for t in AWQ_TENSOR_NAMES)
               for c in PROJECTION_COMPONENTS[name]]) for name in PROJECTION_NAMES)


def random_layer_projections(config: dict, seed: int = 0) -> tuple:
    """Codes and zeros uniform 0..15, scales |N(0,1)| * 0.01 (the benchmark's AWQ spec)."""
    import torch

    from llmserve_b200.quantization.awq import pack_awq_int4
    g = torch.Generator().manual_seed(seed)
    H, I = config["hidden_size"], config["intermediate_size"]
    q, kv = config["num_attention_heads"] * config["head_dim"], config["num_key_value_heads"] * config["head_dim"]
    out = []
    for name, (k, n) in zip(PROJECTION_NAMES, ((H, q + 2 * kv), (q, H), (H, 2 * I), (I, H))):
        out.append(AWQProjectionTensors(
            name, pack_awq_int4(torch.randint(0, 16, (k, n), generator=g, dtype=torch.int32)),
            pack_awq_int4(torch.randint(0, 16, (k // 128, n), generator=g, dtype=torch.int32)),
            (torch.randn(k // 128, n, generator=g).abs() * 0.01).to(torch.bfloat16)))
    return tuple(out)


def summarize_stage_latencies(measurements: dict, *, num_hidden_layers: int) -> dict:
    missing = [n for n in PROJECTION_NAMES if n not in measurements]
    if missing:
        raise ValueError(f"missing projection latency: {', '.join(missing)}")
    per_layer = {s: sum(float(measurements[n][s]) for n in PROJECTION_NAMES) for s in STAGES}
    if any(v <= 0 for v in per_layer.values()):
        raise ValueError("AWQ stage latency totals must be positive")
    if num_hidden_layers <= 0:
        raise ValueError("num_hidden_layers must be positive")
    return {"per_layer_ms": per_layer,
            "dequantize_component_share_pct": per_layer["dequantize"] / (per_layer["dequantize"] + per_layer["matmul"])
            * 100.0,
            "model_reference_total_ms": per_layer["reference"] * num_hidden_layers,
            "model_cuda_total_ms": per_layer["cuda"] * num_hidden_layers,
            "cuda_speedup_vs_reference": per_layer["reference"] / per_layer["cuda"]}


def measure_cuda_operation(operation, *, warmup: int, repeats: int, rotate: int = 1) -> float:
    """Mean ms of ``operation(i)`` over ``repeats`` calls, ``i`` cycling through ``rotate`` copies."""
    import torch
    if warmup < 0 or repeats <= 0:
        raise ValueError("warmup must be non-negative and repeats must be positive")
    out = None
    for i in range(warmup):
        out = operation(i % rotate)
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for i in range(repeats):
        out = operation(i % rotate)
    end.record()
    end.synchronize()
    if out is None:
        raise RuntimeError("CUDA operation did not produce an output")
    return start.elapsed_time(end) / repeats


def measure_projection_cuda(projection: AWQProjectionTensors, *, num_tokens: int, group_size: int, device,
                            warmup: int, repeats: int, hbm_gbs=None) -> dict:
    import torch

    from llmserve_b200.ops import awq as awq_ops
    from llmserve_b200.ops._ext import check_status
    from llmserve_b200.quantization.awq import awq_reference_linear, dequantize_awq_gemm
    if device.type != "cuda":
        raise ValueError("AWQ latency profiling requires a CUDA device")
    with torch.cuda.device(device), torch.inference_mode():
        p = projection.to(device)
        x = torch.randn(num_tokens, p.input_size, device=device).to(p.scales.dtype)
        weight = dequantize_awq_gemm(p.qweight, p.qzeros, p.scales, group_size=group_size)
        copies = max(1, -(-2 * L2_BYTES // p.payload_bytes))
        packed = [awq_ops.prepare_awq_weights(p.qweight, p.qzeros, p.scales, group_size) for _ in range(copies)]
        m = {
            "dequantize": measure_cuda_operation(
                lambda i: dequantize_awq_gemm(p.qweight, p.qzeros, p.scales, group_size=group_size),
                warmup=warmup, repeats=repeats),
            "matmul": measure_cuda_operation(lambda i: torch.matmul(x, weight), warmup=warmup, repeats=repeats),
            "reference": measure_cuda_operation(
                lambda i: awq_reference_linear(x, p.qweight, p.qzeros, p.scales, group_size=group_size),
                warmup=warmup, repeats=repeats),
            "cuda": measure_cuda_operation(lambda i: awq_ops.awq_linear(x, packed[i]), warmup=warmup,
                                           repeats=repeats, rotate=copies),
        }
        check_status(device)
        m["payload_bytes"] = p.payload_bytes
        m["cuda_payload_gbps"] = p.payload_bytes / (m["cuda"] * 1e-3) / 1e9
        if hbm_gbs:
            m["cuda_fraction_of_measured_hbm"] = m["cuda_payload_gbps"] / hbm_gbs
    torch.cuda.empty_cache()
    return m


def build_parser() -> argparse.ArgumentParser:
    p = argparse.ArgumentParser(description="Profile Qwen3 AWQ reference dequantize and matmul stages.")
    p.add_argument("--model", required=True, help=f"AutoAWQ Qwen3 directory, or '{RANDOM_MODEL}'")
    p.add_argument("--layer-id", type=int, default=0)
    p.add_argument("--num-tokens", type=parse_num_tokens, default=parse_num_tokens("1,4,8,16"))
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--repeats", type=int, default=20)
    p.add_argument("--device", default="cuda")
    p.add_argument("--output", type=Path)
    return p


def main(argv=None):
    import torch
    args = build_parser().parse_args(argv)
    if not torch.cuda.is_available():
        raise RuntimeError("CUDA is required for AWQ profiling")
    if args.model == RANDOM_MODEL:
        from llmserve_b200.models.synthetic import QWEN3_8B
        cfg, projections, group = dict(QWEN3_8B), random_layer_projections(QWEN3_8B, args.layer_id), 128
    else:
        cfg = json.loads((Path(args.model) / "config.json").read_text(encoding="utf-8"))
        group = int(cfg.get("quantization_config", {}).get("group_size", 0))
        if group != 128:
            raise ValueError("the W4A16 kernel supports AutoAWQ group_size 128")
        projections = load_layer_projections(args.model, layer_id=args.layer_id)
    device = torch.device(args.device)
    hbm = measured_hbm_gbs()
    rows = []
    for t in args.num_tokens:
        meas = {p.name: measure_projection_cuda(p, num_tokens=t, group_size=group, device=device, warmup=args.warmup,
                                                repeats=args.repeats, hbm_gbs=hbm) for p in projections}
        rows.append({"num_tokens": t, "latency_ms": meas,
                     "summary": summarize_stage_latencies(meas, num_hidden_layers=int(cfg["num_hidden_layers"]))})
    document = {
        "schema_version": 1, "benchmark": "qwen3-awq-linear", "metadata": build_environment_metadata(),
        "model": Path(args.model).name, "model_revision": discover_model_revision(args.model),
        "config": {"layer_id": args.layer_id, "group_size": group, "device": str(device),
                   "num_tokens": list(args.num_tokens), "warmup": args.warmup, "repeats": args.repeats,
                   "num_hidden_layers": int(cfg["num_hidden_layers"]), "measured_hbm_gbs": hbm,
                   "cuda_kernel": "llmserve_b200 sm_100a tcgen05 W4A16"},
        "projections": [{"name": p.name, "input_size": p.input_size, "output_size": p.output_size,
                         "payload_bytes": p.payload_bytes} for p in projections],
        "measurements": rows,
    }
    if args.output is not None:
        atomic_write_json(args.output, document)
    print(json.dumps(document, indent=2))


if __name__ == "__main__":
    main()
