"""Qwen3 projection GEMMs on the sm_100a kernels, timed with CUDA events.

``python -m benchmarks.linear_profile --model DIR_OR_qwen3-8b [--num-tokens 1,4,8,16,64] [--tp 1]``

Behaviour parity with ``benchmarks/linear_profile.py`` of the reference (``qwen3_projection_shapes``
:26-45, ``summarize_latencies`` :48-71, ``parse_num_tokens`` :74-83, document schema in ``main``
:183-233): the four projections of one decoder layer (qkv, o, gate_up, down) are timed for each
token count and summarised per layer and per model.  The reference times ``F.linear`` (cuBLAS);
here each projection runs through the engine's own operator (``llmserve_b200.ops.gemm.linear`` on
a tile-packed weight: the stream-K decode GEMM plus its partial reduction for small T, the 2-SM
kernel for prefill-sized T), with the cuBLAS time beside it for comparison.  Two B200 additions:

* the weights of each projection are rotated among enough copies to exceed twice the 126 MB L2,
  so every timed call streams its weight from HBM as in a real decode step;
* each measurement reports the achieved weight bandwidth and its fraction of the measured HBM
  copy bandwidth (``MEASURED_PEAKS.json`` ``hbm_gbs`` when present).
"""
import argparse
import json
from dataclasses import dataclass
from pathlib import Path

from benchmarks.environment import atomic_write_json, build_environment_metadata, discover_model_revision

PROJECTION_NAMES = ("qkv", "o", "gate_up", "down")
L2_BYTES = 126 * 1024 * 1024
QWEN3_8B_NAME = "qwen3-8b"


@dataclass(frozen=True)
class LinearShape:
    name: str
    input_size: int
    output_size: int


def qwen3_projection_shapes(config, tp: int = 1) -> tuple:
    """(qkv, o, gate_up, down) shapes of one rank: column-parallel outputs and row-parallel
    inputs divided by ``tp``."""
    hidden, inter = int(config.hidden_size), int(config.intermediate_size)
    heads, kv_heads = int(config.num_attention_heads), int(config.num_key_value_heads)
    head_dim = getattr(config, "head_dim", None)
    if head_dim is None:
        if hidden % heads:
            raise ValueError("hidden_size must be divisible by num_attention_heads")
        head_dim = hidden // heads
    q, kv = heads * int(head_dim), kv_heads * int(head_dim)
    for what, v in (("query width", q), ("kv width", kv), ("intermediate", inter)):
        if v % tp:
            raise ValueError(f"{what} {v} is not divisible by tp={tp}")
    return (LinearShape("qkv", hidden, (q + 2 * kv) // tp), LinearShape("o", q // tp, hidden),
            LinearShape("gate_up", hidden, 2 * inter // tp), LinearShape("down", inter // tp, hidden))


def summarize_latencies(latencies_ms: dict, *, num_hidden_layers: int) -> dict:
    missing = [n for n in PROJECTION_NAMES if n not in latencies_ms]
    if missing:
        raise ValueError(f"missing projection latency: {', '.join(missing)}")
    total = sum(float(latencies_ms[n]) for n in PROJECTION_NAMES)
    if total <= 0:
        raise ValueError("projection latency total must be positive")
    if num_hidden_layers <= 0:
        raise ValueError("num_hidden_layers must be positive")
    return {"per_layer_total_ms": total, "model_projection_total_ms": total * num_hidden_layers,
            "share_pct": {n: float(latencies_ms[n]) / total * 100.0 for n in PROJECTION_NAMES}}


def parse_num_tokens(value: str) -> tuple:
    try:
        values = tuple(int(v.strip()) for v in value.split(","))
    except ValueError as e:
        raise ValueError("num_tokens must be comma-separated integers") from e
    if not values or any(v <= 0 for v in values):
        raise ValueError("num_tokens must contain positive integers")
    if len(set(values)) != len(values):
        raise ValueError("num_tokens values must be unique")
    return values


def measured_hbm_gbs():
    path = Path(__file__).resolve().parents[1] / "MEASURED_PEAKS.json"
    try:
        return float(json.loads(path.read_text())["hbm_gbs"])
    except (OSError, KeyError, ValueError):
        return None


def build_parser() -> argparse.ArgumentParser:
    p = argparse.ArgumentParser(description="Profile Qwen3 dense projection shapes with CUDA events.")
    p.add_argument("--model", required=True, help=f"HF Qwen3 directory, or '{QWEN3_8B_NAME}' for the built-in shape")
    p.add_argument("--dtype", choices=("bfloat16",), default="bfloat16")
    p.add_argument("--num-tokens", type=parse_num_tokens, default=parse_num_tokens("1,4,8,16"),
                   help="Comma-separated GEMM M values, not request concurrency.")
    p.add_argument("--tp", type=int, default=1, help="tensor-parallel degree of the per-rank shapes")
    p.add_argument("--warmup", type=int, default=10)
    p.add_argument("--repeats", type=int, default=50)
    p.add_argument("--device", default="cuda")
    p.add_argument("--no-cublas", action="store_true", help="skip the cuBLAS comparison column")
    p.add_argument("--output", type=Path)
    return p


def profile_projection_shapes(shapes, *, num_hidden_layers: int, num_tokens, measure_latency) -> list:
    """``measure_latency(shape, T)`` -> ms, or a dict with ``ms`` and extra per-shape fields."""
    results = []
    for t in num_tokens:
        lat, extra = {}, {}
        for shape in shapes:
            m = measure_latency(shape, t)
            if isinstance(m, dict):
                lat[shape.name] = float(m["ms"])
                extra[shape.name] = {k: v for k, v in m.items() if k != "ms"}
            else:
                lat[shape.name] = float(m)
        row = {"num_tokens": t, "latency_ms": lat,
               "summary": summarize_latencies(lat, num_hidden_layers=num_hidden_layers)}
        if extra:
            row["detail"] = extra
        results.append(row)
    return results


def _time_rotating(fn, operands, warmup: int, repeats: int) -> float:
    import torch
    for i in range(warmup):
        fn(*operands[i % len(operands)])
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for i in range(repeats):
        fn(*operands[i % len(operands)])
    end.record()
    end.synchronize()
    return start.elapsed_time(end) / repeats


def measure_dense_cuda(shape: LinearShape, *, num_tokens: int, device, warmup: int, repeats: int,
                       cublas: bool = True, hbm_gbs=None) -> dict:
    import torch
    import torch.nn.functional as F

    from llmserve_b200.ops import gemm
    from llmserve_b200.ops._ext import check_status
    if device.type != "cuda":
        raise ValueError("dense latency profiling requires a CUDA device")
    if warmup < 0 or repeats <= 0:
        raise ValueError("warmup must be non-negative and repeats must be positive")
    wbytes = shape.input_size * shape.output_size * 2
    copies = max(1, -(-2 * L2_BYTES // wbytes))
    with torch.cuda.device(device), torch.inference_mode():
        g = torch.Generator(device=device).manual_seed(0)
        x = torch.randn(num_tokens, shape.input_size, device=device, generator=g).bfloat16()
        dense = [(torch.randn(shape.output_size, shape.input_size, device=device, generator=g) * 0.02).bfloat16()
                 for _ in range(copies)]
        packed = [(x, gemm.pack_weight(w)) for w in dense]
        ms = _time_rotating(gemm.linear, packed, warmup, repeats)
        check_status(device)
        out = {"ms": ms, "weight_bytes": wbytes, "l2_rotation_copies": copies,
               "achieved_weight_gbps": wbytes / (ms * 1e-3) / 1e9,
               "path": "cluster split-K tile kernel" if gemm.use_cluster(num_tokens, packed[0][1])
               else "tile kernel"}
        if hbm_gbs:
            out["fraction_of_measured_hbm"] = out["achieved_weight_gbps"] / hbm_gbs
        if cublas:
            out["cublas_ms"] = _time_rotating(F.linear, [(x, w) for w in dense], warmup, repeats)
        return out


def main(argv=None):
    import torch
    from transformers import AutoConfig
    args = build_parser().parse_args(argv)
    if not torch.cuda.is_available():
        raise RuntimeError("CUDA is required for dense Linear profiling")
    if args.model == QWEN3_8B_NAME:
        from types import SimpleNamespace

        from llmserve_b200.models.synthetic import QWEN3_8B
        config = SimpleNamespace(**QWEN3_8B)
    else:
        config = AutoConfig.from_pretrained(args.model)
    if config.model_type != "qwen3":
        raise ValueError(f"expected a Qwen3 config, got {config.model_type!r}")
    shapes = qwen3_projection_shapes(config, args.tp)
    device = torch.device(args.device)
    hbm = measured_hbm_gbs()

    def measure(shape, t):
        return measure_dense_cuda(shape, num_tokens=t, device=device, warmup=args.warmup, repeats=args.repeats,
                                  cublas=not args.no_cublas, hbm_gbs=hbm)

    document = {
        "schema_version": 1, "benchmark": "qwen3-dense-linear", "metadata": build_environment_metadata(),
        "model": Path(args.model).name, "model_revision": discover_model_revision(args.model),
        "config": {"dtype": args.dtype, "device": str(device), "num_tokens": list(args.num_tokens),
                   "warmup": args.warmup, "repeats": args.repeats, "num_hidden_layers": int(config.num_hidden_layers),
                   "tp": args.tp, "kernel": "llmserve_b200 sm_100a tcgen05 GEMM", "measured_hbm_gbs": hbm},
        "shapes": [{"name": s.name, "input_size": s.input_size, "output_size": s.output_size,
                    "weight_elements": s.input_size * s.output_size,
                    "dense_weight_bytes_per_layer": s.input_size * s.output_size * 2} for s in shapes],
        "measurements": profile_projection_shapes(shapes, num_hidden_layers=int(config.num_hidden_layers),
                                                  num_tokens=args.num_tokens, measure_latency=measure),
    }
    if args.output is not None:
        atomic_write_json(args.output, document)
    print(json.dumps(document, indent=2))


if __name__ == "__main__":
    main()
