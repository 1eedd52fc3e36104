"""Prefill and tree-verify attention kernels on one GPU: tcgen05 vs mma.sync / CUDA-core vs flash-attn / SDPA.

``python -m benchmarks.attention_profile [--heads 32] [--kv-heads 8] [--head-dim 128] [--iters 20]``

Workloads (Qwen3-8B head layout by default, bf16, causal, keys in the paged pool with 256-token
blocks):

* ``prompt4096``   one 4096-token prompt;
* ``batch8x512``   eight 512-token prompts;
* ``chunk2048``    a 2048-token chunk after a cached 2048-token prefix (chunked prefill);
* ``mixed``        the mixed-serving shape: 4 x 128 + 1 x 4096 prompts in one step.

Tree-verify workloads (``--workloads tree10_p2048,...``; EAGLE3 tree speculation of one sequence:
``n`` draft-tree nodes against a ``p``-token prefix in the pool plus the tree's own keys under the
ancestor mask of the fixed tree topology): the tcgen05 tree kernel, the CUDA-core tree kernel and
the reference's formulation (gather the prefix pages, concatenate the tree keys, masked SDPA), with
the K/V bytes each KV head must read once as the roofline.

Each kernel is timed with CUDA events around ``--iters`` back-to-back calls after warm-up (inputs
stay L2-resident only for the smallest workloads; the numbers are per call).  FLOPs count the
causal work actually needed, ``4 * head_dim * heads * sum(keys attended per query row)``, and
are reported as TFLOP/s and as a fraction of the measured bf16 GEMM peak (``MEASURED_PEAKS.json``).
flash-attn (the reference engine's prefill kernel) runs ``flash_attn_varlen_func`` with the same
block table when it is importable.
"""
import argparse
import json
import math
import os


def causal_flops(shapes, heads: int, head_dim: int) -> float:
    """shapes: (q_len, k_len) per sequence; query row i of a sequence sees k_len - q_len + i + 1 keys."""
    rows = 0
    for q, k in shapes:
        shift = k - q
        rows += q * shift + q * (q + 1) // 2
    return 4.0 * head_dim * heads * rows


WORKLOADS = {
    "prompt4096": [(4096, 4096)],
    "batch8x512": [(512, 512)] * 8,
    "chunk2048": [(2048, 4096)],
    "mixed": [(128, 128)] * 4 + [(4096, 4096)],
}


TREE_WORKLOADS = {          # (draft nodes of the fixed EAGLE3 tree, prefix tokens)
    "tree6_p512": (6, 512),
    "tree10_p2048": (10, 2048),
    "tree10_p4096": (10, 4096),
}


def _hbm_peak():
    path = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            return float(json.load(f)["hbm_gbs"])
    except (OSError, KeyError, ValueError):
        return 6650.0


def tree_row(name, nh, nkv, hd, bs, timed, dev, g):
    """One tree-verify workload: tcgen05 kernel vs CUDA-core kernel vs gather + masked SDPA."""
    import torch
    import torch.nn.functional as F

    from llmserve_b200.ops import attention
    from llmserve_b200.speculative.tree import build_fixed_tree_topology
    n, prefix = TREE_WORKLOADS[name]
    topo = build_fixed_tree_topology(n)
    n = len(topo.parents)
    nblk = -(-prefix // bs)
    kc = (torch.randn(nblk, nkv, bs, hd, device=dev, generator=g) * 0.5).bfloat16()
    vc = torch.randn(nblk, nkv, bs, hd, device=dev, generator=g).bfloat16()
    table = torch.randperm(nblk, device=dev).to(torch.int32)
    q = torch.randn(n, nh, hd, device=dev, generator=g).bfloat16()
    tk = (torch.randn(n, nkv, hd, device=dev, generator=g) * 0.5).bfloat16()
    tv = torch.randn(n, nkv, hd, device=dev, generator=g).bfloat16()
    mask = topo.attention_mask(dev)
    w = 1 << torch.arange(n, dtype=torch.int64, device=dev)
    bits = (mask.long() * w).sum(1).to(torch.int32)
    scale = 1.0 / math.sqrt(hd)

    def run(tc):
        saved = attention.TREE_TC
        attention.TREE_TC = tc
        try:
            return attention.tree_attention(q, kc, vc, table, prefix, tk, tv, mask, scale, bits)
        finally:
            attention.TREE_TC = saved

    full_mask = torch.cat([torch.ones(n, prefix, dtype=torch.bool, device=dev), mask], 1)

    def sdpa():
        k = torch.cat([attention._gather_pages(kc, table, prefix), tk], 0)
        v = torch.cat([attention._gather_pages(vc, table, prefix), tv], 0)
        G = nh // nkv
        kk = k.transpose(0, 1).repeat_interleave(G, 0)
        vv = v.transpose(0, 1).repeat_interleave(G, 0)
        return F.scaled_dot_product_attention(q.transpose(0, 1), kk, vv, attn_mask=full_mask,
                                              scale=scale).transpose(0, 1)

    tc, cc, ref = run(True), run(False), sdpa()
    torch.cuda.synchronize()
    err = lambda a: float(((a.float() - ref.float()).norm() / ref.float().norm()).item())
    kv_bytes = 2 * (prefix + n) * nkv * hd * 2
    row = {"workload": name, "tree_nodes": n, "prefix": prefix, "heads": nh, "kv_heads": nkv, "head_dim": hd,
           "block_size": bs, "kv_mb": round(kv_bytes / 1e6, 2), "tc_rel_err_vs_sdpa": err(tc),
           "cuda_core_rel_err_vs_sdpa": err(cc)}
    for key, fn in (("tc", lambda: run(True)), ("cuda_core", lambda: run(False)), ("sdpa", sdpa)):
        us = timed(fn)
        row[f"{key}_us"] = round(us, 1)
        row[f"{key}_gbs"] = round(kv_bytes / us / 1e3, 1)
    row["tc_fraction_of_measured_hbm"] = round(row["tc_gbs"] / _hbm_peak(), 3)
    return row


def _peak():
    path = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            return float(json.load(f)["bf16_tflops"])
    except (OSError, KeyError, ValueError):
        return 1590.0


def main(argv=None):
    import torch

    from llmserve_b200.ops import attention
    p = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    p.add_argument("--heads", type=int, default=32)
    p.add_argument("--kv-heads", type=int, default=8)
    p.add_argument("--head-dim", type=int, default=128)
    p.add_argument("--block-size", type=int, default=256)
    p.add_argument("--iters", type=int, default=20)
    p.add_argument("--workloads", default=",".join(WORKLOADS))
    args = p.parse_args(argv)
    dev = torch.device("cuda", 0)
    nh, nkv, hd, bs = args.heads, args.kv_heads, args.head_dim, args.block_size
    scale = 1.0 / math.sqrt(hd)
    peak = _peak()
    try:
        from flash_attn import flash_attn_varlen_func
    except Exception:  # pragma: no cover - depends on the image
        flash_attn_varlen_func = None

    def timed(fn):
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(args.iters):
            fn()
        b.record()
        torch.cuda.synchronize()
        return a.elapsed_time(b) * 1e3 / args.iters

    g = torch.Generator(device=dev).manual_seed(0)
    for name in args.workloads.split(","):
        if name in TREE_WORKLOADS:
            print(json.dumps(tree_row(name, nh, nkv, hd, bs, timed, dev, g)), flush=True)
            continue
        shapes = WORKLOADS[name]
        nblk_seq = [-(-k // bs) for _, k in shapes]
        nblk = sum(nblk_seq)
        kc = (torch.randn(nblk, nkv, bs, hd, device=dev, generator=g) * 0.5).bfloat16()
        vc = torch.randn(nblk, nkv, bs, hd, device=dev, generator=g).bfloat16()
        width = max(nblk_seq)
        tables = torch.zeros(len(shapes), width, dtype=torch.int32, device=dev)
        off = 0
        for i, n in enumerate(nblk_seq):
            tables[i, :n] = torch.arange(off, off + n, dtype=torch.int32, device=dev)
            off += n
        cu = [0]
        for q, _ in shapes:
            cu.append(cu[-1] + q)
        q = torch.randn(cu[-1], nh, hd, device=dev, generator=g).bfloat16()
        cu_q = torch.tensor(cu, dtype=torch.int32, device=dev)
        ks = torch.tensor([k for _, k in shapes], dtype=torch.int32, device=dev)
        max_q = max(s[0] for s in shapes)
        flops = causal_flops(shapes, nh, hd)
        row = {"workload": name, "shapes": shapes[:2] + (["..."] if len(shapes) > 2 else []), "heads": nh,
               "kv_heads": nkv, "head_dim": hd, "block_size": bs, "gflop": round(flops / 1e9, 2)}
        tc = attention.prefill_attention(q, kc, vc, cu_q, ks, tables, scale, max_q, kernel="tc")
        mm = attention.prefill_attention(q, kc, vc, cu_q, ks, tables, scale, max_q, kernel="mma")
        torch.cuda.synchronize()
        row["tc_vs_mma_rel_err"] = float(((tc.float() - mm.float()).norm() / mm.float().norm()).item())
        for kname in ("tc", "mma"):
            us = timed(lambda k=kname: attention.prefill_attention(q, kc, vc, cu_q, ks, tables, scale, max_q,
                                                                   kernel=k))
            row[f"{kname}_us"] = round(us, 1)
            row[f"{kname}_tflops"] = round(flops / us / 1e6, 1)
        if flash_attn_varlen_func is not None and bs % 256 == 0:
            cu_k = torch.tensor([0] + list(torch.tensor([k for _, k in shapes]).cumsum(0).tolist()), dtype=torch.int32,
                                device=dev)
            kp = kc.transpose(1, 2).contiguous()     # flash-attn's paged layout: [blocks, block, kv_heads, hd]
            vp = vc.transpose(1, 2).contiguous()
            max_k = max(k for _, k in shapes)
            try:
                fa = lambda: flash_attn_varlen_func(q, kp, vp, cu_q, cu_k, max_q, max_k, softmax_scale=scale,
                                                    causal=True, block_table=tables)
                ref = fa()
                torch.cuda.synchronize()
                row["tc_vs_flash_rel_err"] = float(((tc.float() - ref.float()).norm() / ref.float().norm()).item())
                us = timed(fa)
                row["flash_attn_us"] = round(us, 1)
                row["flash_attn_tflops"] = round(flops / us / 1e6, 1)
            except Exception as e:  # pragma: no cover - depends on the flash-attn build
                row["flash_attn_error"] = str(e)[:200]
        row["tc_fraction_of_measured_bf16_peak"] = round(row["tc_tflops"] / peak, 3)
        print(json.dumps(row), flush=True)


if __name__ == "__main__":
    main()
