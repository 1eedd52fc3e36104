"""Row-parallel projection + TP reduction + residual + RMSNorm: fused NVLink kernel vs NCCL.

``torchrun --nproc-per-node N -m benchmarks.collective_profile [--tokens 1,16,64] [--hidden 4096]
[--inner 4096] [--iters 50]``  (N = 2..8, one process per GPU, NCCL for set-up)

For each token count T every rank runs the o_proj-shaped step of one decoder layer on its shard
(x [T, inner / N] @ W [hidden, inner / N]^T) followed by the reduction over ranks, the residual
add and the RMSNorm:

* ``fused``   -- the engine's path (``FusedComm.row_parallel_add_norm``): the tcgen05 GEMM's epilogue
  stores each token row's split-K partials into the inbox of the rank owning the row (peer
  stores of epoch-tagged words), then ``row_parallel_finish`` reduces the rank's rows from its own
  inbox, adds the residual, normalises, pushes the finished rows to every rank and unpacks the
  rows the peers pushed;
* ``nccl``    -- the baseline: the same GEMM (bf16 output), ``dist.all_reduce``, add+RMSNorm kernel;
* ``gemm``    -- the same GEMM alone writing local planes, to separate the collective's share
  (the finishing kernel cannot run alone: it waits for the GEMM's words of its own call).

Each variant's ``--iters`` back-to-back calls are captured in one CUDA graph (the form the decode
step runs them in, without Python launch overhead); times are CUDA events around one replay on
each rank, divided by ``--iters``, max over ranks.  The roofline of the fused step is the slowest of its weight bytes at the
measured HBM bandwidth, its FLOPs at the measured bf16 peak, and the bytes that cross NVLink per
rank at the measured 770 GB/s per direction (``roofline_us``); ``fraction`` = roofline / achieved.
"""
import argparse
import json
import os

NVLINK_GBS = 770.0           # measured peer copy, per direction per GPU


def fused_roofline_us(T: int, hidden: int, inner_shard: int, world: int, planes: int, hbm_gbs: float,
                      bf16_tflops: float, nvlink_gbs: float = NVLINK_GBS) -> dict:
    """Lower bound of one fused row-parallel step on one rank (µs) and its three terms."""
    rows = -(-T // world)
    weight_bytes = hidden * inner_shard * 2
    flops = 2.0 * T * hidden * inner_shard
    # the GEMM stores the fp32 partial planes of the other ranks' rows into their inboxes, then the
    # rank pushes its finished rows (normed output + residual, bf16) to the other ranks; every value
    # travels in an 8-byte epoch-tagged word (4 bytes of payload)
    link_bytes = (T - min(rows, T)) * hidden * 8 * planes + (world - 1) * min(rows, T) * hidden * 8
    terms = {"hbm_us": weight_bytes / (hbm_gbs * 1e3), "compute_us": flops / (bf16_tflops * 1e6),
             "nvlink_us": link_bytes / (nvlink_gbs * 1e3)}
    return dict(terms, roofline_us=max(terms.values()), nvlink_bytes=link_bytes, weight_bytes=weight_bytes)


def _peaks():
    path = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), float(p["bf16_tflops"])
    except (OSError, KeyError, ValueError):
        return 6650.0, 1590.0


def main(argv=None):
    import torch
    import torch.distributed as dist

    from llmserve_b200.ops import gemm, norm as norm_ops
    from llmserve_b200.parallel import state as tp
    from llmserve_b200.parallel.comm import FusedComm
    p = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    p.add_argument("--tokens", default="1,16,64")
    p.add_argument("--hidden", type=int, default=4096)
    p.add_argument("--inner", type=int, default=4096)
    p.add_argument("--iters", type=int, default=50)
    args = p.parse_args(argv)
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", rank)))
    torch.cuda.set_device(dev)
    tp.init_tensor_parallel(rank, world, "env://", dev, 120.0)
    tokens = [int(t) for t in args.tokens.split(",")]
    comm = FusedComm.create(dev, args.hidden, max(tokens))
    hbm, peak = _peaks()
    k = args.inner // world
    g = torch.Generator(device=dev).manual_seed(rank)
    # enough weight copies, used in turn, that the captured loop streams them from HBM (> L2)
    copies = max(1, -(-(256 << 20) // (args.hidden * k * 2)))
    ws = [gemm.pack_weight((torch.randn(args.hidden, k, device=dev, generator=g) * 0.02).bfloat16())
          for _ in range(copies)]
    w = ws[0]
    turn = [0]

    def next_w():
        turn[0] += 1
        return ws[turn[0] % copies]
    nw = torch.ones(args.hidden, device=dev).bfloat16()

    def timed(fn):
        """Device time per call: ``--iters`` calls captured in one CUDA graph (as the engine runs
        them), replayed after warm-up; CUDA events around one replay; max over ranks."""
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        dist.barrier()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=torch.cuda.Stream(device=dev)):
            for _ in range(args.iters):
                fn()
        torch.cuda.synchronize()
        dist.barrier()
        graph.replay()
        torch.cuda.synchronize()
        dist.barrier()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        graph.replay()
        b.record()
        torch.cuda.synchronize()
        del graph
        t = torch.tensor([a.elapsed_time(b) * 1e3 / args.iters], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t)

    with torch.inference_mode():
        for T in tokens:
            x = torch.randn(T, k, device=dev, generator=g).bfloat16()
            res = torch.randn(T, args.hidden, device=dev, generator=g).bfloat16()
            splits = min(gemm.splits_for(T, w), 8)
            # with the cluster-reduced GEMM the K splits meet on chip: one fp32 plane per row crosses
            planes = 1 if gemm.use_cluster(T, w) else splits
            row = {"tokens": T, "world": world, "hidden": args.hidden, "inner_shard": k, "planes": planes}
            if comm is not None and comm.can_handle(T, args.hidden):
                row["fused_us"] = timed(lambda: comm.row_parallel_add_norm(x, next_w(), res, nw, 1e-6))
            if planes == 1:
                row["gemm_us"] = timed(lambda: gemm.linear_reduced(x, next_w(), plane=True))
            else:
                row["gemm_us"] = timed(lambda: gemm.linear_partials(x, next_w(), splits))

            def nccl():
                y = gemm.linear(x, next_w())
                dist.all_reduce(y)
                norm_ops.add_rms_norm(y, res, nw, 1e-6)
            row["nccl_us"] = timed(nccl)
            row.update(fused_roofline_us(T, args.hidden, k, world, planes, hbm, peak))
            if "fused_us" in row:
                row["fraction_of_roofline"] = row["roofline_us"] / row["fused_us"]
            if rank == 0:
                print(json.dumps(row), flush=True)
    if comm is not None:
        comm.close()
    tp.destroy_tensor_parallel()


if __name__ == "__main__":
    main()
