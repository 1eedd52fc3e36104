"""Device timeline of serving steps: per-kernel exclusive time and GPU idle gaps.

``python -m benchmarks.step_timeline [--layers 36] [--concurrency 64] [--warmup 30] [--steps 5] [--tp N]
[--nccl-only] [--eagle3]``

Runs the headline closed-loop workload (Qwen3-8B shapes, random weights, 256-token prompts) to a
steady decode state, records ``--steps`` engine steps with ``torch.profiler`` (CUPTI kernel
activity: the kernels run at full speed, with programmatic dependent launch overlaps intact), and
reports for each kernel the time it alone extends the timeline (overlapping kernels are not
double counted) plus the idle gaps in which the GPU waited for the host.  Use it to see where a
step's time goes; time throughput with ``bench.py`` (CUDA events, no tracing).
"""
import argparse
import collections
import json
import re


def exclusive_times(rows):
    """rows: (name, start_us, end_us) sorted by start -> ({name: exclusive us}, {name: count}, idle us)."""
    excl, cnt = collections.defaultdict(float), collections.Counter()
    frontier, idle = rows[0][1], 0.0
    for name, s, e in rows:
        if s > frontier:
            idle += s - frontier
        excl[name] += max(0.0, e - max(s, frontier))
        cnt[name] += 1
        frontier = max(frontier, e)
    return excl, cnt, idle


def short_name(name: str) -> str:
    n = name.replace("(anonymous namespace)::", "").replace("void ", "")
    m = re.match(r"(?:lsb::)?([A-Za-z_0-9:]+)(<[^(]*>)?", n)
    return (m.group(1) + (m.group(2) or ""))[:60] if m else n[:60]


def main(argv=None):
    p = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    p.add_argument("--layers", type=int, default=36)
    p.add_argument("--concurrency", type=int, default=64)
    p.add_argument("--input-len", type=int, default=256)
    p.add_argument("--output-len", type=int, default=256)
    p.add_argument("--warmup", type=int, default=30)
    p.add_argument("--steps", type=int, default=5)
    p.add_argument("--mem-util", type=float, default=0.5)
    p.add_argument("--json", default=None, help="write the raw (name, start, end) rows here")
    p.add_argument("--tp", type=int, default=1, help="tensor-parallel size (the timeline is rank 0's GPU)")
    p.add_argument("--nccl-only", action="store_true", help="NCCL collectives instead of the fused NVLink path")
    p.add_argument("--eagle3", action="store_true",
                   help="EAGLE3 speculative steps (gamma 3, random-init Qwen3-8B speculator, step CUDA graphs)")
    args = p.parse_args(argv)

    import torch
    from torch.profiler import ProfilerActivity, profile

    import bench
    from llmserve_b200 import LLM, SamplingParams
    from llmserve_b200.engine.model_runner import GreedySampler
    extra = {}
    if args.eagle3:
        import os
        import tempfile

        from llmserve_b200.models.synthetic import EAGLE3_8B, write_config_only
        extra = dict(speculative_model=write_config_only(os.path.join(tempfile.gettempdir(), "llmserve_b200_eagle3_8b"),
                                                         EAGLE3_8B), speculative_gamma=3, speculative_cuda_graphs=True)
    llm = LLM(bench.model_dir(args.layers), load_format="dummy", max_model_len=args.input_len + args.output_len + 16,
              max_num_batched_tokens=max(16384, args.concurrency * args.input_len), max_num_seqs=args.concurrency,
              kvcache_block_size=256, gpu_memory_utilization=args.mem_util, tensor_parallel_size=args.tp,
              fused_collectives=not args.nccl_only, **extra)
    llm.model_runner.sampler = GreedySampler()
    stream = bench.request_stream(llm.config.hf_config.vocab_size, args.input_len)
    sp = SamplingParams(temperature=1.0, max_tokens=args.output_len, ignore_eos=True)
    active = 0

    def step():
        nonlocal active
        while active < args.concurrency:
            llm.add_request(next(stream), sp)
            active += 1
        outs, _ = llm.step()
        active -= len(outs)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        for _ in range(args.steps):
            step()
        torch.cuda.synchronize()
    llm.exit()
    rows = sorted(((e.name, e.time_range.start, e.time_range.end) for e in prof.events()
                   if e.device_type == torch.autograd.DeviceType.CUDA), key=lambda r: r[1])
    if args.json:
        with open(args.json, "w") as f:
            json.dump(rows, f)
    excl, cnt, idle = exclusive_times([(short_name(n), s, e) for n, s, e in rows])
    span = rows[-1][2] - rows[0][1]
    print(f"{args.steps} steps: {span / args.steps:.1f} us per step, GPU idle {idle / args.steps:.1f} us per step, "
          f"{len(rows) / args.steps:.0f} device activities per step")
    for k, v in sorted(excl.items(), key=lambda x: -x[1])[:20]:
        print(f"{v / args.steps:9.1f} us/step  x{cnt[k] / args.steps:6.1f}  {k}")


if __name__ == "__main__":
    main()
