"""Headline benchmark: closed-loop serving throughput of Qwen3-8B (BF16) on B200.

Metric and config come from BASELINE.json: output tok/s (with P99 TTFT / TPOT) for Qwen3-8B under a
closed loop of ``--concurrency`` requests of 256 input / 256 output tokens (prompt ids uniform over
the vocabulary, greedy decoding), tensor parallel over ``--gpus`` GPUs of one node.  Weights are
random N(0, 0.02) drawn on the device (no checkpoint download is possible); shapes are the real
model's.  One "step" is one engine step (schedule + forward + sample + postprocess).

``value``  : output tokens emitted in the K timed steps / device time of those steps (CUDA events on
             every rank, max over ranks).
``e2e``    : the same tokens / wall-clock time of the same steps through the public API
             (``LLM.add_request`` / ``LLM.step``), which includes the per-step host->device copy of
             the step inputs from pinned memory and the device->host read of the sampled tokens.

Usage: ``python bench.py [--gpus N --steps K --warmup W]``; for N > 1 launch with
``torchrun --nproc-per-node N bench.py --gpus N ...`` (one rank per GPU).  ``--impl reference`` runs
the unmodified reference build from ``baseline/_ref`` on the same workload.
"""
import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "output tok/s + P99 TTFT/TPOT, Qwen3-8B closed-loop, TP 1/2/4/8 vs ref build"


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=int(os.environ.get("WORLD_SIZE", 1)))
    p.add_argument("--steps", type=int, default=257)
    p.add_argument("--warmup", type=int, default=20)
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--concurrency", type=int, default=64)
    p.add_argument("--input-len", type=int, default=256)
    p.add_argument("--output-len", type=int, default=256)
    p.add_argument("--layers", type=int, default=36)
    p.add_argument("--eager", action="store_true")
    p.add_argument("--awq", action="store_true",
                   help="AutoAWQ 4-bit g128 Qwen3-8B (random codes/zeros, |N(0,1)|*0.01 scales) on the W4A16 kernel")
    p.add_argument("--nccl-only", action="store_true", help="disable the fused NVLink collectives")
    p.add_argument("--eagle3", action="store_true",
                   help="EAGLE3 speculative decoding, gamma 3, with a random-init Qwen3-8B speculator (1 layer, "
                        "fc 12288->4096, draft vocab 32000); acceptance is not meaningful with random weights")
    p.add_argument("--spec-graphs", action="store_true",
                   help="with --eagle3: run the greedy speculative step through its CUDA graphs")
    p.add_argument("--mem-util", type=float, default=0.85, help="gpu_memory_utilization (KV pool sizing)")
    p.add_argument("--no-overlap", action="store_true",
                   help="synchronous decode loop (no launch of step N+1 before step N's tokens are read)")
    p.add_argument("--profile-range", action="store_true",
                   help="bracket the timed steps with cudaProfilerStart/Stop (for ncu --profile-from-start off)")
    return p.parse_args()


class ClockSampler:
    """SM clocks, power and clock-event reasons of the job's GPUs, sampled every 10 ms by a thread
    during the timed region through NVML (read-only queries; GPUs found by PCI bus id, so the CUDA
    and NVML orderings need not agree).  One sample is taken on entry and one on exit, so even a
    window of a few steps has samples.  Falls back to ``nvidia-smi -lms 50`` without NVML."""

    REASONS = (("hw_slowdown", "nvmlClocksEventReasonHwSlowdown"),
               ("hw_thermal_slowdown", "nvmlClocksEventReasonHwThermalSlowdown"),
               ("sw_thermal_slowdown", "nvmlClocksEventReasonSwThermalSlowdown"),
               ("sw_power_cap", "nvmlClocksEventReasonSwPowerCap"))

    def __init__(self, indices, interval_s: float = 0.01):
        self.indices = indices
        self.interval_s = interval_s
        self.rows = []          # (sm_mhz, max_mhz, power_w, reasons)
        self.proc = None
        self.nvml = None
        self.path = os.path.join(tempfile.mkdtemp(), "clocks.csv")

    def _nvml_handles(self):
        import pynvml
        import torch
        pynvml.nvmlInit()
        handles = []
        for i in range(len(self.indices)):
            p = torch.cuda.get_device_properties(i)
            bus = f"{p.pci_domain_id:08x}:{p.pci_bus_id:02x}:{p.pci_device_id:02x}.0"
            handles.append(pynvml.nvmlDeviceGetHandleByPciBusId(bus))
        return pynvml, handles

    def _sample(self):
        nv, handles = self.nvml
        for h in handles:
            mask = nv.nvmlDeviceGetCurrentClocksEventReasons(h)
            self.rows.append((float(nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM)),
                              float(nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM)),
                              nv.nvmlDeviceGetPowerUsage(h) / 1000.0,
                              {name for name, bit in self.REASONS if mask & getattr(nv, bit)}))

    def _loop(self):
        while not self._stop.wait(self.interval_s):
            self._sample()

    def __enter__(self):
        import threading
        try:
            self.nvml = self._nvml_handles()
            self._sample()
            self._stop = threading.Event()
            self._thread = threading.Thread(target=self._loop, daemon=True)
            self._thread.start()
            return self
        except Exception:
            self.nvml = None
        q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
        try:
            self.f = open(self.path, "w")
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={q}", "--format=csv,noheader,nounits",
                                          "-lms", "50", "-i", ",".join(map(str, self.indices))],
                                         stdout=self.f, stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.nvml is not None:
            self._stop.set()
            self._thread.join(timeout=5)
            self._sample()
            self.nvml[0].nvmlShutdown()
        if self.proc is not None:
            self.proc.terminate()
            self.proc.wait(timeout=10)
            self.f.close()
            self._read_csv()

    def _read_csv(self):
        names = [n for n, _ in self.REASONS]
        try:
            for line in open(self.path):
                parts = [x.strip() for x in line.split(",")]
                if len(parts) >= 9 and parts[1].replace(".", "").isdigit():
                    power = float(parts[3]) if parts[3].replace(".", "").isdigit() else 0.0
                    self.rows.append((float(parts[1]), float(parts[2]), power,
                                      {n for n, v in zip(names, parts[5:9]) if v.lower() == "active"}))
        except OSError:
            pass

    def summary(self):
        if not self.rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        return {"sm_mhz": statistics.median(r[0] for r in self.rows), "sm_max_mhz": max(r[1] for r in self.rows),
                "power_w_max": round(max(r[2] for r in self.rows), 1), "samples": len(self.rows),
                "source": "nvml" if self.nvml is not None else "nvidia-smi",
                "reasons": sorted(set().union(*(r[3] for r in self.rows)))}


def visible_indices(n):
    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    if vis:
        return [int(x) for x in vis.split(",")[:n]]
    return list(range(n))


def model_dir(layers: int, awq: bool = False) -> str:
    from llmserve_b200.models.synthetic import AWQ_QUANT_CONFIG, QWEN3_8B, write_config_only
    cfg = dict(QWEN3_8B, num_hidden_layers=layers)
    if awq:
        cfg.update(torch_dtype="bfloat16", quantization_config=dict(AWQ_QUANT_CONFIG))
    path = os.path.join(tempfile.gettempdir(), f"llmserve_b200_qwen3_8b_L{layers}{'_awq' if awq else ''}")
    write_config_only(path, cfg)
    return path


def request_stream(vocab, n_in, seed=0):
    import random
    rng = random.Random(seed)
    while True:
        yield [rng.randrange(vocab) for _ in range(n_in)]


def window_latency(metrics: list[dict]) -> dict:
    """P50 / P99 TTFT and TPOT (the engine's definitions: first token - arrival; (finish - first) /
    (tokens - 1)) over the finished requests among ``metrics`` (the engine's request records)."""
    from llmserve_b200.engine.llm_engine import percentile
    done = [m for m in metrics if m["finish_time"] is not None and m["first_token_time"] is not None]
    ttft = [m["first_token_time"] - m["arrival_time"] for m in done]
    tpot = [(m["finish_time"] - m["first_token_time"]) / (m["output_tokens"] - 1) for m in done
            if m["output_tokens"] > 1]

    def ms(v, q, nd):
        x = percentile(v, q)
        return None if x is None else round(x * 1e3, nd)
    return {"requests": len(done), "ttft_p50_ms": ms(ttft, 50, 2), "ttft_p99_ms": ms(ttft, 99, 2),
            "tpot_p50_ms": ms(tpot, 50, 3), "tpot_p99_ms": ms(tpot, 99, 3)}


def run_ours(args):
    import torch

    from llmserve_b200 import LLM, SamplingParams
    from llmserve_b200.engine.llm_engine import run_worker
    from llmserve_b200.engine.model_runner import GreedySampler

    rank = int(os.environ.get("RANK", 0))
    world = args.gpus
    kwargs = dict(load_format="dummy", tensor_parallel_size=world, enforce_eager=args.eager,
                  max_model_len=args.input_len + args.output_len + 16,
                  max_num_batched_tokens=max(16384, args.concurrency * args.input_len),
                  max_num_seqs=args.concurrency, kvcache_block_size=256, gpu_memory_utilization=args.mem_util,
                  fused_collectives=not args.nccl_only, comm_timeout_s=300.0, overlap_decode=not args.no_overlap)
    if world > 1:
        kwargs.update(distributed_launcher="external", distributed_init_method="env://",
                      rpc_channel=f"llmserve_b200_bench_{os.environ.get('MASTER_PORT', '0')}")
    path = model_dir(args.layers, args.awq)
    if args.eagle3:
        from llmserve_b200.models.synthetic import EAGLE3_8B, write_config_only
        kwargs.update(speculative_model=write_config_only(os.path.join(tempfile.gettempdir(), "llmserve_b200_eagle3_8b"),
                                                          EAGLE3_8B), speculative_gamma=3,
                      speculative_cuda_graphs=args.spec_graphs)
    if rank > 0:
        run_worker(path, rank, **kwargs)
        return
    llm = LLM(path, **kwargs)
    llm.model_runner.sampler = GreedySampler()
    vocab = llm.config.hf_config.vocab_size
    stream = request_stream(vocab, args.input_len)
    sp = SamplingParams(temperature=1.0, max_tokens=args.output_len, ignore_eos=True)
    active = 0

    def refill():
        nonlocal active
        while active < args.concurrency:
            llm.add_request(next(stream), sp)
            active += 1

    def tokens_so_far():
        return sum(len(m["token_times"]) for m in llm.request_metrics.values())

    refill()
    for _ in range(args.warmup):
        outs, _ = llm.step()
        active -= len(outs)
        refill()
    runner = llm.model_runner
    # the timed window: a barrier + synchronize on every rank on both sides; the step in flight from
    # the warm-up (overlapped loop) completes before the start mark, so the window holds the GPU work
    # of exactly the timed steps' launches
    # the clock sampler starts (NVML set-up) before the window opens, so its set-up is in neither clock
    with ClockSampler(visible_indices(world)) as clocks:
        runner.call("mark_event", "bench_start", "before")
        tok0 = tokens_so_far()
        h2d0, d2h0 = runner.h2d_bytes, runner.d2h_bytes
        if args.profile_range:
            torch.cuda.profiler.start()
        t0 = time.perf_counter()
        for _ in range(args.steps):
            outs, _ = llm.step()
            active -= len(outs)
            refill()
        runner.call("mark_event", "bench_end", "after")
        wall = time.perf_counter() - t0
    if args.profile_range:
        torch.cuda.profiler.stop()
    per_rank = runner.call("gather_elapsed", "bench_start", "bench_end")
    tokens = tokens_so_far() - tok0
    dev_ms = max(r[0] for r in per_rank)
    launches = int(per_rank[0][1])
    h2d = (runner.h2d_bytes - h2d0) / args.steps
    d2h = (runner.d2h_bytes - d2h0) / args.steps
    # Latency window (after the timed steps, not part of `value`): keep the closed loop running
    # until one full wave of requests admitted after this point has finished, so P99 TTFT / TPOT
    # come from complete requests whatever --steps is.
    seen = set(llm.request_metrics)
    lat_steps = 0
    while True:
        new = [m for k, m in llm.request_metrics.items() if k not in seen]
        if sum(m["finish_time"] is not None for m in new) >= args.concurrency or lat_steps > 20 * args.output_len:
            break
        outs, _ = llm.step()
        active -= len(outs)
        refill()
        lat_steps += 1
    latency = window_latency([m for k, m in llm.request_metrics.items() if k not in seen])
    latency["window"] = (f"{lat_steps} steps after the timed ones: the {latency['requests']} requests admitted "
                         "after the timed steps, once a full wave of them finished")
    m = llm.get_metrics()["summary"]
    llm.exit()
    value = tokens / (dev_ms / 1e3)
    line = {
        "metric": METRIC, "value": round(value, 2), "unit": "tok/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(dev_ms / args.steps, 4), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic: random-init Qwen3-8B weights N(0,0.02), prompt ids uniform over the vocab",
        "config": {"model": ("Qwen3-8B" if args.layers == 36 else f"Qwen3-8B-{args.layers}L") + ("-AWQ" if args.awq else "")
                   + ("+EAGLE3" if args.eagle3 else ""),
                   "global_batch": args.concurrency, "seq_len": args.input_len + args.output_len,
                   "parallelism": f"tp{world}", "workload": f"closed-loop {args.input_len} in / {args.output_len} out, "
                   f"concurrency {args.concurrency}, greedy", "cuda_graphs": not args.eager,
                   "collectives": "nccl" if args.nccl_only or world == 1 else "fused-nvlink",
                   "overlapped_decode": not args.no_overlap,
                   "speculative_graphs": bool(args.eagle3 and args.spec_graphs),
                   "l2": "inputs larger than L2: every step streams all 16 GB of weights"},
        "e2e": {"value": round(tokens / wall, 2), "unit": "tok/s", "h2d_bytes_per_step": round(h2d),
                "d2h_bytes_per_step": round(d2h)},
        "gpu_launches": launches,
        "latency": latency,
        "per_rank_device_ms": [round(r[0], 3) for r in per_rank],
        "speculative": None if not args.eagle3 else {
            k: m["speculative"].get(k) for k in ("steps", "acceptance_rate", "acceptance_length", "mean_batch_size")}
        | {"step_latency_p50_ms": None if m["speculative_step_latency"]["p50"] is None
           else round(m["speculative_step_latency"]["p50"] * 1e3, 3)},
        "clocks": clocks.summary(),
        "impl": "ours",
    }
    print(json.dumps(line), flush=True)


REF_TP_UNAVAILABLE = (
    "reference tensor parallelism fails in its stock code path: Sequence.__getstate__ does not ship seq_id "
    "(llmserve/engine/sequence.py:91-93) but ModelRunner.prepare_prefill reads seq.seq_id on every rank "
    "(llmserve/engine/model_runner.py:277-281), so worker ranks raise AttributeError on the first prefill "
    "and rank 0 waits in an NCCL all-reduce until the 600 s watchdog")


def run_reference(args):
    rank = int(os.environ.get("RANK", 0))
    ref = os.path.join(ROOT, "baseline", "_ref")
    why = None
    if not os.path.isdir(os.path.join(ref, "llmserve")):
        why = "reference build not installed under baseline/_ref"
    elif args.gpus > 1:
        why = REF_TP_UNAVAILABLE
    if why:
        if rank == 0:
            print(json.dumps({"impl": "reference", "unavailable": why}), flush=True)
        return
    sys.path.insert(0, os.path.join(ROOT, "baseline"))
    from ref_arm import run as ref_run  # noqa: E402
    ref_run(args, METRIC, window_latency, ClockSampler(visible_indices(1)))


def main():
    args = parse()
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
