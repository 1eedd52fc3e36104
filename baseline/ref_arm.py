"""``bench.py --impl reference``: the unmodified reference build (``baseline/_ref``) on the same
closed-loop workload, through its own public API (``llmserve.LLM`` / ``add_request`` / ``step``).

Nothing of llmserve_b200 runs on this path.  This module only (1) writes a checkpoint directory the
reference can load -- random N(0, 0.02) bf16 weights with the HF Qwen3 names (the reference only
loads from disk), ``config.json`` and a word-level tokenizer (prompts are passed as token ids) --
cached under the system temp dir, and (2) times the reference's engine steps with CUDA events on
its rank-0 device (its TP workers are its own spawned processes, synchronised with rank 0 by NCCL
every step).  Under torchrun, ranks > 0 exit immediately so the reference can use their GPUs.
"""
import json
import os
import socket
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF = os.path.join(ROOT, "baseline", "_ref")


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _write_tokenizer(path, vocab_size, eos):
    from tokenizers import Tokenizer, models, pre_tokenizers
    vocab = {f"t{i}": i for i in range(vocab_size)}
    tok = Tokenizer(models.WordLevel(vocab=vocab, unk_token="t0"))
    tok.pre_tokenizer = pre_tokenizers.Whitespace()
    tok.save(os.path.join(path, "tokenizer.json"))
    with open(os.path.join(path, "tokenizer_config.json"), "w") as f:
        json.dump({"tokenizer_class": "PreTrainedTokenizerFast", "eos_token": f"t{eos}", "unk_token": "t0",
                   "model_max_length": 1 << 20}, f)


def make_checkpoint(layers: int) -> str:
    import torch
    from safetensors.torch import save_file
    sys.path.insert(0, ROOT)
    from llmserve_b200.models.synthetic import QWEN3_8B  # shapes only (a dict of numbers)
    cfg = dict(QWEN3_8B, num_hidden_layers=layers, dtype="bfloat16")
    path = os.path.join(tempfile.gettempdir(), f"lsb_ref_qwen3_8b_L{layers}")
    done = os.path.join(path, ".complete")
    if os.path.exists(done):
        return path
    os.makedirs(path, exist_ok=True)
    with open(os.path.join(path, "config.json"), "w") as f:
        json.dump(cfg, f)
    _write_tokenizer(path, cfg["vocab_size"], cfg["eos_token_id"])
    H, I, V = cfg["hidden_size"], cfg["intermediate_size"], cfg["vocab_size"]
    nh, nkv, hd = cfg["num_attention_heads"], cfg["num_key_value_heads"], cfg["head_dim"]
    g = torch.Generator(device="cuda").manual_seed(0)

    def rnd(*shape):
        return (torch.randn(*shape, device="cuda", generator=g, dtype=torch.float32) * 0.02).bfloat16().cpu()

    def ones(n):
        return torch.ones(n, dtype=torch.bfloat16)

    shard, size, idx = {}, 0, 0

    def add(name, t):
        nonlocal shard, size, idx
        shard[name] = t
        size += t.numel() * 2
        if size > (3 << 30):
            save_file(shard, os.path.join(path, f"model-{idx:05d}.safetensors"))
            shard, size, idx = {}, 0, idx + 1

    add("model.embed_tokens.weight", rnd(V, H))
    for i in range(layers):
        p = f"model.layers.{i}."
        add(p + "self_attn.q_proj.weight", rnd(nh * hd, H))
        add(p + "self_attn.k_proj.weight", rnd(nkv * hd, H))
        add(p + "self_attn.v_proj.weight", rnd(nkv * hd, H))
        add(p + "self_attn.o_proj.weight", rnd(H, nh * hd))
        add(p + "self_attn.q_norm.weight", ones(hd))
        add(p + "self_attn.k_norm.weight", ones(hd))
        add(p + "mlp.gate_proj.weight", rnd(I, H))
        add(p + "mlp.up_proj.weight", rnd(I, H))
        add(p + "mlp.down_proj.weight", rnd(H, I))
        add(p + "input_layernorm.weight", ones(H))
        add(p + "post_attention_layernorm.weight", ones(H))
    add("model.norm.weight", ones(H))
    add("lm_head.weight", rnd(V, H))
    if shard:
        save_file(shard, os.path.join(path, f"model-{idx:05d}.safetensors"))
    open(done, "w").close()
    return path


def make_eagle3_checkpoint() -> str:
    """A random-init EAGLE3 speculator for the Qwen3-8B shape in the RedHat layout (one decoder
    layer, fc 3 x 4096 -> 4096, draft vocabulary 32000 with d2t / t2d); data only."""
    sys.path.insert(0, ROOT)
    from llmserve_b200.models.synthetic import QWEN3_8B, write_eagle3_checkpoint
    path = os.path.join(tempfile.gettempdir(), "lsb_ref_eagle3_qwen3_8b")
    done = os.path.join(path, ".complete")
    if not os.path.exists(done):
        write_eagle3_checkpoint(path, QWEN3_8B, draft_vocab=32000, nested=True, include_embedding=False)
        open(done, "w").close()
    return path


def run(args, metric: str, window_latency, clocks=None):
    rank = int(os.environ.get("RANK", 0))
    if rank > 0:
        return          # the reference spawns its own tensor-parallel workers from rank 0
    import torch
    t_ckpt = time.perf_counter()
    path = make_checkpoint(args.layers)
    t_ckpt = time.perf_counter() - t_ckpt
    sys.path.insert(0, REF)
    import llmserve
    from llmserve import LLM, SamplingParams
    if not os.path.abspath(llmserve.__file__).startswith(os.path.abspath(REF)):
        raise RuntimeError("reference package did not resolve to baseline/_ref")
    import random
    world = args.gpus
    # The reference spawns its own workers and rendezvouses over its tcp:// init method.  Under
    # torchrun the launcher's variables (TORCHELASTIC_USE_AGENT_STORE in particular, which turns a
    # tcp:// rendezvous into a client of a store nobody serves) would leak into it: drop them so
    # the reference runs exactly as it does when started on its own.
    for key in [k for k in os.environ if k.startswith(("TORCHELASTIC_", "TORCH_ELASTIC_"))] + [
            "RANK", "LOCAL_RANK", "WORLD_SIZE", "LOCAL_WORLD_SIZE", "GROUP_RANK", "ROLE_RANK", "ROLE_WORLD_SIZE",
            "GROUP_WORLD_SIZE", "ROLE_NAME", "MASTER_ADDR", "MASTER_PORT"]:
        os.environ.pop(key, None)
    eagle3 = bool(getattr(args, "eagle3", False))
    # the reference speculates only in eager mode (its llm_engine.py:359-368), so --eagle3 runs eager
    extra = dict(speculative_model=make_eagle3_checkpoint(), speculative_gamma=3) if eagle3 else {}
    llm = LLM(path, tensor_parallel_size=world, enforce_eager=args.eager or eagle3,
              max_model_len=args.input_len + args.output_len + 16,
              max_num_batched_tokens=max(16384, args.concurrency * args.input_len), max_num_seqs=args.concurrency,
              distributed_init_method=f"tcp://127.0.0.1:{_free_port()}", **extra)

    class ArgmaxSampler:            # the reference benchmark's sampler (benchmarks/serve.py)
        def __call__(self, logits, temperatures):
            return logits.argmax(dim=-1)

    llm.model_runner.sampler = ArgmaxSampler()
    rng = random.Random(0)
    vocab = 151936
    sp = SamplingParams(temperature=0.01, max_tokens=args.output_len, ignore_eos=True)
    active = 0

    def refill():
        nonlocal active
        while active < args.concurrency:
            llm.add_request([rng.randrange(vocab) for _ in range(args.input_len)], sp)
            active += 1

    def tokens():
        return sum(len(m["token_times"]) for m in llm.request_metrics.values())

    refill()
    for _ in range(args.warmup):
        outs, _ = llm.step()
        active -= len(outs)
        refill()
    # the clock sampler (this repo's bench.ClockSampler: read-only NVML queries on a thread) starts
    # before the window opens, as in the llmserve_b200 arm
    if clocks is not None:
        clocks.__enter__()
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    tok0 = tokens()
    start.record()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        outs, _ = llm.step()
        active -= len(outs)
        refill()
    end.record()
    torch.cuda.synchronize()
    wall = time.perf_counter() - t0
    if clocks is not None:
        clocks.__exit__(None, None, None)
    ms = start.elapsed_time(end)
    n = tokens() - tok0
    # the same latency window as the llmserve_b200 arm: one full wave of requests admitted after
    # the timed steps, run to completion
    seen = set(llm.request_metrics)
    lat_steps = 0
    while True:
        new = [r for k, r in llm.request_metrics.items() if k not in seen]
        if sum(r["finish_time"] is not None for r in new) >= args.concurrency or lat_steps > 20 * args.output_len:
            break
        outs, _ = llm.step()
        active -= len(outs)
        refill()
        lat_steps += 1
    latency = window_latency([r for k, r in llm.request_metrics.items() if k not in seen])
    latency["window"] = (f"{lat_steps} steps after the timed ones: the {latency['requests']} requests admitted "
                         "after the timed steps, once a full wave of them finished")
    m = llm.get_metrics()["summary"]
    llm.exit()
    print(json.dumps({
        "impl": "reference", "metric": metric, "value": round(n / (ms / 1e3), 2), "unit": "tok/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms / args.steps, 4),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic: random-init Qwen3-8B weights N(0,0.02) written as HF safetensors, prompt ids uniform over the vocab",
        "config": {"model": ("Qwen3-8B" if args.layers == 36 else f"Qwen3-8B-{args.layers}L")
                   + ("+EAGLE3" if eagle3 else ""),
                   "global_batch": args.concurrency, "seq_len": args.input_len + args.output_len,
                   "parallelism": f"tp{world}", "cuda_graphs": not (args.eager or eagle3),
                   "workload": f"closed-loop {args.input_len} in / {args.output_len} out, concurrency {args.concurrency}, greedy"},
        "e2e": {"value": round(n / wall, 2), "unit": "tok/s"},
        "latency": latency,
        "speculative": None if not eagle3 else {k: (m.get("speculative") or {}).get(k) for k in
                                                ("steps", "acceptance_rate", "acceptance_length")}
        | {"step_latency_p50_ms": None if (m.get("speculative_step_latency") or {}).get("p50") is None
           else round(m["speculative_step_latency"]["p50"] * 1e3, 3)},
        "timing": "CUDA events on the reference's rank-0 device", "checkpoint_write_s": round(t_ckpt, 1),
        "clocks": clocks.summary() if clocks is not None else {"sm_mhz": None, "sm_max_mhz": None,
                                                              "reasons": ["unsampled"]},
    }), flush=True)
