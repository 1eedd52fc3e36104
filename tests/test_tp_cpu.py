"""Tensor parallelism over gloo CPU ranks, and failure handling of the host control plane.

Failures are injected on the host only (no GPU): a worker whose call raises must surface as an
exception on rank 0 instead of a hang; a worker whose rank 0 disappeared must exit on its own;
RPC waits are bounded.
"""
import os
import socket
import time

import pytest
import torch
import torch.multiprocessing as mp

from llmserve_b200 import LLM, SamplingParams
from llmserve_b200.engine.model_runner import GreedySampler
from llmserve_b200.engine.rpc import RpcChannel, RpcTimeout
from llmserve_b200.models.synthetic import TINY, write_eagle3_checkpoint, write_qwen3_checkpoint


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


@pytest.fixture(scope="module")
def ckpts(tmp_path_factory):
    d = tmp_path_factory.mktemp("tp")
    return (write_qwen3_checkpoint(str(d / "t"), TINY, seed=1),
            write_eagle3_checkpoint(str(d / "d"), TINY, draft_vocab=512, seed=1))


def _gen(path, tp, draft=None, **kw):
    llm = LLM(path, device="cpu", enforce_eager=True, num_kvcache_blocks=64, kvcache_block_size=16, max_model_len=256,
              tensor_parallel_size=tp, speculative_model=draft, comm_timeout_s=60,
              distributed_init_method=f"tcp://127.0.0.1:{_port()}", **kw)
    llm.model_runner.sampler = GreedySampler()
    g = torch.Generator().manual_seed(11)
    prompts = [torch.randint(0, 1024, (int(n),), generator=g).tolist() for n in (9, 33, 17, 50)]
    out = [o["token_ids"] for o in llm.generate(prompts, SamplingParams(max_tokens=12, ignore_eos=True), use_tqdm=False)]
    llm.exit()
    return out


def test_tp2_gloo_matches_tp1_with_and_without_speculation(ckpts):
    tgt, draft = ckpts
    ref = _gen(tgt, 1)
    assert _gen(tgt, 2) == ref
    assert _gen(tgt, 2, draft) == ref
    assert _gen(tgt, 2, draft, speculative_cuda_graphs=True) == ref      # graph step layout, every rank


@pytest.mark.parametrize("speculative", [False, True])
def test_disaggregated_tp2_prefill_tp2_decode_over_gloo(ckpts, speculative):
    """Prefill TP=2 (this process + a worker) and decode TP=2 (a server process + its worker), KV
    blocks pushed rank to rank into the decode pools (shared segments on the CPU tier): the tokens
    equal a single TP=1 engine's.  With an EAGLE3 draft the draft pools and lengths move too: the
    decode side drafts the same tokens, step by step, as a single TP=2 speculative engine."""
    tgt, draft = ckpts
    ref = _gen(tgt, 1)
    g = torch.Generator().manual_seed(11)
    prompts = [torch.randint(0, 1024, (int(n),), generator=g).tolist() for n in (9, 33, 17, 50)]
    kw = dict(device="cpu", enforce_eager=True, num_kvcache_blocks=64, kvcache_block_size=16, max_model_len=256,
              tensor_parallel_size=2, comm_timeout_s=60)
    if speculative:
        kw.update(speculative_model=draft, speculative_trace=True)
    runs = []
    for pd in ((True, False) if speculative else (True,)):
        extra = dict(pd_disaggregation=True, pd_prefill_devices=(0, 1), pd_decode_devices=(2, 3)) if pd else \
            dict(distributed_init_method=f"tcp://127.0.0.1:{_port()}")
        llm = LLM(tgt, **kw, **extra)
        try:
            llm.model_runner.sampler = GreedySampler()
            out = [o["token_ids"] for o in llm.generate(prompts, SamplingParams(max_tokens=12, ignore_eos=True),
                                                        use_tqdm=False)]
            met = llm.get_metrics()
        finally:
            llm.exit()
        runs.append((out, met))
    out, met = runs[0]
    m = met["summary"]
    assert out == ref
    assert m["pd"]["handoffs"] == 4 and m["pd"]["blocks_pushed"] > 0 and m["num_finished"] == 4
    assert m["total_output_tokens"] == 48
    if speculative:
        def drafts(metrics):
            return [[e["draft_token_ids"] for e in r["speculative_trace"]] for r in metrics["requests"]]
        assert m["speculative"]["steps"] > 0
        assert drafts(met) == drafts(runs[1][1]) and any(drafts(met))


def test_tp2_gloo_temperature_sampling_is_rank_consistent(ckpts):
    tgt, _ = ckpts
    llm = LLM(tgt, device="cpu", enforce_eager=True, num_kvcache_blocks=64, kvcache_block_size=16, max_model_len=256,
              tensor_parallel_size=2, distributed_init_method=f"tcp://127.0.0.1:{_port()}")
    out = llm.generate([[3, 4, 5]] * 3, SamplingParams(temperature=1.0, max_tokens=8, ignore_eos=True), use_tqdm=False)
    llm.exit()     # would hang or raise if ranks had diverged (their collectives would mismatch)
    assert all(len(o["token_ids"]) == 8 for o in out)


def _raising_worker(name):
    ch = RpcChannel(name, 1, create=False)
    method, args = ch.recv(0, idle_timeout_s=1.0, parent_pid=os.getppid())
    ch.ack(0, False, f"ValueError: injected failure in {method}")
    ch.close()


def test_worker_exception_surfaces_on_rank0():
    name = f"lsb_test_{os.getpid()}_a"
    ch = RpcChannel(name, 1, create=True)
    p = mp.get_context("spawn").Process(target=_raising_worker, args=(name,))
    p.start()
    ch.send("run", 1, 2)
    with pytest.raises(RuntimeError, match="injected failure"):
        ch.wait_acks(30)
    p.join(10)
    ch.close()


def _orphan_worker(name, q):
    ch = RpcChannel(name, 1, create=False)
    t = time.monotonic()
    try:
        ch.recv(0, idle_timeout_s=0.2, parent_pid=999999999)   # a pid that does not exist
    except RpcTimeout:
        q.put(time.monotonic() - t)
    ch.close()


def test_orphaned_worker_exits_on_its_own():
    name = f"lsb_test_{os.getpid()}_b"
    ch = RpcChannel(name, 1, create=True)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    p = ctx.Process(target=_orphan_worker, args=(name, q))
    p.start()
    waited = q.get(timeout=30)
    p.join(10)
    ch.close()
    assert waited < 5 and p.exitcode == 0


def _counting_worker(name, n, q):
    ch = RpcChannel(name, 1, create=False)
    seen = []
    for _ in range(n):
        method, args = ch.recv(0, idle_timeout_s=5.0, parent_pid=os.getppid())
        seen.append(args[0])
        if args[0] % 7 == 0:
            time.sleep(0.003)        # a slow call: the next send must wait for it
        ch.ack(0, True)
    q.put(seen)
    ch.close()


def test_back_to_back_calls_are_never_skipped():
    """Calls that rank 0 publishes without waiting in between (the overlapped decode launches, the
    sampler mirror) all reach the worker, in order."""
    name = f"lsb_test_{os.getpid()}_d"
    ch = RpcChannel(name, 1, create=True, ack_timeout_s=30)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    p = ctx.Process(target=_counting_worker, args=(name, 60, q))
    p.start()
    for i in range(60):
        ch.send("call", i)
    assert q.get(timeout=60) == list(range(60))
    p.join(10)
    ch.close()


def test_ack_wait_is_bounded():
    ch = RpcChannel(f"lsb_test_{os.getpid()}_c", 1, create=True)
    ch.send("noop")
    t = time.monotonic()
    with pytest.raises(RpcTimeout):
        ch.wait_acks(0.3)
    assert time.monotonic() - t < 3
    ch.close()


def _rank_main(rank, world, port, fail_rank, q):
    import torch.distributed as dist
    from datetime import timedelta
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=timedelta(seconds=3))
    t = torch.ones(4)
    dist.all_reduce(t)
    if rank == fail_rank:
        q.put((rank, "left"))
        return                        # leaves between steps, with nothing in flight
    t0 = time.monotonic()
    try:
        dist.all_reduce(t)
        q.put((rank, "no-error"))
    except Exception:
        q.put((rank, f"error after {time.monotonic() - t0:.1f}s"))


def test_process_group_timeout_ends_collective_after_rank_loss():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    ps = [ctx.Process(target=_rank_main, args=(r, 2, port, 1, q)) for r in range(2)]
    for p in ps:
        p.start()
    res = dict(q.get(timeout=60) for _ in range(2))
    for p in ps:
        p.join(30)
    assert res[1] == "left"
    assert res[0].startswith("error")


def test_disaggregated_decode_server_loss_surfaces_as_an_error(ckpts):
    """Host fault injection: the decode side of a tensor-parallel disaggregated pair dies between
    steps (its server process is killed); the next step raises a clear error instead of hanging,
    and the decode server's own worker exits on its own (orphan check)."""
    tgt, _ = ckpts
    llm = LLM(tgt, device="cpu", enforce_eager=True, num_kvcache_blocks=64, kvcache_block_size=16, max_model_len=256,
              tensor_parallel_size=2, comm_timeout_s=20, pd_disaggregation=True, pd_prefill_devices=(0, 1),
              pd_decode_devices=(2, 3))
    try:
        llm.model_runner.sampler = GreedySampler()
        llm.add_request(list(range(5, 30)), SamplingParams(max_tokens=8, ignore_eos=True))
        llm.step()                                # prefill + handoff + first decode step
        import psutil
        workers = psutil.Process(llm.remote.proc.pid).children(recursive=True)
        llm.remote.proc.kill()                    # the server process this engine started
        llm.remote.proc.join(timeout=30)
        t0 = time.monotonic()
        with pytest.raises((RuntimeError, TimeoutError, EOFError, BrokenPipeError, ConnectionError)):
            while not llm.is_finished():
                llm.step()
        assert time.monotonic() - t0 < 60
        # the server's tensor-parallel worker notices its parent is gone and leaves by itself
        _, alive = psutil.wait_procs(workers, timeout=60)
        assert not alive, [w.pid for w in alive]
    finally:
        try:
            llm.prefill.exit()
        except Exception:
            pass


def test_awq_engine_on_the_host_matches_dequantized_dense_and_shards_over_gloo(tmp_path, ckpts):
    """AutoAWQ GEMM g128 checkpoint on the fp32 host path: the same tokens as a dense checkpoint
    holding the dequantised weights, and TP=2 (packed qweight/qzeros/scales sliced per rank, with
    and without an EAGLE3 draft) equal to TP=1."""
    import json

    from safetensors import safe_open
    from safetensors.torch import save_file

    from llmserve_b200.models.synthetic import write_awq_checkpoint
    from llmserve_b200.quantization.awq import dequantize_awq_gemm
    awq = write_awq_checkpoint(str(tmp_path / "awq"), TINY, seed=3)
    dense_dir = tmp_path / "dense"
    dense_dir.mkdir()
    cfg = json.load(open(os.path.join(awq, "config.json")))
    cfg.pop("quantization_config")
    cfg["torch_dtype"] = "float32"
    json.dump(cfg, open(dense_dir / "config.json", "w"))
    tensors = {}
    with safe_open(os.path.join(awq, "model.safetensors"), "pt") as f:
        for name in f.keys():
            if name.endswith(".qweight"):
                base = name[: -len(".qweight")]
                w = dequantize_awq_gemm(f.get_tensor(name), f.get_tensor(base + ".qzeros"),
                                        f.get_tensor(base + ".scales").float(), group_size=128)
                tensors[base + ".weight"] = w.t().contiguous()
            elif not name.endswith((".qzeros", ".scales")):
                tensors[name] = f.get_tensor(name).float()
    save_file(tensors, str(dense_dir / "model.safetensors"))
    ref = _gen(str(dense_dir), 1)
    assert _gen(awq, 1) == ref
    assert _gen(awq, 2) == ref
    assert _gen(awq, 2, ckpts[1]) == ref          # with an EAGLE3 draft, tensor parallel


@pytest.mark.parametrize("tp", [4, 8])
def test_tp4_and_tp8_gloo_match_tp1(tmp_path, tp):
    """The host side of TP = 4 / 8 (head, KV-head, MLP and vocab shards -- one KV head per rank at
    TP = 8 --, seven RPC workers, the vocab-parallel argmax, an EAGLE3 draft on every rank) on gloo
    CPU ranks: tokens equal TP = 1."""
    cfg = dict(TINY, num_attention_heads=16, num_key_value_heads=8, head_dim=16)
    path = write_qwen3_checkpoint(str(tmp_path / "t"), cfg, seed=3)
    draft = write_eagle3_checkpoint(str(tmp_path / "d"), cfg, draft_vocab=512, seed=3)
    ref = _gen(path, 1)
    assert _gen(path, tp) == ref
    assert _gen(path, tp, draft) == ref          # EAGLE3 chain speculation on every rank


def test_disaggregated_tp4_prefill_tp4_decode_over_gloo(tmp_path):
    """The disaggregated shape the benchmark asks for -- prefill TP = 4 on devices 0-3, decode TP = 4
    on devices 4-7, each rank pushing its KV-head shard to its decode peer -- on gloo CPU ranks:
    tokens equal a single TP = 1 engine's."""
    cfg = dict(TINY, num_attention_heads=16, num_key_value_heads=8, head_dim=16)
    path = write_qwen3_checkpoint(str(tmp_path / "t"), cfg, seed=5)
    ref = _gen(path, 1)
    g = torch.Generator().manual_seed(11)
    prompts = [torch.randint(0, 1024, (int(n),), generator=g).tolist() for n in (9, 33, 17, 50)]
    llm = LLM(path, device="cpu", enforce_eager=True, num_kvcache_blocks=64, kvcache_block_size=16, max_model_len=256,
              tensor_parallel_size=4, comm_timeout_s=60, pd_disaggregation=True, pd_prefill_devices=(0, 1, 2, 3),
              pd_decode_devices=(4, 5, 6, 7))
    try:
        llm.model_runner.sampler = GreedySampler()
        out = [o["token_ids"] for o in llm.generate(prompts, SamplingParams(max_tokens=12, ignore_eos=True),
                                                    use_tqdm=False)]
        m = llm.get_metrics()["summary"]
    finally:
        llm.exit()
    assert out == ref
    assert m["pd"]["handoffs"] == 4 and m["pd"]["blocks_pushed"] > 0
