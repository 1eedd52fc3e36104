"""Prefill/decode disaggregation: prefill on one GPU, decode on another, KV blocks pushed over NVLink.

No counterpart in the reference (it has one engine per process).  ``LLM(model,
pd_disaggregation=True, pd_prefill_devices=(a,), pd_decode_devices=(b,))`` builds a
:class:`PDEngine` with the same public API as :class:`LLMEngine`.

* Two engines share one request table: the prefill engine (``device_offset=a``) runs every
  prompt's prefill and samples its first token; the decode engine (``device_offset=b``) runs all
  decode steps (with its own CUDA graphs and overlapped decode loop).
* Handoff, right after the prefill step that produced a sequence's first token: its prefill-side
  blocks are released, decode-side blocks are allocated (prefix-cache hits in the decode pool
  are reused and not copied), and the remaining blocks -- every layer, K and V -- are copied into
  the decode pool by one ``kv_push`` kernel on the prefill GPU whose stores go straight to the
  decode GPU's memory.  An event recorded after the push orders the decode stream behind it.
  The released prefill blocks are only reused by later prefill kernels, which the prefill stream
  runs after the push.
* A sequence that finds no room in the decode pool waits (parked) until decode blocks free up;
  the prefill engine never decodes it.

With one GPU per side both engines live in this process (the same device for both sides is
allowed and runs the same protocol).  With ``tensor_parallel_size = p > 1`` each side is a
tensor-parallel group of ``p`` consecutive GPUs (``pd_prefill_devices=(0, 1, 2, 3)``,
``pd_decode_devices=(4, 5, 6, 7)``): the prefill engine's rank 0 runs here, the decode engine runs
in a child process (its own rank 0 and workers, its own process group) that this process drives
through a pipe.  Decode rank r exports its pools to prefill rank r (CUDA IPC; both hold the same
KV-head shard), and every prefill rank pushes its shard of each handed-off block with the same
kernel; the push returns once the blocks landed, before the decode side admits the sequences.

With an EAGLE3 draft the prefill engine also runs the draft's prefill, the same block ids of the
draft pools are pushed with the target's (every rank holds the whole draft pool), and the draft
K/V length (host state of the speculative executor) moves with the sequence, so the decode engine
drafts exactly as a single speculative engine would.
"""
import os
import socket
import traceback
from time import perf_counter

import torch

from llmserve_b200.engine.sequence import Sequence
from llmserve_b200.ops import kv as kv_ops


class _RunnerPair:
    """``llm.model_runner``: the sampler set on it goes to both runners; other attributes are
    the decode runner's."""

    def __init__(self, prefill_runner, decode_runner):
        object.__setattr__(self, "_pre", prefill_runner)
        object.__setattr__(self, "_dec", decode_runner)

    def __getattr__(self, name):
        return getattr(self._dec, name)

    def __setattr__(self, name, value):
        if name == "sampler":
            self._pre.sampler = value
        setattr(self._dec, name, value)


def _free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


class _DecodeServer:
    """The decode engine of a tensor-parallel disaggregated pair, in its own process."""

    def __init__(self, engine):
        self.eng = engine
        self.pending = {}

    def reserve(self, items):
        """Allocate decode blocks for handed-off sequences, in order, until the pool is full.
        Returns ``(seq_id, block_table, prefix-hit blocks)`` for each sequence that fits."""
        from llmserve_b200.engine.sequence import Sequence
        from llmserve_b200.sampling_params import SamplingParams
        bm = self.eng.scheduler.block_manager
        out = []
        for seq_id, token_ids, n_prompt, max_tokens, ignore_eos, temperature in items:
            seq = Sequence(list(token_ids), SamplingParams(temperature=temperature, max_tokens=max_tokens,
                                                           ignore_eos=ignore_eos))
            seq.seq_id, seq.num_prompt_tokens = seq_id, n_prompt
            if not bm.can_allocate(seq):
                break
            bm.allocate(seq)
            hits = seq.num_cached_tokens // bm.block_size
            seq.num_cached_tokens = seq.num_tokens
            self.pending[seq_id] = seq
            out.append((seq_id, list(seq.block_table), hits))
        return out

    def admit(self, seq_ids, draft_lengths=None):
        from llmserve_b200.engine.sequence import SequenceStatus
        if draft_lengths:
            self.eng.model_runner.call("set_draft_lengths", draft_lengths)     # every decode rank
        for sid in seq_ids:
            s = self.pending.pop(sid)
            s.status = SequenceStatus.RUNNING
            self.eng.request_metrics[sid] = self.eng.new_request_metric(sid, s.num_prompt_tokens)
            self.eng.scheduler.running.append(s)

    def step(self):
        """One decode step: finished sequences, sequences that emitted, tokens, and the speculative
        counters of the finished sequences' records (the parent keeps the request table)."""
        if self.eng.is_finished():
            return [], [], 0, {}
        done, n = self.eng.step()
        spec = {}
        for sid, _ in done:
            m = self.eng.request_metrics.pop(sid, None) or {}
            spec[sid] = {k: v for k, v in m.items() if k.startswith("speculative_")}
        return done, list(self.eng.last_step_events.get("decode_seq_ids", [])), n, spec

    def set_sampler(self, sampler):
        self.eng.model_runner.sampler = sampler

    def kv_metrics(self):
        return self.eng.scheduler.kv_capacity_metrics()


def _decode_server_main(model, kwargs, conn):
    from llmserve_b200.engine.llm_engine import LLMEngine
    try:
        eng = LLMEngine(model, **kwargs)
        conn.send(("ok", (eng.model_runner.call("export_kv"), eng.config.num_kvcache_blocks)))
    except Exception as e:  # reported to the parent, which raises
        conn.send(("error", f"{type(e).__name__}: {e}\n{traceback.format_exc()}"))
        return
    server = _DecodeServer(eng)
    while True:
        try:
            cmd, args = conn.recv()
        except EOFError:             # the parent is gone
            eng.exit()
            return
        if cmd == "exit":
            eng.exit()
            conn.send(("ok", None))
            return
        try:
            conn.send(("ok", getattr(server, cmd)(*args)))
        except Exception as e:
            conn.send(("error", f"{type(e).__name__}: {e}\n{traceback.format_exc()}"))


class _RemoteDecode:
    """Parent side of the decode server: synchronous calls with a bounded wait."""

    def __init__(self, model, kwargs, timeout_s: float):
        import torch.multiprocessing as mp
        ctx = mp.get_context("spawn")
        self.conn, child = ctx.Pipe()
        self.proc = ctx.Process(target=_decode_server_main, args=(model, kwargs, child), daemon=False)
        self.proc.start()
        self.timeout_s = timeout_s
        self.ready = self._reply(max(timeout_s, 600.0))

    def _reply(self, timeout_s):
        if not self.conn.poll(timeout_s):
            raise TimeoutError(f"decode server did not answer within {timeout_s:.0f}s")
        status, value = self.conn.recv()
        if status != "ok":
            raise RuntimeError(f"decode server failed: {value}")
        return value

    def call(self, cmd, *args):
        if not self.proc.is_alive():
            raise RuntimeError("decode server exited")
        self.conn.send((cmd, args))
        return self._reply(self.timeout_s)

    def close(self):
        try:
            if self.proc.is_alive():
                self.call("exit")
        finally:
            self.proc.join(timeout=self.timeout_s)
            if self.proc.is_alive():
                self.proc.terminate()


class _RemoteRunnerPair:
    """``llm.model_runner`` of the tensor-parallel pair: the sampler goes to both sides."""

    def __init__(self, prefill_runner, remote):
        object.__setattr__(self, "_pre", prefill_runner)
        object.__setattr__(self, "_remote", remote)

    def __getattr__(self, name):
        return getattr(self._pre, name)

    def __setattr__(self, name, value):
        if name == "sampler":
            self._remote.call("set_sampler", value)
        setattr(self._pre, name, value)


class PDEngine:

    def __init__(self, model, **kwargs):
        from llmserve_b200.engine.llm_engine import LLMEngine
        pre = tuple(kwargs.pop("pd_prefill_devices", ()) or ())
        dec = tuple(kwargs.pop("pd_decode_devices", ()) or ())
        kwargs.pop("pd_disaggregation", None)
        kwargs.pop("device_offset", None)
        kwargs.pop("overlap_decode", None)
        kwargs.pop("pd_role", None)
        tp = kwargs.get("tensor_parallel_size", 1)
        if len(pre) != tp or len(dec) != tp:
            raise ValueError("pd_disaggregation needs tensor_parallel_size devices on each side")
        self.pd_stats = {"handoffs": 0, "blocks_pushed": 0, "blocks_reused": 0, "bytes_pushed": 0,
                         "parked_steps": 0}
        self._parked: list[Sequence] = []
        self.last_step_events: dict = {}
        self.remote = None
        if tp > 1:
            self._init_tensor_parallel(model, kwargs, pre, dec)
            return
        self.prefill = LLMEngine(model, **kwargs, device_offset=pre[0], overlap_decode=False)
        self.decode = LLMEngine(model, **kwargs, device_offset=dec[0])
        self.decode.request_metrics = self.prefill.request_metrics
        self.config = self.prefill.config
        self.tokenizer = self.prefill.tokenizer
        self.model_runner = _RunnerPair(self.prefill.model_runner, self.decode.model_runner)
        self.request_metrics = self.prefill.request_metrics
        pr, dr = self.prefill.model_runner, self.decode.model_runner
        self._cuda = pr.is_cuda
        if pr.k_cache.shape[0] != dr.k_cache.shape[0] or pr.k_cache.shape[2:] != dr.k_cache.shape[2:]:
            raise ValueError("prefill and decode KV pools have different block shapes")

    def _init_tensor_parallel(self, model, kwargs, pre, dec):
        from llmserve_b200.engine.llm_engine import LLMEngine
        p = len(pre)
        if pre != tuple(range(pre[0], pre[0] + p)) or dec != tuple(range(dec[0], dec[0] + p)):
            raise ValueError("each side of a tensor-parallel pair takes consecutive GPUs")
        timeout = float(kwargs.get("comm_timeout_s", 120.0))
        tag = f"{os.getpid()}_{id(self)}"
        dkw = dict(kwargs, device_offset=dec[0], pd_role="decode", rpc_channel=f"llmserve_b200_pdd_{tag}",
                   distributed_init_method=f"tcp://127.0.0.1:{_free_port()}")
        self.remote = _RemoteDecode(model, dkw, timeout)
        descs, self.decode_blocks = self.remote.ready
        try:
            self.prefill = LLMEngine(model, **dict(kwargs, rpc_channel=f"llmserve_b200_pdp_{tag}",
                                                   distributed_init_method=f"tcp://127.0.0.1:{_free_port()}"),
                                     device_offset=pre[0], overlap_decode=False)
            self.prefill.model_runner.call("open_peer_kv", descs)
        except Exception:
            self.remote.close()
            raise
        self.decode = None
        self.config = self.prefill.config
        self.tokenizer = self.prefill.tokenizer
        self.request_metrics = self.prefill.request_metrics
        self.model_runner = _RemoteRunnerPair(self.prefill.model_runner, self.remote)
        self._remote_seqs: dict = {}
        self._cuda = self.prefill.model_runner.is_cuda

    # ---- API --------------------------------------------------------------------------------
    def add_request(self, prompt, sampling_params) -> int:
        return self.prefill.add_request(prompt, sampling_params)

    def is_finished(self) -> bool:
        if self.remote is not None:
            return self.prefill.is_finished() and not self._parked and not self._remote_seqs
        return self.prefill.is_finished() and self.decode.is_finished() and not self._parked

    def _on(self, engine):
        dev = engine.model_runner.device
        return torch.cuda.device(dev) if dev.type == "cuda" else _Null()

    def step(self):
        t0 = perf_counter()
        outputs, tokens = [], 0
        if not self.prefill.is_finished():
            with self._on(self.prefill):
                done, n = self.prefill.step()
            outputs += done
            tokens += n
            self._park_new_first_tokens()
        if self.remote is not None:
            return self._remote_step(t0, outputs, tokens)
        self._handoff()
        if not self.decode.is_finished():
            with self._on(self.decode):
                done, n = self.decode.step()
            outputs += done
            tokens += n
        self.last_step_events = {"step_start": t0, "step_end": perf_counter(), "num_tokens": tokens,
                                 "prefill": self.prefill.last_step_events, "decode": self.decode.last_step_events,
                                 "parked": len(self._parked)}
        return outputs, tokens

    def generate(self, prompts, sampling_params, use_tqdm: bool = True):
        from tqdm.auto import tqdm
        bar = tqdm(total=len(prompts), desc="Generating", dynamic_ncols=True, disable=not use_tqdm)
        if not isinstance(sampling_params, list):
            sampling_params = [sampling_params] * len(prompts)
        for p, sp in zip(prompts, sampling_params):
            self.add_request(p, sp)
        done = {}
        while not self.is_finished():
            t = perf_counter()
            out, n = self.step()
            bar.set_postfix({"tok/s": f"{int(n / max(perf_counter() - t, 1e-9))}"})
            for sid, toks in out:
                done[sid] = toks
                bar.update(1)
        bar.close()
        return [{"text": self.tokenizer.decode(done[k]), "token_ids": done[k]} for k in sorted(done)]

    def get_metrics(self) -> dict:
        if self.remote is not None:
            m = self.prefill.get_metrics()
            m["summary"]["kv_cache_prefill"] = m["summary"]["kv_cache"]
            m["summary"]["kv_cache"] = self.remote.call("kv_metrics")
        else:
            m = self.decode.get_metrics()
            m["summary"]["kv_cache_prefill"] = self.prefill.get_metrics()["summary"]["kv_cache"]
        m["summary"]["pd"] = dict(self.pd_stats, parked=len(self._parked))
        return m

    def reset_metrics(self):
        self.prefill.reset_metrics()
        if self.decode is not None:
            self.decode.reset_metrics()
        self.pd_stats = dict.fromkeys(self.pd_stats, 0)

    def exit(self):
        if self.remote is not None:
            try:
                self.remote.close()
            finally:
                self.prefill.exit()
            return
        self.decode.exit()
        self.prefill.exit()

    # ---- tensor-parallel pair ---------------------------------------------------------------
    def _remote_step(self, t0, outputs, tokens):
        self._remote_handoff()
        if self._remote_seqs:
            done, emitted, n, spec = self.remote.call("step")
            t = perf_counter()
            tokens += n
            for sid in emitted:
                m = self.request_metrics.get(sid)
                if m is not None:
                    m["token_times"].append(t)
                    m["output_event_times"].append(t)
                    m["output_tokens"] += 1
            for sid, toks in done:
                m = self.request_metrics.get(sid)
                if m is not None:
                    m["finish_time"], m["success"], m["output_tokens"] = t, True, len(toks)
                    m.update(spec.get(sid, {}))
                self._remote_seqs.pop(sid, None)
                outputs.append((sid, toks))
        self.last_step_events = {"step_start": t0, "step_end": perf_counter(), "num_tokens": tokens,
                                 "prefill": self.prefill.last_step_events, "parked": len(self._parked),
                                 "decoding": len(self._remote_seqs)}
        return outputs, tokens

    def _remote_handoff(self):
        if not self._parked:
            return
        items = [(s.seq_id, list(s.token_ids), s.num_prompt_tokens, s.max_tokens, s.ignore_eos, s.temperature)
                 for s in self._parked]
        reserved = self.remote.call("reserve", items)
        if not reserved:
            self.pd_stats["parked_steps"] += 1
            return
        pre_r = self.prefill.model_runner
        bs = self.prefill.scheduler.block_manager.block_size
        src, dst, moved = [], [], []
        for (sid, table, hits), s in zip(reserved, list(self._parked)):
            n_kv_blocks = -(-(len(s) - 1) // bs)
            src += s.block_table[hits:n_kv_blocks]
            dst += table[hits:n_kv_blocks]
            self.pd_stats["blocks_reused"] += min(hits, n_kv_blocks)
            moved.append(s)
        if src:
            pre_r.call("push_kv", src, dst)          # every prefill rank pushes its KV-head shard
            if pre_r.channel is not None:
                pre_r.channel.wait_acks(self.remote.timeout_s)
        bm = self.prefill.scheduler.block_manager
        for s in moved:
            bm.deallocate(s)                          # after every rank's copy landed
            self._parked.remove(s)
            self._remote_seqs[s.seq_id] = s
        ids = [s.seq_id for s in moved]
        lengths = None
        if pre_r.draft_model is not None:
            lengths = {sid: pre_r.spec.draft_kv_len[sid] for sid in ids if sid in pre_r.spec.draft_kv_len}
            pre_r.call("clear_speculative_state", ids)                        # every prefill rank
        self.remote.call("admit", ids, lengths)
        per_block = 2 * pre_r.k_cache[:, 0].numel() * pre_r.k_cache.element_size() * pre_r.world_size
        if pre_r.draft_model is not None:
            per_block += 2 * pre_r.draft_k_cache[0].numel() * pre_r.draft_k_cache.element_size() * pre_r.world_size
        self.pd_stats["handoffs"] += len(moved)
        self.pd_stats["blocks_pushed"] += len(src)
        self.pd_stats["bytes_pushed"] += len(src) * per_block

    # ---- handoff ----------------------------------------------------------------------------
    def _park_new_first_tokens(self):
        """Move every sequence whose prefill emitted its first token out of the prefill scheduler."""
        sched = self.prefill.scheduler
        ready = [s for s in sched.running if s.num_completion_tokens >= 1 and not s.is_finished]
        for s in ready:
            sched.running.remove(s)
            sched._release_reservation(s)
            self._parked.append(s)

    def _handoff(self):
        if not self._parked:
            return
        pre_r, dec_r = self.prefill.model_runner, self.decode.model_runner
        pre_bm, dec_bm = self.prefill.scheduler.block_manager, self.decode.scheduler.block_manager
        bs = pre_bm.block_size
        src, dst, moved = [], [], []
        for s in list(self._parked):
            if not dec_bm.can_allocate(s):
                break                                    # FIFO: wait for decode blocks
            n_kv_blocks = -(-(len(s) - 1) // bs)         # blocks holding computed KV
            old_table = list(s.block_table)
            pre_bm.deallocate(s)
            dec_bm.allocate(s)                           # seals full blocks; counts prefix hits
            hits = s.num_cached_tokens // bs
            for i in range(hits, n_kv_blocks):
                src.append(old_table[i])
                dst.append(s.block_table[i])
            self.pd_stats["blocks_reused"] += min(hits, n_kv_blocks)
            s.num_cached_tokens = s.num_tokens
            self._parked.remove(s)
            moved.append(s)
        if not moved:
            self.pd_stats["parked_steps"] += 1
            return
        draft = pre_r.draft_model is not None
        if draft:
            # the draft's prompt K/V lives in the same block ids of the draft pools; the length of
            # the draft K/V (host state of the speculative executor) moves with the sequence
            for s in moved:
                n = pre_r.spec.draft_kv_len.pop(s.seq_id, None)
                if n is not None:
                    dec_r.spec.draft_kv_len[s.seq_id] = n
                pre_r.spec.prev_correction.pop(s.seq_id, None)
        if src:
            with self._on(self.prefill):
                kv_ops.push_blocks(pre_r.k_cache, pre_r.v_cache, dec_r.k_cache, dec_r.v_cache, src, dst)
                if draft:
                    kv_ops.push_blocks(pre_r.draft_k_cache.unsqueeze(0), pre_r.draft_v_cache.unsqueeze(0),
                                       dec_r.draft_k_cache.unsqueeze(0), dec_r.draft_v_cache.unsqueeze(0), src, dst)
                if self._cuda:
                    ev = torch.cuda.Event()
                    ev.record()
            if self._cuda:
                with self._on(self.decode):
                    torch.cuda.current_stream().wait_event(ev)
        per_block = 2 * pre_r.k_cache[:, 0].numel() * pre_r.k_cache.element_size()
        if draft:
            per_block += 2 * pre_r.draft_k_cache[0].numel() * pre_r.draft_k_cache.element_size()
        self.pd_stats["handoffs"] += len(moved)
        self.pd_stats["blocks_pushed"] += len(src)
        self.pd_stats["bytes_pushed"] += len(src) * per_block
        self.decode.scheduler.running.extend(moved)


class _Null:
    def __enter__(self):
        return self

    def __exit__(self, *exc):
        return False
