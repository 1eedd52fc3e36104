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

Scope: one GPU per side (``tensor_parallel_size=1``), no speculative draft; both engines live in
this process (the same device for both sides is allowed and runs the same protocol).
"""
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


class PDEngine:

    def __init__(self, model, **kwargs):
        from llmserve_b200.engine.llm_engine import LLMEngine
        pre = tuple(kwargs.pop("pd_prefill_devices", ()) or ())
        dec = tuple(kwargs.pop("pd_decode_devices", ()) or ())
        kwargs.pop("pd_disaggregation", None)
        kwargs.pop("device_offset", None)
        kwargs.pop("overlap_decode", None)
        if len(pre) != 1 or len(dec) != 1:
            raise ValueError("pd_disaggregation takes one prefill device and one decode device")
        if kwargs.get("tensor_parallel_size", 1) != 1:
            raise ValueError("pd_disaggregation runs each side on one GPU (tensor_parallel_size=1)")
        if kwargs.get("speculative_model"):
            raise ValueError("pd_disaggregation does not support a speculative draft model")
        self.prefill = LLMEngine(model, **kwargs, device_offset=pre[0], overlap_decode=False)
        self.decode = LLMEngine(model, **kwargs, device_offset=dec[0])
        self.decode.request_metrics = self.prefill.request_metrics
        self.config = self.prefill.config
        self.tokenizer = self.prefill.tokenizer
        self.model_runner = _RunnerPair(self.prefill.model_runner, self.decode.model_runner)
        self.request_metrics = self.prefill.request_metrics
        self.last_step_events: dict = {}
        self._parked: list[Sequence] = []
        self.pd_stats = {"handoffs": 0, "blocks_pushed": 0, "blocks_reused": 0, "bytes_pushed": 0,
                         "parked_steps": 0}
        pr, dr = self.prefill.model_runner, self.decode.model_runner
        self._cuda = pr.is_cuda
        if pr.k_cache.shape[0] != dr.k_cache.shape[0] or pr.k_cache.shape[2:] != dr.k_cache.shape[2:]:
            raise ValueError("prefill and decode KV pools have different block shapes")

    # ---- API --------------------------------------------------------------------------------
    def add_request(self, prompt, sampling_params) -> int:
        return self.prefill.add_request(prompt, sampling_params)

    def is_finished(self) -> bool:
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

    def generate(self, prompts, sampling_params, use_tqdm: bool = False):
        if not isinstance(sampling_params, list):
            sampling_params = [sampling_params] * len(prompts)
        for p, sp in zip(prompts, sampling_params):
            self.add_request(p, sp)
        done = {}
        while not self.is_finished():
            out, _ = self.step()
            for sid, toks in out:
                done[sid] = toks
        return [{"text": self.tokenizer.decode(done[k]), "token_ids": done[k]} for k in sorted(done)]

    def get_metrics(self) -> dict:
        m = self.decode.get_metrics()
        m["summary"]["kv_cache_prefill"] = self.prefill.get_metrics()["summary"]["kv_cache"]
        m["summary"]["pd"] = dict(self.pd_stats, parked=len(self._parked))
        return m

    def reset_metrics(self):
        self.prefill.reset_metrics()
        self.decode.reset_metrics()
        self.pd_stats = dict.fromkeys(self.pd_stats, 0)

    def exit(self):
        self.decode.exit()
        self.prefill.exit()

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
        if src:
            with self._on(self.prefill):
                kv_ops.push_blocks(pre_r.k_cache, pre_r.v_cache, dec_r.k_cache, dec_r.v_cache, src, dst)
                if self._cuda:
                    ev = torch.cuda.Event()
                    ev.record()
            if self._cuda:
                with self._on(self.decode):
                    torch.cuda.current_stream().wait_event(ev)
        per_block = 2 * pre_r.k_cache[:, 0].numel() * pre_r.k_cache.element_size()
        self.pd_stats["handoffs"] += len(moved)
        self.pd_stats["blocks_pushed"] += len(src)
        self.pd_stats["bytes_pushed"] += len(src) * per_block
        self.decode.scheduler.running.extend(moved)


class _Null:
    def __enter__(self):
        return self

    def __exit__(self, *exc):
        return False
