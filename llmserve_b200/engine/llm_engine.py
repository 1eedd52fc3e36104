"""Engine: request intake, step loop, per-request timing and metrics.

API and metric semantics follow ``llmserve/engine/llm_engine.py`` of the reference:
``add_request`` / ``step`` / ``is_finished`` / ``get_metrics`` / ``reset_metrics`` / ``exit`` /
``generate``; ``last_step_events`` per step; a request's token times are the end of the step that
emitted them (several identical stamps for a speculative step -> 0 ms burst ITL samples),
``output_event_times`` once per emitting step, and the ``get_metrics`` summary/requests layout
(``:370-554``).  A speculative step runs whenever the batch is pure decode and the draft is loaded;
unlike the reference it is not restricted to eager mode or to one GPU.
"""
import atexit
import itertools
import os
from dataclasses import fields
from time import perf_counter

import numpy as np
import torch.multiprocessing as mp
from tqdm.auto import tqdm

from llmserve_b200.config import Config
from llmserve_b200.engine.model_runner import ModelRunner
from llmserve_b200.engine.scheduler import Scheduler
from llmserve_b200.engine.sequence import Sequence
from llmserve_b200.sampling_params import SamplingParams
from llmserve_b200.utils.nvtx import nvtx_range
from llmserve_b200.utils.tokenizer import load_tokenizer

_engine_ids = itertools.count()


def _worker_main(config, rank, channel_name, parent_pid):
    ModelRunner(config, rank, channel_name, parent_pid)


def run_worker(model, rank: int, **kwargs):
    """Tensor-parallel worker body for ranks started by an external launcher (torchrun).

    Rank 0 builds ``LLM(model, distributed_launcher="external", ...)`` with the same kwargs; this
    call returns when rank 0 calls ``exit()``."""
    names = {f.name for f in fields(Config)}
    config = Config(model, **{k: v for k, v in kwargs.items() if k in names})
    Sequence.block_size = config.kvcache_block_size
    ModelRunner(config, rank, config.rpc_channel or "llmserve_b200_ext", os.getppid())


def percentile(values, q):
    """Linear-interpolation percentile (the reference's ``_percentile``)."""
    if not values:
        return None
    v = sorted(values)
    if len(v) == 1:
        return v[0]
    rank = (len(v) - 1) * q / 100
    lo = int(rank)
    hi = min(lo + 1, len(v) - 1)
    w = rank - lo
    return v[lo] * (1 - w) + v[hi] * w


def summarize(values):
    if not values:
        return {"mean": None, "p50": None, "p99": None, "max": None}
    return {"mean": sum(values) / len(values), "p50": percentile(values, 50), "p99": percentile(values, 99),
            "max": max(values)}


def _diffs(times):
    return [b - a for a, b in zip(times, times[1:])]


class LLMEngine:

    def __new__(cls, model=None, **kwargs):
        if kwargs.get("pd_disaggregation"):
            from llmserve_b200.engine.pd_engine import PDEngine
            return PDEngine(model, **kwargs)
        return super().__new__(cls)

    def __init__(self, model, **kwargs):
        names = {f.name for f in fields(Config)}
        config = Config(model, **{k: v for k, v in kwargs.items() if k in names})
        self.config = config
        Sequence.block_size = config.kvcache_block_size
        self.ps = []
        channel = config.rpc_channel or f"llmserve_b200_{os.getpid()}_{next(_engine_ids)}"
        if config.distributed_launcher == "external":
            channel = config.rpc_channel or "llmserve_b200_ext"
        elif config.tensor_parallel_size > 1:
            ctx = mp.get_context("spawn")
            for rank in range(1, config.tensor_parallel_size):
                p = ctx.Process(target=_worker_main, args=(config, rank, channel, os.getpid()), daemon=True)
                p.start()
                self.ps.append(p)
        self.model_runner = ModelRunner(config, 0, channel)
        self.tokenizer = load_tokenizer(config.model, config.hf_config)
        eos = getattr(self.tokenizer, "eos_token_id", -1)
        config.eos = -1 if eos is None else eos
        self.scheduler = Scheduler(config)
        self.request_metrics: dict[int, dict] = {}
        self.last_step_events: dict = {}
        self.speculative_batch_calls = 0
        self.speculative_batch_sequences = 0
        self.speculative_max_batch_size = 0
        self._inflight: list[Sequence] | None = None
        self.overlapped_launches = 0
        self._exited = False
        atexit.register(self.exit)

    # ---- lifecycle ---------------------------------------------------------------------------
    def exit(self):
        if self._exited:
            return
        self._exited = True
        try:
            if self._inflight is not None:
                self._inflight = None
                self.model_runner.drain_decode()
        except Exception:
            pass
        try:
            self.model_runner.call("exit")
        finally:
            for p in self.ps:
                p.join(timeout=self.config.comm_timeout_s)
                if p.is_alive():
                    p.terminate()

    def reset_metrics(self):
        if not self.scheduler.is_finished():
            raise RuntimeError("cannot reset metrics while requests are active")
        self.request_metrics.clear()
        self.last_step_events = {}
        self.speculative_batch_calls = self.speculative_batch_sequences = self.speculative_max_batch_size = 0
        self.scheduler.reset_metrics()

    # ---- requests ----------------------------------------------------------------------------
    @staticmethod
    def new_request_metric(seq_id: int, prompt_tokens: int) -> dict:
        return {
            "seq_id": seq_id, "arrival_time": perf_counter(), "first_token_time": None,
            "token_times": [], "output_event_times": [], "speculative_step_latencies": [],
            "finish_time": None, "prompt_tokens": prompt_tokens, "output_tokens": 0, "success": False,
            "failure_reason": None, "speculative_steps": 0, "speculative_draft_tokens": 0,
            "speculative_accepted_tokens": 0, "speculative_emitted_tokens": 0,
            "speculative_accept_all_count": 0, "speculative_gamma_counts": {}, "speculative_trace": [],
            "speculative_timing": {},
        }

    def add_request(self, prompt: str | list[int], sampling_params: SamplingParams) -> int:
        if isinstance(prompt, str):
            prompt = self.tokenizer.encode(prompt)
        seq = Sequence(list(prompt), sampling_params)
        self.request_metrics[seq.seq_id] = self.new_request_metric(seq.seq_id, len(prompt))
        self.scheduler.add(seq)
        return seq.seq_id

    def is_finished(self) -> bool:
        return self.scheduler.is_finished()

    # ---- stepping ----------------------------------------------------------------------------
    def _can_run_speculative_step(self, out) -> bool:
        return (not out.prefill_seqs and bool(out.decode_seqs)
                and getattr(self.model_runner, "draft_model", None) is not None)

    def _record_emission(self, seq, metric, emitted: int, step_end: float, events: dict):
        if emitted > 0:
            if metric["first_token_time"] is None:
                metric["first_token_time"] = step_end
                events["first_token_seq_ids"].append(seq.seq_id)
            events["decode_seq_ids"].append(seq.seq_id)
            metric["token_times"].extend([step_end] * emitted)
            metric["output_event_times"].append(step_end)
            metric["output_tokens"] = seq.num_completion_tokens
        if seq.is_finished and metric["finish_time"] is None:
            metric["finish_time"] = step_end
            metric["success"] = True
            events["finished_seq_ids"].append(seq.seq_id)

    def _base_events(self, step_start, step_end, seqs, prefill_seqs, num_tokens):
        return {
            "step_start": step_start, "step_end": step_end, "is_prefill": bool(prefill_seqs),
            "num_tokens": num_tokens, "scheduled_seq_ids": [s.seq_id for s in seqs],
            "prefill_seq_ids": [s.seq_id for s in prefill_seqs], "first_token_seq_ids": [],
            "decode_seq_ids": [], "finished_seq_ids": [],
            "waiting_queue_size": len(self.scheduler.waiting), "running_queue_size": len(self.scheduler.running),
        }

    def step(self):
        with nvtx_range("llmserve.step"):
            return self._step()

    def _step(self):
        if self._inflight is not None:
            return self._overlapped_step()
        step_start = perf_counter()
        with nvtx_range("schedule"):
            out = self.scheduler.schedule()
        seqs = out.scheduled_seqs
        if self._can_run_speculative_step(out):
            reserve = self.model_runner.speculative_gamma + 2
            bm = self.scheduler.block_manager
            ready = bm.ensure_slots(seqs[0], reserve) if len(seqs) == 1 else bm.ensure_slots_batch(seqs, reserve)
            if ready:
                if len(seqs) == 1:
                    method = ("run_speculative_tree_single" if self.model_runner.speculative_tree_nodes
                              else "run_speculative_single")
                    results = [self.model_runner.call(method, seqs[0])]
                else:
                    results = self.model_runner.call("run_speculative_batch", seqs)
                return self._postprocess_speculative_step(seqs, results, step_start)

        if self._can_overlap(out):
            return self._start_overlap(out, step_start)
        before = {s.seq_id: s.num_completion_tokens for s in seqs}
        token_ids = self.model_runner.call("run", out)
        self.scheduler.postprocess(out, token_ids)
        step_end = perf_counter()
        events = self._base_events(step_start, step_end, seqs, out.prefill_seqs, out.num_batched_tokens)
        for s in seqs:
            metric = self.request_metrics.get(s.seq_id)
            if metric is not None:
                self._record_emission(s, metric, s.num_completion_tokens - before[s.seq_id], step_end, events)
        self.last_step_events = events
        return [(s.seq_id, s.completion_token_ids) for s in seqs if s.is_finished], out.num_batched_tokens

    # ---- overlapped decode ---------------------------------------------------------------------
    # In a run of pure-decode steps with greedy sampling, step N+1 is launched before step N's
    # tokens reach the host: its input ids are taken from step N's output on the device, its
    # positions and block slots only depend on sequence lengths, and the host work of a step
    # (reading tokens, postprocessing, metrics, scheduling, packing the next launch) runs while the
    # GPU computes the next one.  A sequence that stops on EOS is computed one extra step and
    # that token is dropped; its KV write lands in its own unsealed tail block.  Anything else --
    # a waiting request, a full pool, a batch the graphs do not cover -- drains the pipeline and
    # the scheduler takes over again.
    def _can_overlap(self, out) -> bool:
        r = self.model_runner
        return (self.config.overlap_decode and not out.prefill_seqs and bool(out.decode_seqs)
                and r.can_overlap()
                and r.overlap_fits(len(out.decode_seqs), max(len(s.block_table) for s in out.decode_seqs) + 1))

    def _start_overlap(self, out, step_start):
        seqs = list(out.decode_seqs)
        pos = np.fromiter((len(s) - 1 for s in seqs), dtype=np.int32, count=len(seqs))
        ids = np.fromiter((s.last_token for s in seqs), dtype=np.int32, count=len(seqs))
        self.model_runner.overlap_launch(seqs, pos, ids, -1, False)
        self.overlapped_launches += 1
        self._inflight = seqs
        self.last_step_events = self._base_events(step_start, perf_counter(), seqs, [], len(seqs))
        return [], len(seqs)

    def _plan_next(self, prev: list[Sequence]):
        """Sequences, positions and feed rows of the step after ``prev``; None to drain."""
        sched = self.scheduler
        if sched.waiting:
            return None
        live = [s for s in prev if not s.is_finished]
        if len(live) != len(sched.running):
            return None
        bm, bsz = sched.block_manager, sched.block_manager.block_size
        rows, seqs = [], []
        need = 0
        for i, s in enumerate(prev):
            if s.is_finished or s.num_completion_tokens + 1 >= s.max_tokens:
                continue          # done, or the in-flight token is its last
            L = len(s)            # the in-flight token sits at position L
            if L % bsz == 0 and len(s.block_table) <= L // bsz:
                need += 1
            rows.append(i)
            seqs.append(s)
        if not seqs or need > len(bm.free_block_ids):
            return None
        if not self.model_runner.overlap_fits(len(seqs), max(len(s.block_table) for s in seqs) + 1):
            return None
        for s in seqs:
            L = len(s)
            if L % bsz == 0:
                bm._seal(s, L // bsz - 1)            # every token of that block is known now
                if len(s.block_table) <= L // bsz:
                    s.block_table.append(bm._take_next_free().block_id)
        pos = np.fromiter((len(s) for s in seqs), dtype=np.int32, count=len(seqs))
        return seqs, pos, np.asarray(rows, dtype=np.int32)

    def _overlapped_step(self):
        step_start = perf_counter()
        prev = self._inflight
        plan = self._plan_next(prev)
        runner = self.model_runner
        if plan is None:
            self._inflight = None
            tokens = runner.drain_decode()
            launched = 0
        else:
            seqs, pos, feed = plan
            runner.overlap_launch(seqs, pos, 0, feed, True)
            self.overlapped_launches += 1
            tokens = runner.collect_decode()
            self._inflight = seqs
            launched = len(seqs)
        step_end = perf_counter()
        events = self._base_events(step_start, step_end, prev, [], launched)
        done = []
        bm = self.scheduler.block_manager
        for s, t in zip(prev, tokens):
            if s.is_finished:
                continue          # stopped on EOS one step earlier: this token is dropped
            self.scheduler._postprocess_sequence(s, t, is_prefill=False)
            if not s.is_finished and len(s) % bm.block_size == 0:
                bm._seal(s, len(s) // bm.block_size - 1)   # as the synchronous may_append would
            metric = self.request_metrics.get(s.seq_id)
            if metric is not None:
                self._record_emission(s, metric, 1, step_end, events)
            if s.is_finished:
                done.append((s.seq_id, s.completion_token_ids))
        self.last_step_events = events
        return done, launched

    def _postprocess_speculative_step(self, seqs, results, step_start):
        if len(seqs) != len(results):
            raise ValueError("speculative output count does not match scheduled sequences")
        before = {s.seq_id: s.num_completion_tokens for s in seqs}
        for s, r in zip(seqs, results):
            self.scheduler.postprocess_speculative(s, r.token_ids)
        step_end = perf_counter()
        self.speculative_batch_calls += 1
        self.speculative_batch_sequences += len(seqs)
        self.speculative_max_batch_size = max(self.speculative_max_batch_size, len(seqs))
        events = self._base_events(step_start, step_end, seqs, [], 0)
        n_draft = n_acc = n_emit = 0
        debug_by_seq = {}
        for s, r in zip(seqs, results):
            emitted = s.num_completion_tokens - before[s.seq_id]
            n_draft += r.num_draft_tokens
            n_acc += r.num_accepted
            n_emit += emitted
            m = self.request_metrics.get(s.seq_id)
            if m is not None:
                m["speculative_step_latencies"].append(step_end - step_start)
                m["speculative_steps"] += 1
                m["speculative_draft_tokens"] += r.num_draft_tokens
                m["speculative_accepted_tokens"] += r.num_accepted
                m["speculative_emitted_tokens"] += emitted
                m["speculative_accept_all_count"] += int(r.accepted_all)
                key = str(r.num_draft_tokens)
                m["speculative_gamma_counts"][key] = m["speculative_gamma_counts"].get(key, 0) + 1
                for name, value in (r.timing or {}).items():
                    m["speculative_timing"][name] = m["speculative_timing"].get(name, 0.0) + float(value)
                if r.debug is not None:
                    entry = {"step": m["speculative_steps"], "draft_token_ids": r.debug.get("draft_token_ids"),
                             "matches": r.debug.get("matches"),
                             "emitted_token_ids": [int(t) for t in r.token_ids],
                             "num_accepted": int(r.num_accepted), "accepted_all": bool(r.accepted_all)}
                    for k in ("start_token_id", "target_argmax_token_ids", "draft_token_target_ranks"):
                        if k in r.debug:
                            entry[k] = r.debug[k]
                    m["speculative_trace"].append(entry)
                self._record_emission(s, m, emitted, step_end, events)
            if r.debug is not None:
                debug_by_seq[s.seq_id] = r.debug
        events.update({
            "num_tokens": n_emit, "speculative": True, "speculative_batch_size": len(seqs),
            "speculative_num_draft_tokens": n_draft, "speculative_num_accepted": n_acc,
            "speculative_accepted_all": all(r.accepted_all for r in results),
            "speculative_emitted_tokens": n_emit,
        })
        if debug_by_seq:
            events["speculative_debug_by_seq"] = debug_by_seq
            if len(seqs) == 1:
                events["speculative_debug"] = debug_by_seq[seqs[0].seq_id]
        self.last_step_events = events
        done = [s.seq_id for s in seqs if s.is_finished]
        if done:
            self.model_runner.call("clear_speculative_state", done)
        return [(s.seq_id, s.completion_token_ids) for s in seqs if s.is_finished], n_emit

    # ---- metrics -----------------------------------------------------------------------------
    def get_metrics(self) -> dict:
        now = perf_counter()
        kv = self.scheduler.kv_capacity_metrics()
        kv.update(self.model_runner.get_memory_metrics())
        requests = []
        ttfts, itls, events_lat, spec_lat, e2e, tpots = [], [], [], [], [], []
        wall_start = wall_end = None
        tot = dict(out=0, steps=0, draft=0, acc=0, emit=0, all=0)
        gamma_counts, timing = {}, {}
        for m in self.request_metrics.values():
            arrival, first, finish = m["arrival_time"], m["first_token_time"], m["finish_time"]
            wall_start = arrival if wall_start is None else min(wall_start, arrival)
            end = finish if finish is not None else now
            wall_end = end if wall_end is None else max(wall_end, end)
            tot["out"] += m["output_tokens"]
            tot["steps"] += m["speculative_steps"]
            tot["draft"] += m["speculative_draft_tokens"]
            tot["acc"] += m["speculative_accepted_tokens"]
            tot["emit"] += m["speculative_emitted_tokens"]
            tot["all"] += m["speculative_accept_all_count"]
            for k, c in m["speculative_gamma_counts"].items():
                gamma_counts[k] = gamma_counts.get(k, 0) + c
            for k, v in m["speculative_timing"].items():
                timing[k] = timing.get(k, 0.0) + v
            ttft = None if first is None else first - arrival
            if ttft is not None:
                ttfts.append(ttft)
            req_itl = _diffs(m["token_times"])
            req_ev = _diffs(m["output_event_times"])
            itls += req_itl
            events_lat += req_ev
            spec_lat += m["speculative_step_latencies"]
            latency = None
            failure = m["failure_reason"]
            if finish is not None:
                latency = finish - arrival
                e2e.append(latency)
                if m["output_tokens"] > 1 and first is not None:
                    tpots.append((finish - first) / (m["output_tokens"] - 1))
                elif m["output_tokens"] == 1:
                    tpots.append(0.0)
            elif not m["success"]:
                failure = failure or "unfinished"
            requests.append({
                "seq_id": m["seq_id"], "prompt_tokens": m["prompt_tokens"], "output_tokens": m["output_tokens"],
                "success": m["success"], "failure_reason": None if m["success"] else failure,
                "arrival_time": arrival, "first_token_time": first, "token_times": m["token_times"],
                "finish_time": finish, "ttft": ttft, "output_event_times": m["output_event_times"],
                "burst_itl": req_itl, "itl": req_itl, "output_event_latency": req_ev,
                "speculative_step_latency": m["speculative_step_latencies"], "latency": latency,
                "speculative_steps": m["speculative_steps"],
                "speculative_draft_tokens": m["speculative_draft_tokens"],
                "speculative_accepted_tokens": m["speculative_accepted_tokens"],
                "speculative_emitted_tokens": m["speculative_emitted_tokens"],
                "speculative_accept_all_count": m["speculative_accept_all_count"],
                "speculative_gamma_counts": dict(sorted(m["speculative_gamma_counts"].items(),
                                                        key=lambda kv_: int(kv_[0]))),
                "speculative_trace": m["speculative_trace"], "speculative_timing": m["speculative_timing"],
            })
        wall = (wall_end - wall_start) if wall_start is not None else 0.0
        steps, calls = tot["steps"], self.speculative_batch_calls
        n_ok = sum(1 for r in requests if r["success"])
        return {
            "summary": {
                "num_requests": len(requests), "num_finished": n_ok, "num_failed": len(requests) - n_ok,
                "total_output_tokens": tot["out"], "wall_time": wall,
                "throughput": tot["out"] / wall if wall > 0 else 0.0,
                "ttft": summarize(ttfts), "burst_itl": summarize(itls), "itl": summarize(itls),
                "output_event_latency": summarize(events_lat), "speculative_step_latency": summarize(spec_lat),
                "tpot": summarize(tpots), "request_latency": summarize(e2e),
                "speculative": {
                    "steps": steps, "batch_calls": calls,
                    "mean_batch_size": self.speculative_batch_sequences / calls if calls else None,
                    "max_batch_size": self.speculative_max_batch_size,
                    "draft_tokens": tot["draft"], "accepted_tokens": tot["acc"], "emitted_tokens": tot["emit"],
                    "acceptance_rate": tot["acc"] / tot["draft"] if tot["draft"] else None,
                    "acceptance_length": tot["emit"] / steps if steps else None,
                    "accepted_length": tot["acc"] / steps if steps else None,
                    "draft_tokens_per_step": tot["draft"] / steps if steps else None,
                    "accept_all_count": tot["all"],
                    "gamma_counts": dict(sorted(gamma_counts.items(), key=lambda kv_: int(kv_[0]))),
                    "timing": {k: {"total": v, "mean": v / steps if steps else None}
                               for k, v in sorted(timing.items())},
                },
                "kv_cache": kv,
            },
            "requests": sorted(requests, key=lambda r: r["seq_id"]),
        }

    # ---- offline generation ------------------------------------------------------------------
    def generate(self, prompts, sampling_params, use_tqdm: bool = True):
        bar = tqdm(total=len(prompts), desc="Generating", dynamic_ncols=True, disable=not use_tqdm)
        if not isinstance(sampling_params, list):
            sampling_params = [sampling_params] * len(prompts)
        for prompt, sp in zip(prompts, sampling_params):
            self.add_request(prompt, sp)
        done = {}
        prefill_tps = decode_tps = 0.0
        while not self.is_finished():
            t = perf_counter()
            output, num_tokens = self.step()
            dt = max(perf_counter() - t, 1e-9)
            if self.last_step_events.get("prefill_seq_ids"):
                prefill_tps = num_tokens / dt
            else:
                decode_tps = num_tokens / dt
            bar.set_postfix({"Prefill": f"{int(prefill_tps)}tok/s", "Decode": f"{int(decode_tps)}tok/s"})
            for seq_id, toks in output:
                done[seq_id] = toks
                bar.update(1)
        bar.close()
        return [{"text": self.tokenizer.decode(done[k]), "token_ids": done[k]} for k in sorted(done)]
