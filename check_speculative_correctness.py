"""Speculative decoding correctness check: the same prompt(s) through a plain engine and an EAGLE3
engine, compared token for token, plus a serial-vs-batched consistency mode.

``python check_speculative_correctness.py --model TARGET --speculative-model DRAFT [--argmax-sampler]
[--require-token-match] [--batch-consistency --batch-sizes 2,4] [--output-json report.json]``

Behaviour parity with ``check_speculative_correctness.py`` of the reference (arguments :51-74,
``build_checks`` :236-281, ``build_batch_checks`` :284-313, report layout of ``run_comparison``
:374-433 and ``run_batch_consistency`` :316-371, exit status of ``main`` :495-519).  Each run uses
a fresh engine (built by ``engine_factory``, injectable for tests), greedy argmax sampling where
asked, and a step limit; the checks cover completion, output lengths against the metrics, and the
consistency of the speculative counters.  Matching token ids is reported as an observation (and
required with ``--require-token-match``).  Engines here default to the B200 path; ``--device cpu``
runs the fp32 host path.
"""
import argparse
import gc
import json
import os
from dataclasses import asdict, dataclass

DEFAULT_BATCH_PROMPTS = [
    "Explain speculative decoding in one concise paragraph.",
    "Summarize why paged KV cache improves LLM serving.",
    "Describe the difference between prefill and decode.",
    "Explain continuous batching to a systems engineer.",
]


@dataclass(slots=True)
class RunResult:
    token_ids: list
    metrics: dict
    step_events: list


@dataclass(slots=True)
class BatchRunResult:
    token_ids: list
    metrics: dict
    step_events: list


class ArgmaxSampler:
    is_greedy = True

    def __call__(self, logits, temperatures):
        return logits.argmax(dim=-1)


def parse_token_ids(value: str) -> list:
    ids = [v.strip() for v in value.split(",") if v.strip()]
    if not ids:
        raise ValueError("--prompt-token-ids must contain at least one token id")
    return [int(v) for v in ids]


def parse_batch_sizes(value: str) -> list:
    sizes = [int(v) for v in value.split(",") if v.strip()]
    if not sizes:
        raise ValueError("--batch-sizes must contain at least one positive integer")
    if any(s <= 0 for s in sizes):
        raise ValueError("--batch-sizes values must be positive")
    return sorted(set(sizes))


def build_parser() -> argparse.ArgumentParser:
    p = argparse.ArgumentParser(description="Small speculative decoding correctness check for llmserve_b200")
    p.add_argument("--model", default=os.environ.get("MODEL_PATH", "~/models/Qwen3-8B/"))
    p.add_argument("--speculative-model", default=os.environ.get("SPECULATIVE_MODEL"))
    p.add_argument("--prompt", default=None)
    p.add_argument("--prompt-token-ids", default=None, type=parse_token_ids)
    p.add_argument("--output-len", type=int, default=4)
    p.add_argument("--temperature", type=float, default=1.0)
    p.add_argument("--seed", type=int, default=0)
    p.add_argument("--speculative-gamma", type=int, default=3)
    p.add_argument("--speculative-tree-nodes", type=int, choices=[0, 6, 10], default=0)
    p.add_argument("--speculative-accept-mode", choices=["greedy", "rejection"], default="greedy")
    p.add_argument("--speculative-trace", action="store_true")
    p.add_argument("--speculative-cuda-graphs", action="store_true",
                   help="run the speculative engine's greedy chain step through its CUDA graphs")
    p.add_argument("--argmax-sampler", action="store_true")
    p.add_argument("--max-model-len", type=int, default=64)
    p.add_argument("--max-num-batched-tokens", type=int, default=64)
    p.add_argument("--max-steps", type=int, default=64)
    p.add_argument("--require-token-match", action="store_true")
    p.add_argument("--batch-consistency", action="store_true")
    p.add_argument("--batch-sizes", type=parse_batch_sizes, default=[2, 4])
    p.add_argument("--device", choices=["cuda", "cpu"], default="cuda")
    p.add_argument("--load-format", choices=["auto", "dummy"], default="auto")
    p.add_argument("--output-json", default=None)
    return p


def default_engine_factory(model: str, **kwargs):
    from llmserve_b200 import LLM
    return LLM(model, **kwargs)


def _release():
    gc.collect()
    try:
        import torch
        if torch.cuda.is_available():
            torch.cuda.empty_cache()
    except ImportError:  # pragma: no cover
        pass


class Checker:
    """Runs engines for the checks; ``engine_factory(model, **engine_kwargs)`` builds one."""

    def __init__(self, args, engine_factory=default_engine_factory):
        self.args = args
        self.factory = engine_factory
        self.model = os.path.expanduser(args.model)
        self.draft = os.path.expanduser(args.speculative_model) if args.speculative_model else None
        if self.draft is None:
            raise ValueError("--speculative-model or SPECULATIVE_MODEL is required")

    def _engine(self, speculative: bool, tree_nodes: int = 0, accept_mode: str = "greedy", trace: bool = False):
        import torch
        torch.manual_seed(self.args.seed)
        a = self.args
        graphs = speculative and getattr(a, "speculative_cuda_graphs", False)
        extra = {"speculative_cuda_graphs": True} if graphs else {}
        return self.factory(self.model, enforce_eager=not graphs, tensor_parallel_size=1,
                            max_model_len=a.max_model_len, max_num_batched_tokens=a.max_num_batched_tokens,
                            speculative_model=self.draft if speculative else None,
                            speculative_gamma=a.speculative_gamma, speculative_tree_nodes=tree_nodes,
                            speculative_accept_mode=accept_mode, speculative_trace=trace, device=a.device,
                            load_format=a.load_format, seed=a.seed, **extra)

    def _drain(self, engine, outputs, events, limit):
        steps = 0
        while not engine.is_finished():
            done, _ = engine.step()
            steps += 1
            events.append(dict(getattr(engine, "last_step_events", {})))
            for sid, toks in done:
                outputs[sid] = toks
            if steps > limit:
                raise RuntimeError(f"requests did not finish within {limit} engine steps")

    def run_single(self, prompt, speculative: bool) -> RunResult:
        from llmserve_b200 import SamplingParams
        a = self.args
        engine = self._engine(speculative, a.speculative_tree_nodes if speculative else 0,
                              a.speculative_accept_mode, a.speculative_trace)
        try:
            if a.argmax_sampler:
                engine.model_runner.sampler = ArgmaxSampler()
            sid = engine.add_request(prompt, SamplingParams(temperature=a.temperature, max_tokens=a.output_len,
                                                            ignore_eos=True))
            outputs, events = {}, []
            self._drain(engine, outputs, events, a.max_steps)
            return RunResult(outputs.get(sid, []), engine.get_metrics(), events)
        finally:
            engine.exit()
            _release()

    def run_group(self, prompts, submit_all: bool) -> BatchRunResult:
        from llmserve_b200 import SamplingParams
        a = self.args
        engine = self._engine(True)
        try:
            engine.model_runner.sampler = ArgmaxSampler()
            sp = SamplingParams(temperature=1.0, max_tokens=a.output_len, ignore_eos=True)
            outputs, events, ids = {}, [], []
            if submit_all:
                ids = [engine.add_request(p, sp) for p in prompts]
                self._drain(engine, outputs, events, a.max_steps * len(prompts))
            else:
                for p in prompts:
                    ids.append(engine.add_request(p, sp))
                    self._drain(engine, outputs, events, a.max_steps)
            return BatchRunResult([outputs.get(i, []) for i in ids], engine.get_metrics(), events)
        finally:
            engine.exit()
            _release()


def build_checks(baseline: RunResult, speculative: RunResult, max_tokens: int) -> dict:
    b, s = baseline.metrics["summary"], speculative.metrics["summary"]
    spec = s.get("speculative", {})
    rate = spec.get("acceptance_rate")
    checks = {
        "baseline_finished": b["num_finished"] == 1 and b["num_failed"] == 0,
        "speculative_finished": s["num_finished"] == 1 and s["num_failed"] == 0,
        "baseline_output_len_matches_metrics": len(baseline.token_ids) == b["total_output_tokens"],
        "speculative_output_len_matches_metrics": len(speculative.token_ids) == s["total_output_tokens"],
        "baseline_output_len_within_max": len(baseline.token_ids) <= max_tokens,
        "speculative_output_len_within_max": len(speculative.token_ids) <= max_tokens,
        "speculative_metrics_present": spec.get("steps", 0) > 0,
        "speculative_metrics_consistent": (
            spec.get("draft_tokens", 0) >= spec.get("accepted_tokens", 0) >= 0
            and 0 <= spec.get("emitted_tokens", 0) <= s["total_output_tokens"]
            and (rate is None or 0.0 <= rate <= 1.0)),
        "token_ids_match": baseline.token_ids == speculative.token_ids,
    }
    checks["required_checks_pass"] = all(v for k, v in checks.items() if k != "token_ids_match")
    return checks


def build_batch_checks(serial_token_ids: list, batched: BatchRunResult, expected_batch_size: int,
                       output_len: int) -> dict:
    summ = batched.metrics["summary"]
    spec = summ.get("speculative", {})
    per_request = [a == b for a, b in zip(serial_token_ids, batched.token_ids)]
    checks = {
        "request_count_matches": len(batched.token_ids) == expected_batch_size,
        "all_requests_finished": summ.get("num_finished") == expected_batch_size and summ.get("num_failed") == 0,
        "all_output_lengths_match": all(len(t) == output_len for t in batched.token_ids),
        "speculative_metrics_present": spec.get("steps", 0) > 0,
        "multi_request_batch_used": (spec.get("max_batch_size") or 0) >= expected_batch_size,
        "token_ids_match": len(per_request) == expected_batch_size and all(per_request),
    }
    checks["required_checks_pass"] = all(checks.values())
    checks["per_request_matches"] = per_request
    return checks


def _config(args, checker: Checker, **extra) -> dict:
    return {"model": checker.model, "speculative_model": checker.draft, "output_len": args.output_len,
            "seed": args.seed, "speculative_gamma": args.speculative_gamma, "max_model_len": args.max_model_len,
            "max_num_batched_tokens": args.max_num_batched_tokens, **extra}


def run_comparison(args, engine_factory=default_engine_factory) -> dict:
    checker = Checker(args, engine_factory)
    prompt = args.prompt if args.prompt is not None else (args.prompt_token_ids or [1, 2, 3, 4])
    base = checker.run_single(prompt, speculative=False)
    spec = checker.run_single(prompt, speculative=True)
    return {"config": _config(args, checker, prompt=args.prompt,
                              prompt_token_ids=None if args.prompt is not None else prompt,
                              temperature=args.temperature, speculative_tree_nodes=args.speculative_tree_nodes,
                              speculative_accept_mode=args.speculative_accept_mode,
                              speculative_trace=args.speculative_trace, argmax_sampler=args.argmax_sampler),
            "baseline": asdict(base), "speculative": asdict(spec),
            "checks": build_checks(base, spec, args.output_len)}


def run_batch_consistency(args, engine_factory=default_engine_factory) -> dict:
    checker = Checker(args, engine_factory)
    sizes = args.batch_sizes
    prompts = [DEFAULT_BATCH_PROMPTS[i % len(DEFAULT_BATCH_PROMPTS)] for i in range(max(sizes))]
    serial = checker.run_group(prompts, submit_all=False)
    batches = []
    for n in sizes:
        batched = checker.run_group(prompts[:n], submit_all=True)
        batches.append({"batch_size": n, "prompts": prompts[:n], "serial_token_ids": serial.token_ids[:n],
                        "batched": asdict(batched),
                        "checks": build_batch_checks(serial.token_ids[:n], batched, n, args.output_len)})
    return {"config": _config(args, checker, batch_sizes=sizes, argmax_sampler=True), "serial": asdict(serial),
            "batches": batches, "required_checks_pass": all(b["checks"]["required_checks_pass"] for b in batches)}


def _mark(v: bool) -> str:
    return "PASS" if v else "FAIL"


def print_report(report: dict):
    c = report["checks"]
    spec = report["speculative"]["metrics"]["summary"].get("speculative", {})
    print("\nSpeculative Correctness Check\n=============================")
    print(f"baseline tokens:     {report['baseline']['token_ids']}")
    print(f"speculative tokens:  {report['speculative']['token_ids']}")
    print(f"token ids match:     {c['token_ids_match']}  (observation, not a distribution proof)\n")
    print("Required Checks\n---------------")
    for k, v in c.items():
        if k not in ("token_ids_match", "required_checks_pass"):
            print(f"{k:<40} {_mark(v)}")
    print(f"{'required_checks_pass':<40} {_mark(c['required_checks_pass'])}\n")
    print("Speculative Metrics\n-------------------")
    for label, key in (("steps", "steps"), ("draft tokens", "draft_tokens"), ("accepted", "accepted_tokens"),
                       ("emitted", "emitted_tokens"), ("acceptance", "acceptance_rate"),
                       ("accept-all", "accept_all_count")):
        print(f"{label + ':':<16}{spec.get(key)}")
    print()


def print_batch_report(report: dict):
    print("\nBatched Speculative Consistency Check\n=====================================")
    for b in report["batches"]:
        c = b["checks"]
        print(f"batch size:       {b['batch_size']}")
        print(f"token ids match:  {_mark(c['token_ids_match'])}")
        print(f"finished:         {_mark(c['all_requests_finished'])}")
        print(f"max batch seen:   {b['batched']['metrics']['summary']['speculative'].get('max_batch_size')}")
        print(f"per request:      {c['per_request_matches']}\n")
    print(f"required checks:  {_mark(report['required_checks_pass'])}\n")


def main(argv=None, engine_factory=default_engine_factory) -> int:
    args = build_parser().parse_args(argv)
    if args.batch_consistency:
        report = run_batch_consistency(args, engine_factory)
        print_batch_report(report)
        ok = report["required_checks_pass"]
    else:
        report = run_comparison(args, engine_factory)
        print_report(report)
        ok = report["checks"]["required_checks_pass"] and (
            not args.require_token_match or report["checks"]["token_ids_match"])
    if args.output_json:
        out = os.path.expanduser(args.output_json)
        os.makedirs(os.path.dirname(out) or ".", exist_ok=True)
        with open(out, "w") as f:
            json.dump(report, f, indent=2)
        print(f"Wrote JSON results to {out}")
    return 0 if ok else 1


if __name__ == "__main__":
    raise SystemExit(main())
