"""Test helpers: the reference implementation as an oracle (read-only import), tiny checkpoints."""
import importlib
import os
import sys

import pytest

# the reference checkout named by LLMSERVE_REFERENCE_PATH, else its package installed under baseline/_ref
_REF_CANDIDATES = [os.environ.get("LLMSERVE_REFERENCE_PATH", ""),
                   os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "baseline", "_ref")]


def reference_module(name: str):
    """Import ``llmserve.<name>`` from the reference checkout, or skip the test."""
    for root in _REF_CANDIDATES:
        if root and os.path.isdir(os.path.join(root, "llmserve")):
            if root not in sys.path:
                sys.path.append(root)
            break
    else:
        pytest.skip("reference implementation not available")
    try:
        return importlib.import_module(name)
    except Exception as e:  # pragma: no cover - depends on the environment
        pytest.skip(f"reference module {name} not importable: {e}")


class RecordingSampler:
    """A non-greedy sampler (so the engine hands it the full-vocabulary logits, gathered over the
    tensor-parallel ranks) that keeps a host fp32 copy of every call's logits.  It returns the
    argmax, or, with ``forced`` (one token list per call, e.g. another run's ``tokens``), those
    tokens: teacher forcing keeps two runs on the same sequences, so their logits can be compared
    step by step even where a near-tie flips an argmax."""
    is_greedy = False

    def __init__(self, forced=None):
        self.forced = forced
        self.logits = []
        self.tokens = []

    def __call__(self, logits, temperatures):
        import torch
        self.logits.append(logits.float().cpu())
        if self.forced is not None:
            out = torch.tensor(self.forced[len(self.tokens)], dtype=torch.int64, device=logits.device)
        else:
            out = logits.float().argmax(-1)
        self.tokens.append(out.tolist())
        return out


def compare_logits(got, ref, rel_tol: float):
    """Per-call checks of logits ``got`` against ``ref`` (lists of [rows, V] fp32 tensors):
    relative Frobenius error below ``rel_tol``, and the same argmax on every row whose reference
    top-2 gap exceeds twice the largest deviation of that row (where no perturbation of that size
    can change the winner).  Returns (worst relative error, rows compared by argmax)."""
    assert len(got) == len(ref), (len(got), len(ref))
    worst, checked = 0.0, 0
    for step, (a, b) in enumerate(zip(got, ref)):
        assert a.shape == b.shape, (step, a.shape, b.shape)
        rel = ((a - b).norm() / b.norm()).item()
        worst = max(worst, rel)
        assert rel < rel_tol, f"call {step}: relative logit error {rel:.3e} >= {rel_tol}"
        top2 = b.topk(2, dim=-1).values
        gap = top2[:, 0] - top2[:, 1]
        dev = (a - b).abs().amax(dim=-1)
        safe = gap > 2 * dev
        assert bool((a.argmax(-1)[safe] == b.argmax(-1)[safe]).all()), f"call {step}: argmax differs"
        checked += int(safe.sum())
    return worst, checked
