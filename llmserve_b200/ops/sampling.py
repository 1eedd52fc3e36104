"""Token selection kernels.

* ``argmax``       -- greedy token per row (benchmarks' ``ArgmaxSampler``).
* ``sample``       -- temperature sampling by the exponential race of the reference's sampler
  (``llmserve/layers/sampler.py:7-12``): ``argmax_i p_i / E_i`` with ``E_i ~ Exp(1)``, evaluated
  in log space as ``argmax_i (logit_i / T - log E_i)`` so no softmax is materialised.  The noise
  comes from a counter-based hash (the SplitMix64 finaliser, Steele, Lea & Flood 2014) of
  (seed, flat index), so a step is reproducible from its seed.
* ``local_argmax`` -- per-shard (max, index) pairs for vocab-parallel greedy decoding; the shards
  are combined with a tiny all-gather instead of gathering full logits.
"""
import numpy as np
import torch

from llmserve_b200.ops._ext import C, status


def argmax(logits: torch.Tensor) -> torch.Tensor:
    if not logits.is_cuda:
        return logits.float().argmax(dim=-1)
    out = torch.empty(logits.shape[0], dtype=torch.int64, device=logits.device)
    vals = torch.empty(logits.shape[0], dtype=torch.float32, device=logits.device)
    C().argmax_rows(out, vals, logits.contiguous())
    return out


def local_argmax(logits: torch.Tensor):
    """(values fp32 [B], indices int64 [B]) of each row's max (lowest index on ties)."""
    if not logits.is_cuda:
        v, i = logits.float().max(dim=-1)
        return v, i
    out = torch.empty(logits.shape[0], dtype=torch.int64, device=logits.device)
    vals = torch.empty(logits.shape[0], dtype=torch.float32, device=logits.device)
    C().argmax_rows(out, vals, logits.contiguous())
    return vals, out


def feed_ids(ids32: torch.Tensor, feed32: torch.Tensor, prev: torch.Tensor) -> torch.Tensor:
    """int64 step ids: ``prev[feed[i]]`` where ``feed[i] >= 0`` (the previous step's token, still on
    the device), else ``ids32[i]``."""
    if not ids32.is_cuda:
        out = ids32.long()
        m = feed32 >= 0
        out[m] = prev[feed32[m].long()]
        return out
    out = torch.empty(ids32.shape[0], dtype=torch.int64, device=ids32.device)
    C().feed_ids(out, ids32, feed32, prev, status(ids32.device))
    return out


def local_argmax_into(logits: torch.Tensor, values: torch.Tensor, indices: torch.Tensor) -> None:
    """``local_argmax`` writing into caller-owned ``values`` (fp32) / ``indices`` (int64)."""
    if not logits.is_cuda:
        v, i = logits.float().max(dim=-1)
        values.copy_(v)
        indices.copy_(i)
        return
    C().argmax_rows(indices, values, logits.contiguous())


def noise_uniform_ref(shape, seed: int) -> torch.Tensor:
    """Uniforms in (0, 1) identical to the CUDA kernel's (SplitMix64 finaliser of a counter)."""
    rows, cols = shape
    with np.errstate(over="ignore"):
        idx = np.arange(rows * cols, dtype=np.uint64)
        z = np.uint64(seed & (2**64 - 1)) * np.uint64(0x9E3779B97F4A7C15) + idx * np.uint64(0xBF58476D1CE4E5B9)
        z = (z ^ (z >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)
        z = (z ^ (z >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)
        z = z ^ (z >> np.uint64(31))
    u = ((z >> np.uint64(40)).astype(np.float64) + 0.5) / float(1 << 24)
    return torch.from_numpy(u.reshape(rows, cols))


def sample(logits: torch.Tensor, temperatures: torch.Tensor, seed: int) -> torch.Tensor:
    if not logits.is_cuda:
        u = noise_uniform_ref(logits.shape, seed).to(logits.device)
        score = logits.double() / temperatures.double().unsqueeze(1) - torch.log(-torch.log(u))
        return score.argmax(dim=-1)
    out = torch.empty(logits.shape[0], dtype=torch.int64, device=logits.device)
    C().sample_rows(out, logits.contiguous(), temperatures.float().contiguous(), int(seed) & (2**63 - 1))
    return out
