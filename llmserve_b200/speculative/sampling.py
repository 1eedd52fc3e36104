"""Acceptance rules (``llmserve/speculative/sampling.py`` of the reference).

* greedy: accept draft tokens while they equal the target argmax; the first mismatch emits the
  target token, full acceptance emits the bonus token from the last verify row;
* rejection sampling (Leviathan et al., 2023): accept ``x`` with ``min(1, p(x)/q(x))``; on reject
  sample from ``norm(max(p - q, 0))``; after full acceptance sample the bonus from ``p``.

``greedy_accept_batch`` is the batched tensor form (one comparison, a cumulative product and a
gather for the whole batch); ``greedy_accept_packed`` is what the executor uses: one sm_100a
kernel that also packs the start and draft tokens, so the step needs a single host copy.
"""
import torch

from llmserve_b200.speculative.types import SpeculativeSampleResult


def sample_from_logits(logits: torch.Tensor, temperature: float) -> torch.Tensor:
    if not temperature > 1e-10:
        raise ValueError("temperature must be > 1e-10")
    probs = torch.softmax(logits.float() / temperature, dim=-1)
    return torch.multinomial(probs.reshape(-1, probs.shape[-1]), 1).view(*logits.shape[:-1])


def sample_from_probs(probs: torch.Tensor) -> int:
    return int(torch.multinomial(probs.float(), 1).item())


def correction_distribution(target_probs: torch.Tensor, draft_probs: torch.Tensor) -> torch.Tensor:
    diff = (target_probs.float() - draft_probs.float()).clamp_min(0)
    total = diff.sum()
    if total <= 0:
        return target_probs.float() / target_probs.float().sum()
    return diff / total


def speculative_accept_reject(target_probs, draft_probs, draft_token_ids, random_values=None):
    n = int(draft_token_ids.numel())
    if target_probs.ndim != 2 or draft_probs.ndim != 2:
        raise ValueError("probabilities must be two-dimensional")
    if target_probs.shape[0] != n + 1 or draft_probs.shape[0] != n:
        raise ValueError("need gamma draft rows and gamma + 1 target rows")
    accepted: list[int] = []
    for i in range(n):
        tok = int(draft_token_ids[i])
        p, q = float(target_probs[i, tok]), float(draft_probs[i, tok])
        ratio = 1.0 if q <= 0 else min(1.0, p / q)
        u = float(random_values[i]) if random_values is not None else float(torch.rand(()))
        if u <= ratio:
            accepted.append(tok)
            continue
        fix = sample_from_probs(correction_distribution(target_probs[i], draft_probs[i]))
        return SpeculativeSampleResult(accepted + [fix], accepted, fix, len(accepted), False)
    bonus = sample_from_probs(target_probs[n])
    return SpeculativeSampleResult(accepted + [bonus], accepted, bonus, len(accepted), True)


def speculative_accept_reject_from_logits(target_logits, draft_logits, draft_token_ids, temperature,
                                          random_values=None):
    if not temperature > 1e-10:
        raise ValueError("temperature must be > 1e-10")
    tp_ = torch.softmax(target_logits.float() / temperature, dim=-1)
    dp_ = torch.softmax(draft_logits.float() / temperature, dim=-1)
    return speculative_accept_reject(tp_, dp_, draft_token_ids, random_values=random_values)


def greedy_accept_from_ids(target_ids: list[int], draft_ids: list[int]) -> SpeculativeSampleResult:
    accepted: list[int] = []
    for i, d in enumerate(draft_ids):
        if target_ids[i] != d:
            return SpeculativeSampleResult(accepted + [target_ids[i]], accepted, target_ids[i], len(accepted), False)
        accepted.append(d)
    bonus = target_ids[len(draft_ids)]
    return SpeculativeSampleResult(accepted + [bonus], accepted, bonus, len(accepted), True)


def speculative_accept_greedy_from_logits(target_logits, draft_token_ids) -> SpeculativeSampleResult:
    n = int(draft_token_ids.numel())
    if target_logits.ndim != 2 or target_logits.shape[0] != n + 1:
        raise ValueError("need gamma + 1 target rows")
    return greedy_accept_from_ids(target_logits.argmax(dim=-1).tolist(), [int(x) for x in draft_token_ids.tolist()])


def greedy_accept_batch(target_ids: torch.Tensor, draft_ids: torch.Tensor):
    """target_ids [B, g+1], draft_ids [B, g] (device) -> (num_accepted [B], final [B]) on device."""
    match = (target_ids[:, :-1] == draft_ids).to(torch.int32)
    num_acc = torch.cumprod(match, dim=1).sum(dim=1)
    final = target_ids.gather(1, num_acc.unsqueeze(1).long()).squeeze(1)
    return num_acc, final


def greedy_accept_packed(target_ids: torch.Tensor, draft_ids: torch.Tensor, start_ids: torch.Tensor) -> torch.Tensor:
    """``[B, g + 3]`` int64 rows ``[accepted, final, start, drafts...]`` for one host copy (one
    sm_100a kernel on CUDA; the batched torch form on the host)."""
    B, g = draft_ids.shape
    if not target_ids.is_cuda:
        num_acc, final = greedy_accept_batch(target_ids, draft_ids)
        return torch.cat([num_acc.unsqueeze(1).long(), final.unsqueeze(1).long(), start_ids.view(B, 1).long(),
                          draft_ids.long()], 1)
    from llmserve_b200.ops._ext import C
    out = torch.empty(B, g + 3, dtype=torch.int64, device=target_ids.device)
    C().greedy_accept(out, target_ids.long().contiguous(), draft_ids.long().contiguous(),
                      start_ids.long().contiguous().view(-1))
    return out
