"""Tensor-parallel process state.

One process per GPU.  ``torch.distributed`` (NCCL on CUDA, gloo on the CPU tier) is the
plumbing: rendezvous, barriers, and the baseline collectives.  The row-parallel reductions of the
decode hot path go through ``llmserve_b200.parallel.fused`` (in-kernel NVLink peer loads/stores)
when ``Config.fused_collectives`` is set and the peers are reachable.

Reference: ``llmserve/engine/model_runner.py:19-25`` (``init_process_group("nccl", tcp://...)``)
and the ``dist.all_reduce`` / ``dist.gather`` call sites in ``linear.py:234-235`` and
``embed_head.py:35-65``.  Differences: an explicit process-group timeout (ranks that lose a peer
fail instead of blocking forever) and a vocab-parallel argmax that moves 12 bytes per row instead
of gathering whole logit rows to rank 0.
"""
from datetime import timedelta

import torch
import torch.distributed as dist


class _TP:
    rank = 0
    world_size = 1
    group = None
    device = torch.device("cpu")
    fused = None


_tp = _TP()


def init_tensor_parallel(rank: int, world_size: int, init_method: str, device: torch.device,
                         timeout_s: float = 120.0):
    _tp.rank, _tp.world_size, _tp.device = rank, world_size, device
    if world_size == 1:
        return
    if not dist.is_initialized():
        backend = "nccl" if device.type == "cuda" else "gloo"
        kwargs = {"device_id": device} if device.type == "cuda" else {}
        dist.init_process_group(backend, init_method=init_method, world_size=world_size, rank=rank,
                                timeout=timedelta(seconds=timeout_s), **kwargs)
    _tp.group = dist.group.WORLD


def destroy_tensor_parallel():
    if _tp.fused is not None:
        _tp.fused.close()
        _tp.fused = None
    if _tp.world_size > 1 and dist.is_initialized():
        dist.destroy_process_group()
    _tp.rank, _tp.world_size, _tp.group = 0, 1, None


def get_tp_rank() -> int:
    return _tp.rank


def get_tp_size() -> int:
    return _tp.world_size


def get_tp_device() -> torch.device:
    return _tp.device


def set_fused_comm(fused):
    _tp.fused = fused


def get_fused_comm():
    return _tp.fused


def all_reduce(x: torch.Tensor) -> torch.Tensor:
    if _tp.world_size > 1:
        dist.all_reduce(x, group=_tp.group)
    return x


def broadcast(x: torch.Tensor, src: int = 0) -> torch.Tensor:
    if _tp.world_size > 1:
        dist.broadcast(x, src=src, group=_tp.group)
    return x


def barrier():
    if _tp.world_size > 1:
        if _tp.device.type == "cuda":
            dist.barrier(group=_tp.group, device_ids=[_tp.device.index])
        else:
            dist.barrier(group=_tp.group)


def vocab_parallel_argmax(values: torch.Tensor, indices: torch.Tensor, shard_offset: int) -> torch.Tensor:
    """Combine per-shard (max value, local index) into the global argmax.

    Ties resolve to the lowest global index, matching ``argmax`` over the concatenated logits.
    """
    gidx = indices.to(torch.int64) + shard_offset
    if _tp.world_size == 1:
        return gidx
    vals = [torch.empty_like(values) for _ in range(_tp.world_size)]
    idxs = [torch.empty_like(gidx) for _ in range(_tp.world_size)]
    dist.all_gather(vals, values.contiguous(), group=_tp.group)
    dist.all_gather(idxs, gidx.contiguous(), group=_tp.group)
    v = torch.stack(vals, 0)
    i = torch.stack(idxs, 0)
    best = v.max(dim=0, keepdim=True).values
    cand = torch.where(v == best, i, torch.full_like(i, torch.iinfo(torch.int64).max))
    return cand.min(dim=0).values


def gather_logits(logits: torch.Tensor) -> torch.Tensor:
    """Full-vocab logits on every rank (temperature sampling, rejection acceptance, traces)."""
    if _tp.world_size == 1:
        return logits
    parts = [torch.empty_like(logits) for _ in range(_tp.world_size)]
    dist.all_gather(parts, logits.contiguous(), group=_tp.group)
    return torch.cat(parts, dim=-1)
