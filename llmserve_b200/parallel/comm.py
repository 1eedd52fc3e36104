"""Peer-mapped buffers and the fused row-parallel collective (``ops/csrc/comm.cu``).

Every rank ``cudaMalloc``s one buffer ``[flags | normed out | residual | split-K partials]``,
exports its CUDA IPC handle, and maps every peer's buffer (exchange through ``torch.distributed``
at start-up only).  A row-parallel projection then runs as: sm_100a GEMM writing fp32 split-K
partials into this rank's buffer, followed by ``fused_allreduce_add_rmsnorm`` which reduces them
over NVLink, adds the residual, applies RMSNorm and all-gathers the rows into every rank's
buffers.  The outputs alias the buffers (they are valid until the next fused call), which also
makes the path CUDA-graph friendly.  Steps with more than ``max_tokens`` tokens (large prefills)
take the NCCL path; all ranks decide identically from the step shape.
"""
import logging

import torch
import torch.distributed as dist

from llmserve_b200.ops import gemm
from llmserve_b200.ops._ext import C, status
from llmserve_b200.parallel import state as tp

log = logging.getLogger(__name__)

FLAG_BYTES = 4096
MAX_SPLITS = 8


class FusedComm:

    def __init__(self, device, hidden: int, max_tokens: int, base: int, peers: list[int], opened: list[int]):
        self.device = device
        self.hidden = hidden
        self.max_tokens = max_tokens
        self.rank, self.world = tp.get_tp_rank(), tp.get_tp_size()
        self.base = base
        self.opened = opened
        out_bytes = max_tokens * hidden * 2
        self.flag_ptrs = list(peers)
        self.out_ptrs = [p + FLAG_BYTES for p in peers]
        self.res_ptrs = [p + FLAG_BYTES + out_bytes for p in peers]
        self.part_ptrs = [p + FLAG_BYTES + 2 * out_bytes for p in peers]
        # local views of the same memory
        nbytes = FLAG_BYTES + 2 * out_bytes + MAX_SPLITS * max_tokens * hidden * 4
        self._local = _wrap(base, nbytes, device)
        self.out_buf = self._local[FLAG_BYTES:FLAG_BYTES + out_bytes].view(torch.bfloat16)
        self.res_buf = self._local[FLAG_BYTES + out_bytes:FLAG_BYTES + 2 * out_bytes].view(torch.bfloat16)
        self.part_buf = self._local[FLAG_BYTES + 2 * out_bytes:].view(torch.float32)

    @staticmethod
    def buffer_bytes(hidden: int, max_tokens: int) -> int:
        return FLAG_BYTES + 2 * max_tokens * hidden * 2 + MAX_SPLITS * max_tokens * hidden * 4

    @classmethod
    def create(cls, device, hidden: int, max_tokens: int, timeout_s: float = 120.0):
        """Collective: returns a FusedComm on every rank, or None on every rank."""
        max_tokens = min(max_tokens, 512)
        base, opened, peers, ok = 0, [], [], 1
        try:
            base = C().comm_alloc(cls.buffer_bytes(hidden, max_tokens))
            handle = C().comm_ipc_handle(base)
        except Exception as e:  # pragma: no cover - depends on the box
            log.warning("fused collectives unavailable (%s); using NCCL", e)
            handle, ok = None, 0
        handles = [None] * tp.get_tp_size()
        dist.all_gather_object(handles, handle)
        if ok and all(h is not None for h in handles):
            try:
                for r, h in enumerate(handles):
                    if r == tp.get_tp_rank():
                        peers.append(base)
                    else:
                        p = C().comm_open_handle(h)
                        opened.append(p)
                        peers.append(p)
            except Exception as e:  # pragma: no cover
                log.warning("could not map peer buffers (%s); using NCCL", e)
                ok = 0
        else:
            ok = 0
        flag = torch.tensor([ok], device=device)
        dist.all_reduce(flag, op=dist.ReduceOp.MIN)
        if int(flag.item()) == 0:
            for p in opened:
                C().comm_close_handle(p)
            if base:
                C().comm_free(base)
            return None
        torch.cuda.synchronize(device)
        tp.barrier()
        return cls(device, hidden, max_tokens, base, peers, opened)

    def can_handle(self, T: int, N: int) -> bool:
        return 0 < T <= self.max_tokens and N == self.hidden

    def row_parallel_add_norm(self, x, weight, residual, norm_weight, eps):
        T, K = x.shape
        N = weight.shape[0]
        from llmserve_b200.parallel.fused import ROW_PARALLEL_MAX_SPLITS
        # plain K splits: every partial plane crosses NVLink, so the fewer the better here
        splits = min(gemm.splits_for(T, weight, streamk=False), ROW_PARALLEL_MAX_SPLITS, MAX_SPLITS)
        part = self.part_buf[: splits * T * N].view(splits, T, N)
        gemm.linear_partials(x, weight, splits, partials=part, streamk=False)
        C().fused_allreduce_add_rmsnorm(self.part_ptrs, self.out_ptrs, self.res_ptrs, self.flag_ptrs,
                                        residual.contiguous(), norm_weight, self.rank, splits, T, N, float(eps),
                                        status(x.device))
        return self.out_buf[: T * N].view(T, N), self.res_buf[: T * N].view(T, N)

    def close(self):
        torch.cuda.synchronize(self.device)
        for p in self.opened:
            C().comm_close_handle(p)
        self.opened = []
        if self.base:
            C().comm_free(self.base)
            self.base = 0


def _wrap(ptr: int, nbytes: int, device) -> torch.Tensor:
    """A uint8 tensor viewing raw device memory owned by this module (freed by ``close``)."""
    class _Holder:
        __cuda_array_interface__ = {"shape": (nbytes,), "typestr": "|u1", "data": (ptr, False), "version": 3,
                                    "strides": None}
    with torch.cuda.device(device):
        return torch.as_tensor(_Holder(), device=device)
