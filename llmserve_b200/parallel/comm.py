"""Peer-mapped buffers and the fused row-parallel collective (``ops/csrc/comm.cu``).

Every rank ``cudaMalloc``s one buffer ``[control | out | residual | all-gather inbox | reduce
inbox]``, exports its CUDA IPC handle, and maps every peer's buffer (handles exchanged through
``torch.distributed`` at start-up only).  A row-parallel projection then runs as two kernels:

* the sm_100a GEMM (dense or W4A16) whose epilogue stores the fp32 split-K partials of each token
  row straight into the reduce inbox of the rank that owns the row (peer stores over NVLink), each
  value in a 64-bit word tagged with the call's epoch;
* ``row_parallel_finish``: for the rows this rank owns, poll the inbox until every word carries the
  epoch, reduce, add the residual, RMSNorm, and store the finished (out, residual) pairs into every
  peer's all-gather inbox (again epoch-tagged words); for the other rows, poll the all-gather inbox
  and unpack.  No fence, flag or barrier round: a word with the expected epoch carries its data.

The outputs alias the buffers (valid until the next fused call), which also makes the path
CUDA-graph friendly.  The control block also carries the greedy vocab-parallel argmax exchange
(``argmax``), so a decode step's sampling needs no NCCL call either.  Steps with more than
``max_tokens`` tokens (large prefills) take the NCCL path; all ranks decide identically from the
step shape.
"""
import logging

import torch
import torch.distributed as dist

from llmserve_b200.ops import gemm
from llmserve_b200.ops._ext import C, status
from llmserve_b200.parallel import state as tp

log = logging.getLogger(__name__)

CTRL_BYTES = 1 << 17          # flag words + argmax slots (ops/csrc/comm.cu), rounded up
MAX_SPLITS = 8


def _rows_per_rank(T: int, world: int) -> int:
    return max(1, -(-T // world))


class FusedComm:

    def __init__(self, device, hidden: int, max_tokens: int, base: int, peers: list[int], opened: list[int]):
        self.device = device
        self.hidden = hidden
        self.max_tokens = max_tokens
        self.rank, self.world = tp.get_tp_rank(), tp.get_tp_size()
        self.base = base
        self.opened = opened
        self.ctrl_ptrs = list(peers)
        off = self.offsets(hidden, max_tokens, self.world)
        self.ag_ptrs = [p + off["ag"] for p in peers]
        self.inbox_ptrs = [p + off["inbox"] for p in peers]
        self.epoch_ptr = base                      # this rank's epoch word (control word 0)
        self._local = _wrap(base, off["total"], device)
        out_bytes = max_tokens * hidden * 2
        self.out_ptr, self.res_ptr = base + off["out"], base + off["res"]
        self.out_buf = self._local[off["out"]:off["out"] + out_bytes].view(torch.bfloat16)
        self.res_buf = self._local[off["res"]:off["res"] + out_bytes].view(torch.bfloat16)

    @staticmethod
    def offsets(hidden: int, max_tokens: int, world: int) -> dict:
        """Byte offsets of the regions of one rank's buffer (see ``ops/csrc/comm.cu``)."""
        out_bytes = max_tokens * hidden * 2
        ag_bytes = max_tokens * hidden * 8
        inbox_bytes = world * MAX_SPLITS * _rows_per_rank(max_tokens, world) * hidden * 8
        out = CTRL_BYTES
        res = out + out_bytes
        ag = res + out_bytes
        inbox = ag + ag_bytes
        return {"out": out, "res": res, "ag": ag, "inbox": inbox, "total": inbox + inbox_bytes}

    @staticmethod
    def buffer_bytes(hidden: int, max_tokens: int, world: int) -> int:
        return FusedComm.offsets(hidden, max_tokens, world)["total"]

    @classmethod
    def create(cls, device, hidden: int, max_tokens: int, timeout_s: float = 120.0):
        """Collective: returns a FusedComm on every rank, or None on every rank."""
        max_tokens = min(max_tokens, 512)
        base, opened, peers, ok = 0, [], [], 1
        try:
            assert C().comm_control_bytes() <= CTRL_BYTES
            base = C().comm_alloc(cls.buffer_bytes(hidden, max_tokens, tp.get_tp_size()))
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
        from llmserve_b200.ops import awq as awq_ops
        from llmserve_b200.parallel.fused import ROW_PARALLEL_MAX_SPLITS
        T, K = x.shape
        rows = _rows_per_rank(T, self.world)
        st = status(x.device)
        if isinstance(weight, awq_ops.AWQPacked):
            # W4A16
            splits = min(gemm.splits_for(T, weight), ROW_PARALLEL_MAX_SPLITS, MAX_SPLITS)
            # decode-sized: the K splits reduce in a cluster and one plane crosses NVLink
            reduce = awq_ops.AWQ_CLUSTER and splits > 1 and T <= 128
            planes = 1 if reduce else splits
            C().awq_gemm_to_owners(x, weight.qtiles, weight.sztiles, weight.n, self.inbox_ptrs, self.rank, rows,
                                   splits, reduce, self.epoch_ptr, st)
        else:
            # dense: the K splits reduce on chip, one fp32 plane per rank crosses NVLink
            data, n, packed = gemm._operand(weight)
            reduce = gemm.use_cluster(T, weight)
            splits = (gemm.cluster_splits(T, n, K) if reduce
                      else min(gemm.splits_for(T, weight), ROW_PARALLEL_MAX_SPLITS, MAX_SPLITS))
            planes = 1 if reduce else splits
            C().gemm_bf16_to_owners(x, data, n, packed, self.inbox_ptrs, self.rank, rows, splits, reduce,
                                    self.epoch_ptr, st, gemm.stages_for_tokens(T))
        return self.finish(residual, norm_weight, eps, T, planes)

    def finish(self, residual, norm_weight, eps, T: int, planes: int, phases: int = 3):
        """The collective half alone: reduce this rank's rows from its inbox (``planes`` planes per
        source rank), add the residual, RMSNorm, push the rows to every rank, receive the others;
        outputs alias the buffers."""
        N = self.hidden
        C().row_parallel_finish(self.ag_ptrs, self.inbox_ptrs[self.rank], self.ctrl_ptrs[self.rank], self.out_ptr,
                                self.res_ptr, residual.contiguous(), norm_weight, self.rank, planes, T, N,
                                _rows_per_rank(T, self.world), float(eps), phases, status(residual.device))
        return self.out_buf[: T * N].view(T, N), self.res_buf[: T * N].view(T, N)

    def argmax(self, values: torch.Tensor, indices: torch.Tensor, shard_offset: int, out: torch.Tensor):
        """Greedy token ids ``out[int64 rows]`` from every rank's per-shard (max value, local index),
        exchanged through the control blocks (one kernel, capturable; ties -> lowest global id)."""
        C().vocab_argmax_exchange(self.ctrl_ptrs, values, indices, int(shard_offset), out, self.rank,
                                  status(values.device))
        return out

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
