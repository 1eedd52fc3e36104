"""CUDA graphs of the batched greedy EAGLE3 step (draft x gamma -> packed verify -> accept).

The eager speculative step launches every kernel of gamma draft forwards and one verify forward
of ``B * (gamma + 1)`` tokens from the host, so at serving batch sizes it is bound by launch
overhead.  This module captures the device part of the step once per batch bucket:

* gamma draft decode steps over the paged draft pool, each followed by the draft's greedy pick
  (argmax + ``d2t``) fed straight into the next depth;
* the packed target verify of ``[start, drafts]`` per sequence (prefill attention over the paged
  target pool, all-token logits, per-row argmax);
* greedy acceptance (one kernel -> rows ``[accepted, final, start, drafts...]``) and the gather
  of each sequence's correction-token auxiliary hidden state.

Every per-step input lives in one packed int32 device buffer filled by a single host-to-device
copy from pinned memory: draft slots / context lengths / positions per depth, verify positions
and slots, key counts and block tables.  Start tokens and start auxiliary states are written
into static device buffers by the executor (the fresh ones come from the target decode, the
carried ones from the previous step's correction).  Padded rows of a bucket store nothing
(slot -1) and their results are ignored.

Scope: greedy acceptance, chain drafting (no tree), no per-step trace; every tensor-parallel
rank captures and replays its own graphs (the verify's vocab-parallel argmax is a collective
inside them, and the draft is replicated).  Other steps run eagerly.  It is opt-in (``Config.speculative_cuda_graphs``).  On the host tier
(``device="cpu"``) the same body runs eagerly over the same static buffers, which is how the
buffer layout and the step logic are tested without a GPU.
"""
import numpy as np
import torch

from llmserve_b200.ops import sampling as sampling_ops
from llmserve_b200.ops._ext import LaunchCounter
from llmserve_b200.speculative.sampling import greedy_accept_packed
from llmserve_b200.utils.context import reset_context, set_context

BUCKETS = (1, 2, 4, 8, 16, 32, 48, 64)


class SpeculativeGraphs:

    def __init__(self, executor, max_batch: int):
        r = executor.r
        self.ex, self.r = executor, r
        self.g = r.speculative_gamma
        self.n = self.g + 1
        self.buckets = [b for b in BUCKETS if b <= max_batch] or [max_batch]
        self.mb = self.buckets[-1]
        self.W = r.graph_W
        mb, g, n, d = self.mb, self.g, self.n, r.device
        # packed int32 inputs: draft slots / lengths / positions [g, mb] each, verify positions and
        # slots [mb * n] each, key counts [mb], block tables [mb, W]
        self.off_dslot, self.off_dlen, self.off_dpos = 0, g * mb, 2 * g * mb
        self.off_vpos = 3 * g * mb
        self.off_vslot = self.off_vpos + mb * n
        self.off_seqk = self.off_vslot + mb * n
        self.off_tables = self.off_seqk + mb
        size = self.off_tables + mb * self.W
        self.pack = torch.zeros(size, dtype=torch.int32, device=d)
        self.host = torch.zeros(size, dtype=torch.int32, pin_memory=r.is_cuda)
        self.host_np = self.host.numpy()
        width = r.draft_model.fc.weight.shape[1]
        self.ids = torch.zeros(mb, dtype=torch.int64, device=d)
        self.aux = torch.zeros(mb, width, dtype=r.dtype, device=d)
        self.drafts = torch.zeros(mb, g, dtype=torch.int64, device=d)
        self.packed = torch.zeros(mb, g + 3, dtype=torch.int64, device=d)
        self.corr_aux = torch.zeros(mb, width, dtype=r.dtype, device=d)
        self.cu_q = torch.arange(0, (mb + 1) * n, n, dtype=torch.int32, device=d)
        self.rows = torch.arange(mb, device=d)
        self.graphs, self.pool, self.launches = {}, None, {}
        self.steps = 0

    # ---- views of the packed inputs ----------------------------------------------------------
    def _view(self, off, count):
        return self.pack[off:off + count]

    def _inputs(self, B):
        mb, g, n = self.mb, self.g, self.n
        dslot = self._view(self.off_dslot, g * mb).view(g, mb)[:, :B]
        dlen = self._view(self.off_dlen, g * mb).view(g, mb)[:, :B]
        dpos = self._view(self.off_dpos, g * mb).view(g, mb)[:, :B]
        vpos = self._view(self.off_vpos, mb * n)[:B * n]
        vslot = self._view(self.off_vslot, mb * n)[:B * n]
        seqk = self._view(self.off_seqk, mb)[:B]
        tables = self._view(self.off_tables, mb * self.W).view(mb, self.W)[:B]
        return dslot, dlen, dpos, vpos, vslot, seqk, tables

    # ---- the captured step -------------------------------------------------------------------
    def body(self, B: int):
        r, g, n = self.r, self.g, self.n
        dslot, dlen, dpos, vpos, vslot, seqk, tables = self._inputs(B)
        cur_ids, cur_in = self.ids[:B], self.aux[:B]
        for depth in range(g):
            set_context(False, slot_mapping=dslot[depth], context_lens=dlen[depth], block_tables=tables,
                        decode_workspace=r.decode_workspace)
            try:
                hidden, logits = r.draft_model(cur_ids, cur_in, dpos[depth].long())
            finally:
                reset_context()
            nxt = r.draft_model.greedy_sample(logits)
            self.drafts[:B, depth] = nxt
            cur_ids, cur_in = nxt, hidden
        vin = torch.cat([self.ids[:B].unsqueeze(1), self.drafts[:B]], 1).reshape(-1)
        set_context(True, cu_seqlens_q=self.cu_q[:B + 1], max_seqlen_q=n, slot_mapping=vslot,
                    block_tables=tables, seqlens_k=seqk, uniform_q=n, decode_workspace=r.decode_workspace)
        try:
            hidden, aux = r.model.forward_with_eagle3_aux(vin, vpos.long())
            logits = r.model.compute_logits(hidden, all_tokens=True)
        finally:
            reset_context()
        vals, idx = sampling_ops.local_argmax(logits)
        # global greedy ids: the NVLink (value, index) exchange when the fused collectives are up
        # (capturable, no NCCL call), else NCCL all-gathers
        target = r._greedy_from_shards(vals, idx).view(B, n)
        self.packed[:B] = greedy_accept_packed(target, self.drafts[:B], self.ids[:B])
        self.corr_aux[:B] = aux.view(B, n, -1)[self.rows[:B], self.packed[:B, 0]]

    def capture(self):
        """One graph per bucket (largest first, sharing one memory pool)."""
        for B in reversed(self.buckets):
            self._fill_padding(0)
            self.pack.copy_(self.host)
            self.body(B)                                  # warm-up outside capture
            torch.cuda.synchronize()
            graph = torch.cuda.CUDAGraph()
            before = LaunchCounter.launches
            with torch.cuda.graph(graph, self.pool, stream=self.r.capture_stream()):
                self.body(B)
            self.launches[B] = LaunchCounter.launches - before
            if self.pool is None:
                self.pool = graph.pool()
            self.graphs[B] = graph
            torch.cuda.synchronize()

    # ---- one step ----------------------------------------------------------------------------
    def bucket(self, B: int) -> int | None:
        return next((b for b in self.buckets if b >= B), None)

    def fits(self, seqs) -> bool:
        return self.bucket(len(seqs)) is not None and max(len(s.block_table) for s in seqs) <= self.W

    def _fill_padding(self, start: int):
        """Rows ``start ..`` of every input: store nothing (slot -1), one key, block 0."""
        a, mb, g, n = self.host_np, self.mb, self.g, self.n
        for d in range(g):
            a[self.off_dslot + d * mb + start:self.off_dslot + (d + 1) * mb] = -1
            a[self.off_dlen + d * mb + start:self.off_dlen + (d + 1) * mb] = 1
            a[self.off_dpos + d * mb + start:self.off_dpos + (d + 1) * mb] = 0
        a[self.off_vpos + start * n:self.off_vpos + mb * n] = 0
        a[self.off_vslot + start * n:self.off_vslot + mb * n] = -1
        a[self.off_seqk + start:self.off_seqk + mb] = n
        a[self.off_tables + start * self.W:self.off_tables + mb * self.W] = 0

    def fill(self, seqs, kv0: list[int], base: list[int]):
        """Host metadata of one step: draft depth ``d`` of sequence ``i`` writes draft position
        ``kv0[i] + d``; the verify covers target positions ``base[i] .. base[i] + gamma``.  Built
        with whole-batch array operations (one pass over the sequences copies the block tables)."""
        a, mb, g, n, W, bsz = self.host_np, self.mb, self.g, self.n, self.W, self.r.block_size
        B = len(seqs)
        tables = a[self.off_tables:self.off_tables + mb * W].reshape(mb, W)
        for i, s in enumerate(seqs):
            t = s.block_table
            tables[i, :len(t)] = t
            tables[i, len(t):] = 0
        tb = tables[:B].astype(np.int64)
        dp = np.asarray(kv0, dtype=np.int64)[:, None] + np.arange(g)            # [B, g]
        dslot = np.take_along_axis(tb, dp // bsz, 1) * bsz + dp % bsz
        a[self.off_dslot:self.off_dslot + g * mb].reshape(g, mb)[:, :B] = dslot.T
        a[self.off_dlen:self.off_dlen + g * mb].reshape(g, mb)[:, :B] = (dp + 1).T
        a[self.off_dpos:self.off_dpos + g * mb].reshape(g, mb)[:, :B] = dp.T
        bs_ = np.asarray(base, dtype=np.int64)
        vp = bs_[:, None] + np.arange(n)                                         # [B, n]
        a[self.off_vpos:self.off_vpos + B * n] = vp.reshape(-1)
        a[self.off_vslot:self.off_vslot + B * n] = (np.take_along_axis(tb, vp // bsz, 1) * bsz + vp % bsz).reshape(-1)
        a[self.off_seqk:self.off_seqk + B] = bs_ + n
        self._fill_padding(B)
        if self.r.config.debug_bounds_checks:
            self._check(B)

    def _check(self, B):
        a, mb, n = self.host_np, self.mb, self.n
        cap = self.r.k_cache.shape[1] * self.r.block_size
        slots = np.concatenate([a[self.off_dslot + d * mb:self.off_dslot + d * mb + B] for d in range(self.g)]
                               + [a[self.off_vslot:self.off_vslot + B * n]])
        if slots.min() < 0 or slots.max() >= cap:
            raise RuntimeError(f"speculative graph step: slot out of range 0..{cap - 1}")

    def run(self, B: int) -> list[list[int]]:
        """Copy the staged inputs, replay (or run the body on the host tier) and return the accept
        rows ``[accepted, final, start, drafts...]`` of the first ``B`` sequences."""
        gb = self.bucket(B)
        r = self.r
        if r.is_cuda:
            self.pack.copy_(self.host, non_blocking=True)
            r.h2d_bytes += self.host.numel() * 4
            self.graphs[gb].replay()
            LaunchCounter.launches += self.launches[gb]
        else:
            self.pack.copy_(self.host)
            self.body(gb)
        self.steps += 1
        rows = self.packed[:B].tolist()
        r.d2h_bytes += 8 * B * (self.g + 3)
        return rows
