"""EAGLE3 speculative decoding on top of a :class:`ModelRunner`.

Algorithm parity with ``llmserve/engine/speculative_executor.py`` of the reference:

* draft prefill pairs token ``x_{p+1}`` with target hidden ``h_p`` (``:60-75``), including the
  first sampled token at the last prompt position (``:148-185``);
* a *merged* step reuses the previous correction/bonus token -- appended to the sequence but
  without target KV yet -- as the start token and verifies from ``len(seq) - 1``
  (``:542-553``, ``:742-778``);
* batched chain drafting, one packed target verify, greedy or rejection acceptance, then the
  draft KV keeps ``old_len + min(accepted + 1, gamma)`` entries (``:121-146``);
* the fixed-tree variant for single sequences (``:437-540``).

Design differences: the draft's K/V live in a paged pool addressed by the target's block
tables, so "trimming" the draft KV is just a length update and the batched draft is a plain
paged decode; draft prefill runs chunk by chunk alongside the target's (chunked) prefill;
greedy acceptance is computed on the device for the whole batch with one host copy; the target
verify logits are vocab-parallel, so speculation also runs with tensor parallelism (the
reference requires ``world_size == 1``, ``llm_engine.py:366-367``).
"""
import os
from time import perf_counter

import torch

from llmserve_b200.models.eagle3 import Eagle3Speculator
from llmserve_b200.ops import kv as kv_ops
from llmserve_b200.ops import sampling as sampling_ops
from llmserve_b200.parallel import state as tp
from llmserve_b200.speculative.sampling import greedy_accept_packed, speculative_accept_reject_from_logits
from llmserve_b200.speculative.tree import build_fixed_tree_topology, select_greedy_tree_path
from llmserve_b200.speculative.tree_kv import TreeKVCacheManager
from llmserve_b200.speculative.types import SpeculativeDecodeOutput
from llmserve_b200.utils.context import reset_context, set_context
from llmserve_b200.utils.loader import seed_for
from llmserve_b200.utils.nvtx import nvtx_range


def _mask_bits(mask: torch.Tensor) -> torch.Tensor:
    weights = 1 << torch.arange(mask.shape[1], dtype=torch.int64, device=mask.device)
    return (mask.long() * weights).sum(1).to(torch.int32)


class SpeculativeExecutor:

    def __init__(self, runner):
        self.r = runner
        self.draft_kv_len: dict[int, int] = {}
        self.prev_correction: dict[int, tuple[int, torch.Tensor]] = {}
        self.graphs = None          # SpeculativeGraphs when Config.speculative_cuda_graphs applies

    # ---- set-up ------------------------------------------------------------------------------
    def load_draft_model(self):
        r = self.r
        cfg = r.config
        if cfg.speculative_model is None:
            return None
        path = cfg.speculative_model
        target_emb = r.model.model.embed_tokens.weight
        if any(n.endswith(".safetensors") for n in os.listdir(path)):
            draft = Eagle3Speculator.from_pretrained(
                path, target_model_path=cfg.model if cfg.load_format == "auto" else None,
                target_embedding=target_emb)
        else:
            draft = Eagle3Speculator(Eagle3Speculator.read_config(path))
            draft.embed_tokens.weight = target_emb
            self._random_init_draft(draft, cfg.seed)
        draft = draft.to(device=r.device, dtype=r.dtype)
        draft.eval()
        draft.prepare()
        return draft

    @staticmethod
    @torch.no_grad()
    def _random_init_draft(draft, seed: int):
        for name, p in draft.named_parameters():
            if name == "embed_tokens.weight":
                continue
            g = torch.Generator().manual_seed(seed_for("draft." + name, seed))
            if name.endswith("norm.weight"):
                p.data.fill_(1.0)
            else:
                p.data.copy_(torch.randn(p.shape, generator=g) * 0.02)
        g = torch.Generator().manual_seed(seed + 17)
        ids = torch.randperm(draft.target_vocab_size, generator=g)[:draft.draft_vocab_size].sort().values
        draft.d2t.copy_(ids - torch.arange(draft.draft_vocab_size))
        draft.t2d.zero_()
        draft.t2d[ids] = True

    def setup_graphs(self):
        """Graphs (host tier: static-buffer emulation) of the greedy chain step, when enabled and
        in scope: greedy acceptance, no tree.  Every rank captures its own (same order)."""
        r = self.r
        cfg = r.config
        if (not getattr(cfg, "speculative_cuda_graphs", False) or r.draft_model is None
                or r.speculative_accept_mode != "greedy" or r.speculative_tree_nodes
                or (r.is_cuda and r.enforce_eager)):
            return
        from llmserve_b200.engine.speculative_graphs import SpeculativeGraphs
        graphs = SpeculativeGraphs(self, min(cfg.max_num_seqs, 64))
        if r.is_cuda:
            graphs.capture()
        self.graphs = graphs

    def clear_all(self):
        self.draft_kv_len.clear()
        self.prev_correction.clear()

    def clear_speculative_state(self, seq_ids):
        for sid in seq_ids:
            self.draft_kv_len.pop(sid, None)
            self.prev_correction.pop(sid, None)

    def note_plain_step(self, decode_seqs):
        """A plain decode writes the pending correction token's target KV itself."""
        for s in decode_seqs:
            self.prev_correction.pop(s.seq_id, None)

    # ---- draft helpers -----------------------------------------------------------------------
    def _draft_decode(self, seqs, ids, inputs, positions: list[int]):
        r = self.r
        d = r.device
        set_context(False, slot_mapping=torch.tensor([s.slot(p) for s, p in zip(seqs, positions)],
                                                     dtype=torch.int32, device=d),
                    context_lens=torch.tensor([p + 1 for p in positions], dtype=torch.int32, device=d),
                    block_tables=r.prepare_block_tables(seqs), decode_workspace=r.decode_workspace)
        try:
            return r.draft_model(ids, inputs, torch.tensor(positions, dtype=torch.int64, device=d))
        finally:
            reset_context()

    @torch.inference_mode()
    def after_prefill(self, seqs, decode_seqs, aux, token_list):
        """Feed the draft the chunk that the target just prefilled (draft prefill)."""
        r = self.r
        decode_ids = {s.seq_id for s in decode_seqs}
        rows, ids, pos, slots = [], [], [], []
        cu_q, lens_k, members = [0], [], []
        offset = 0
        for i, s in enumerate(seqs):
            if s.seq_id in decode_ids:
                offset += 1
                continue
            start = min(s.num_cached_tokens, len(s) - 1)
            q = s.num_scheduled_tokens
            count = 0
            for p in range(start, start + q):
                if p + 1 < len(s):
                    tok = s.token_ids[p + 1]
                elif s.num_completion_tokens == 0:
                    tok = token_list[i]
                else:
                    break
                rows.append(offset + p - start)
                ids.append(tok)
                pos.append(p)
                slots.append(s.slot(p))
                count += 1
            offset += q
            if count:
                members.append(s)
                cu_q.append(cu_q[-1] + count)
                lens_k.append(start + count)
                self.draft_kv_len[s.seq_id] = start + count
        if not members:
            return
        d = r.device
        set_context(True, cu_seqlens_q=torch.tensor(cu_q, dtype=torch.int32, device=d),
                    max_seqlen_q=max(b - a for a, b in zip(cu_q, cu_q[1:])), max_seqlen_k=max(lens_k),
                    slot_mapping=torch.tensor(slots, dtype=torch.int32, device=d),
                    block_tables=r.prepare_block_tables(members),
                    seqlens_k=torch.tensor(lens_k, dtype=torch.int32, device=d))
        try:
            r.draft_model(torch.tensor(ids, dtype=torch.int64, device=d),
                          aux.index_select(0, torch.tensor(rows, dtype=torch.int64, device=d)),
                          torch.tensor(pos, dtype=torch.int64, device=d))
        finally:
            reset_context()

    def _target_decode_with_aux(self, seqs):
        r = self.r
        ids, pos = r.prepare_decode(seqs)
        temps = r.prepare_sample(seqs)
        try:
            hidden, aux = r.model.forward_with_eagle3_aux(ids, pos)
            logits = r.model.compute_logits(hidden)
        finally:
            reset_context()
        return r.sample_tokens(logits, temps), aux

    def _target_ids(self, logits):
        vals, idx = sampling_ops.local_argmax(logits)
        return tp.vocab_parallel_argmax(vals, idx, self.r.model.lm_head.vocab_start)

    # ---- chain speculation (batched) ---------------------------------------------------------
    @torch.inference_mode()
    def run_speculative_batch(self, seqs) -> list[SpeculativeDecodeOutput]:
        r = self.r
        if r.draft_model is None:
            raise RuntimeError("no draft model loaded")
        if not seqs:
            return []
        t_total = perf_counter()
        B, g, dev = len(seqs), r.speculative_gamma, r.device
        greedy = r.speculative_accept_mode == "greedy"
        merged = [s.seq_id in self.prev_correction for s in seqs]
        start_ids = torch.empty(B, dtype=torch.int64, device=dev)
        start_aux = torch.empty(B, r.draft_model.fc.weight.shape[1], dtype=r.dtype, device=dev)

        t = perf_counter()
        fresh = [i for i in range(B) if not merged[i]]
        if fresh:
            toks, aux = self._target_decode_with_aux([seqs[i] for i in fresh])
            sel = torch.tensor(fresh, dtype=torch.int64, device=dev)
            start_ids[sel] = toks
            start_aux[sel] = aux
        carried = [i for i in range(B) if merged[i]]
        if carried:
            # one gather for every carried correction token and aux row (not two copies per sequence)
            prev = [self.prev_correction[seqs[i].seq_id] for i in carried]
            sel = torch.tensor(carried, dtype=torch.int64, device=dev)
            start_ids[sel] = torch.tensor([p[0] for p in prev], dtype=torch.int64, device=dev)
            start_aux[sel] = torch.stack([p[1] for p in prev]).to(start_aux.dtype)
        target_decode_time = perf_counter() - t

        kv0 = [self.draft_kv_len.get(s.seq_id, len(s)) for s in seqs]
        base = [len(s) - (1 if m else 0) for s, m in zip(seqs, merged)]
        sg = self.graphs
        if sg is not None and greedy and not r.speculative_trace and sg.fits(seqs):
            t = perf_counter()
            sg.ids[:B].copy_(start_ids)
            sg.aux[:B].copy_(start_aux)
            sg.fill(seqs, kv0, base)
            with nvtx_range("speculative.graph"):
                host = sg.run(B)
            graph_time = perf_counter() - t
            accepts = [(row[0], row[1], row[3:], row[0] == g) for row in host]
            starts = [row[2] for row in host]
            timing = {"target_decode_time": target_decode_time, "fresh": len(fresh), "draft_time": 0.0,
                      "verify_time": graph_time, "accept_time": 0.0, "fwd_time": 0.0, "sample_time": 0.0}
            return self._finish(seqs, merged, accepts, starts, sg.corr_aux[:B].clone(), kv0, None,
                                verify_width=g + 1, timing=timing, t_total=t_total)
        t = perf_counter()
        draft_tokens = torch.empty(B, g, dtype=torch.int64, device=dev)
        mapped_logits = []
        cur_ids, cur_in = start_ids, start_aux
        fwd_time = sample_time = 0.0
        temps = torch.tensor([s.temperature for s in seqs], device=dev).unsqueeze(1)
        for depth in range(g):
            ts = perf_counter()
            with nvtx_range(f"draft.{depth}"):
                hidden, logits = self._draft_decode(seqs, cur_ids, cur_in, [k + depth for k in kv0])
            fwd_time += perf_counter() - ts
            ts = perf_counter()
            if greedy:
                nxt = r.draft_model.greedy_sample(logits)
            else:
                mapped = r.draft_model.map_draft_logits(logits.float())
                mapped_logits.append(mapped)
                nxt = torch.multinomial(torch.softmax(mapped / temps, -1), 1).squeeze(1)
                nxt = tp.broadcast(nxt.contiguous(), 0)
            sample_time += perf_counter() - ts
            draft_tokens[:, depth] = nxt
            cur_ids, cur_in = nxt, hidden
        draft_time = perf_counter() - t

        t = perf_counter()
        n = g + 1
        vin = torch.cat([start_ids.unsqueeze(1), draft_tokens], 1).reshape(-1)
        vpos = torch.tensor([b + j for b in base for j in range(n)], dtype=torch.int64, device=dev)
        vslots = torch.tensor([s.slot(b + j) for s, b in zip(seqs, base) for j in range(n)],
                              dtype=torch.int32, device=dev)
        set_context(True, cu_seqlens_q=torch.arange(0, (B + 1) * n, n, dtype=torch.int32, device=dev),
                    max_seqlen_q=n, max_seqlen_k=max(base) + n, slot_mapping=vslots,
                    block_tables=r.prepare_block_tables(seqs),
                    seqlens_k=torch.tensor([b + n for b in base], dtype=torch.int32, device=dev),
                    uniform_q=n, decode_workspace=r.decode_workspace)
        try:
            with nvtx_range("verify"):
                hidden, aux = r.model.forward_with_eagle3_aux(vin, vpos)
                logits = r.model.compute_logits(hidden, all_tokens=True)
        finally:
            reset_context()
        verify_time = perf_counter() - t

        t = perf_counter()
        if greedy:
            target_ids = self._target_ids(logits).view(B, n)
            packed = greedy_accept_packed(target_ids, draft_tokens, start_ids)
            num_acc = packed[:, 0]
            host = packed.tolist()
            r.d2h_bytes += 8 * B * (g + 3)
            accepts = [(row[0], row[1], row[3:], row[0] == g) for row in host]
            starts = [row[2] for row in host]
        else:
            full = tp.gather_logits(logits).view(B, n, -1)
            drafts = draft_tokens.tolist()
            starts = start_ids.tolist()
            accepts = []
            for i, s in enumerate(seqs):
                dl = torch.stack([mapped_logits[d][i] for d in range(g)], 0)
                res = speculative_accept_reject_from_logits(full[i], dl, torch.tensor(drafts[i]), s.temperature)
                accepts.append((res.num_accepted, res.final_token_id, drafts[i], res.accepted_all))
            if r.world_size > 1:
                flat = torch.tensor([[a[0], a[1]] for a in accepts], dtype=torch.int64, device=dev)
                tp.broadcast(flat, 0)
                accepts = [(int(x[0]), int(x[1]), accepts[i][2], int(x[0]) == g) for i, x in enumerate(flat.tolist())]
            num_acc = torch.tensor([a[0] for a in accepts], device=dev)
        corr_aux = aux.view(B, n, -1)[torch.arange(B, device=dev), num_acc.long()]
        accept_time = perf_counter() - t
        timing = {"target_decode_time": target_decode_time, "fresh": len(fresh), "draft_time": draft_time,
                  "verify_time": verify_time, "accept_time": accept_time, "fwd_time": fwd_time,
                  "sample_time": sample_time}
        return self._finish(seqs, merged, accepts, starts, corr_aux, kv0, logits, verify_width=n, timing=timing,
                            t_total=t_total)

    def _finish(self, seqs, merged, accepts, starts, corr_aux, kv0, logits, *, verify_width, timing, t_total):
        """Per-sequence outputs of a chain step and the state the next step starts from: the
        correction token with its auxiliary hidden state, and the kept draft K/V length."""
        r = self.r
        B, g = len(seqs), r.speculative_gamma
        t = perf_counter()
        outputs = []
        for i, s in enumerate(seqs):
            acc, fin, drafts, all_ok = accepts[i]
            tokens = ([] if merged[i] else [starts[i]]) + list(drafts[:acc]) + [fin]
            self.prev_correction[s.seq_id] = (fin, corr_aux[i])
            self.draft_kv_len[s.seq_id] = kv0[i] + min(acc + 1, g)
            debug = None
            if r.speculative_trace and logits is not None:
                debug = self._debug(logits, i, verify_width, starts[i], list(drafts), tokens, acc, all_ok, kv0[i])
            outputs.append(SpeculativeDecodeOutput(tokens, g, acc, bool(all_ok), len(tokens), None, debug))
        kv_time = perf_counter() - t
        total = perf_counter() - t_total
        fresh = timing["fresh"]
        for i, o in enumerate(outputs):
            o.timing = {
                "target_decode_time": (timing["target_decode_time"] / fresh) if not merged[i] else 0.0,
                "draft_proposal_time": timing["draft_time"] / B,
                "target_verify_time": timing["verify_time"] / B,
                "accept_time": timing["accept_time"] / B,
                "kv_update_time": kv_time / B,
                "trace_time": 0.0,
                "total_time": total / B,
                "draft_pack_time": 0.0,
                "draft_forward_time": timing["fwd_time"] / B,
                "draft_sample_time": timing["sample_time"] / B,
                "draft_compact_time": 0.0,
            }
        return outputs

    def _debug(self, logits, i, n, start, drafts, emitted, acc, all_ok, kv_len):
        full = tp.gather_logits(logits).float()
        full = full.view(-1, n, full.shape[-1])[i]
        target_argmax = full.argmax(-1).tolist()
        ranks, vals = [], []
        for j, tok in enumerate(drafts):
            v = full[j, tok]
            ranks.append(int((full[j] > v).sum()) + 1)
            vals.append(float(v))
        top = torch.topk(full, k=min(5, full.shape[1]), dim=-1)
        return {
            "accept_mode": self.r.speculative_accept_mode, "start_token_id": int(start),
            "draft_token_ids": [int(x) for x in drafts], "target_argmax_token_ids": target_argmax,
            "matches": [target_argmax[j] == drafts[j] for j in range(len(drafts))],
            "num_accepted": int(acc), "accepted_all": bool(all_ok), "emitted_token_ids": emitted,
            "draft_kv_len_before": int(kv_len), "draft_token_target_ranks": ranks,
            "draft_token_target_logits": vals, "target_top_token_ids": top.indices.tolist(),
            "target_top_logits": top.values.tolist(),
        }

    # ---- tree speculation (single sequence) ----------------------------------------------------
    @torch.inference_mode()
    def run_speculative_tree_single(self, seq) -> SpeculativeDecodeOutput:
        r = self.r
        if r.speculative_tree_nodes not in (6, 10) or r.speculative_accept_mode != "greedy":
            raise RuntimeError("tree speculation needs 6 or 10 nodes and greedy acceptance")
        t_total = perf_counter()
        dev, draft = r.device, r.draft_model
        merged = seq.seq_id in self.prev_correction
        t = perf_counter()
        if merged:
            start, start_aux = self.prev_correction[seq.seq_id]
            start = int(start)
        else:
            toks, aux = self._target_decode_with_aux([seq])
            start, start_aux = int(toks[0]), aux[0]
        target_decode_time = perf_counter() - t
        kv0 = self.draft_kv_len.get(seq.seq_id, len(seq))
        topo = build_fixed_tree_topology(r.speculative_tree_nodes)
        n_nodes = len(topo.parents)
        depths = topo.depths
        mask = topo.attention_mask(dev)
        bits = _mask_bits(mask)
        table = torch.tensor(seq.block_table, dtype=torch.int32, device=dev)

        t = perf_counter()
        tokens = [start] + [0] * (n_nodes - 1)
        inputs = {0: start_aux}
        side_k = torch.zeros(n_nodes, draft.num_kv_heads, draft.head_dim, dtype=r.dtype, device=dev)
        side_v = torch.zeros_like(side_k)
        processed = set()
        for depth in range(max(depths)):
            active = [i for i in range(n_nodes) if depths[i] == depth and topo.children(i)]
            ids = torch.tensor([tokens[i] for i in active], dtype=torch.int64, device=dev)
            x = torch.stack([inputs[i] for i in active], 0)
            set_context(True, tree_attention_mask=mask[active], tree_prefix_len=kv0, tree_block_table=table,
                        tree_mask_bits=bits[active], tree_rows=active, tree_side_k=side_k, tree_side_v=side_v)
            try:
                hidden, logits = draft(ids, x, torch.full((len(active),), kv0 + depth, dtype=torch.int64, device=dev))
            finally:
                reset_context()
            processed.update(active)
            for j, a in enumerate(active):
                kids = topo.children(a)
                picks = draft.greedy_topk(logits[j:j + 1], len(kids)).flatten().tolist()
                for c, tok in zip(kids, picks):
                    tokens[c] = int(tok)
                    inputs[c] = hidden[j]
        draft_time = perf_counter() - t

        t = perf_counter()
        base = len(seq) - (1 if merged else 0)
        set_context(True, tree_attention_mask=mask, tree_prefix_len=base, tree_block_table=table,
                    tree_mask_bits=bits)
        try:
            hidden, aux = r.model.forward_with_eagle3_aux(
                torch.tensor(tokens, dtype=torch.int64, device=dev),
                torch.tensor([base + dd for dd in depths], dtype=torch.int64, device=dev))
            logits = r.model.compute_logits(hidden, all_tokens=True)
        finally:
            reset_context()
        verify_time = perf_counter() - t

        t = perf_counter()
        res = select_greedy_tree_path(topo, tokens[1:], self._target_ids(logits).tolist())
        emitted = ([] if merged else [start]) + res.token_ids
        self.prev_correction[seq.seq_id] = (res.final_token_id, aux[res.final_node_index].clone())
        accept_time = perf_counter() - t

        t = perf_counter()
        manager = TreeKVCacheManager([layer.self_attn.attn for layer in r.model.model.layers],
                                     k_cache=r.k_cache, v_cache=r.v_cache)
        commit = [int(i) for i in res.commit_node_indices]
        slots = torch.tensor([seq.slot(base + j) for j in range(len(commit))], dtype=torch.int32, device=dev)
        manager.commit(commit, slots)
        commit_time = perf_counter() - t

        t = perf_counter()
        node = res.accepted_node_indices[-1] if res.accepted_node_indices else 0
        while node not in processed:
            node = topo.parents[node]
        chain = list(reversed(topo.ancestors_and_self(node)))
        keep = min(res.num_accepted + 1, r.speculative_gamma, len(chain))
        dslots = torch.tensor([seq.slot(kv0 + j) for j in range(keep)], dtype=torch.int32, device=dev)
        kv_ops.commit_tree_kv(side_k.unsqueeze(0), side_v.unsqueeze(0), r.draft_k_cache.unsqueeze(0),
                              r.draft_v_cache.unsqueeze(0), torch.tensor(chain[:keep], dtype=torch.int32, device=dev),
                              dslots)
        self.draft_kv_len[seq.seq_id] = kv0 + keep
        draft_kv_time = perf_counter() - t
        timing = {
            "target_decode_time": target_decode_time, "draft_proposal_time": draft_time,
            "target_verify_time": verify_time, "accept_time": accept_time,
            "kv_update_time": commit_time + draft_kv_time, "target_tree_kv_commit_time": commit_time,
            "draft_kv_update_time": draft_kv_time, "trace_time": 0.0, "total_time": perf_counter() - t_total,
        }
        return SpeculativeDecodeOutput(emitted, topo.num_draft_nodes, res.num_accepted, res.accepted_all,
                                       len(emitted), timing)
