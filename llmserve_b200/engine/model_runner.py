"""Per-rank executor: model, KV pools, step metadata, CUDA graphs, sampling.

Reference: ``llmserve/engine/model_runner.py`` (init ``:30-74``, RPC ``:87-115``, warm-up and KV
sizing ``:186-229``, metadata ``:258-338``, graphs ``:383-418``).  Differences by design:

* KV pools are ``k/v_cache[L, blocks, kv_heads, block_size, head_dim]`` (see ``ops.attention``)
  plus an EAGLE3 draft pool with the same block ids;
* prefill metadata carries per-sequence key lengths for the paged varlen kernel and the LM-head
  row selection; every prefill reads K/V from the pool (one kernel path for plain, chunked,
  prefix-cached and verify batches);
* greedy sampling is vocab-parallel (per-shard max/index, then a 12-byte-per-row exchange); other
  samplers receive full logits on every rank and rank 0's choice is broadcast;
* the sampler set on rank 0 (``runner.sampler = ...``, as the benchmarks do) is mirrored to the
  workers through the RPC channel;
* decode CUDA graphs also hold the LM head, so one replay yields the logit shard.
"""
import dataclasses
import os
import time

import numpy as np
import torch

from llmserve_b200.config import Config
from llmserve_b200.engine.rpc import RpcChannel, RpcTimeout
from llmserve_b200.engine.scheduler import SchedulerOutput
from llmserve_b200.engine.sequence import Sequence
from llmserve_b200.models.qwen3 import Qwen3ForCausalLM
from llmserve_b200.ops import attention as attn_ops
from llmserve_b200.ops import sampling as sampling_ops
from llmserve_b200.ops._ext import LaunchCounter
from llmserve_b200.parallel import state as tp
from llmserve_b200.utils.context import reset_context, set_context
from llmserve_b200.utils.loader import init_dummy_weights, load_model


class Sampler:
    """Temperature sampling by exponential race (``llmserve/layers/sampler.py``)."""
    is_greedy = False

    def __init__(self, seed: int = 0):
        self.seed = seed
        self.calls = 0

    def __call__(self, logits: torch.Tensor, temperatures: torch.Tensor) -> torch.Tensor:
        self.calls += 1
        return sampling_ops.sample(logits, temperatures, self.seed * 1000003 + self.calls)


class GreedySampler:
    """Argmax sampler; on a tensor-parallel runner it never gathers full logits."""
    is_greedy = True

    def __call__(self, logits: torch.Tensor, temperatures: torch.Tensor) -> torch.Tensor:
        return sampling_ops.argmax(logits)


def _to_device(values, dtype, device) -> torch.Tensor:
    t = torch.as_tensor(values, dtype=dtype)
    if device.type == "cuda":
        return t.pin_memory().to(device, non_blocking=True)
    return t


class ModelRunner:
    _graph_exchanges_argmax = False

    def __init__(self, config: Config, rank: int, channel_name: str | None = None, parent_pid: int | None = None):
        self.config = config
        hf = config.hf_config
        self.hf_config = hf
        self.block_size = config.kvcache_block_size
        Sequence.block_size = config.kvcache_block_size
        self.enforce_eager = config.enforce_eager
        self.world_size = config.tensor_parallel_size
        self.rank = rank
        self.step_profile = {} if os.environ.get("LLMSERVE_STEP_PROFILE") == "1" else None
        self.is_cuda = config.device == "cuda"
        if self.is_cuda:
            self.device = torch.device("cuda", config.device_offset + rank)
            torch.cuda.set_device(self.device)
        else:
            self.device = torch.device("cpu")
            if self.world_size > 1:
                # CPU tier: split the cores between ranks instead of oversubscribing them
                torch.set_num_threads(max(1, (os.cpu_count() or 1) // self.world_size))
        tp.init_tensor_parallel(rank, self.world_size, config.distributed_init_method, self.device,
                                config.comm_timeout_s)
        self.dtype = hf.dtype if self.is_cuda else torch.float32
        self.channel = None
        self.h2d_bytes = 0
        self.d2h_bytes = 0

        quant_config = config.quant_config
        if quant_config is not None and not self.is_cuda:
            # the fp32 host path dequantises AWQ weights with fp32 scales (loaded from bf16)
            quant_config = dataclasses.replace(quant_config, activation_dtype=self.dtype)
        prev_dtype = torch.get_default_dtype()
        torch.set_default_dtype(self.dtype)
        with torch.device(self.device):
            self.model = Qwen3ForCausalLM(hf, quant_config=quant_config)
        torch.set_default_dtype(prev_dtype)
        if config.load_format == "dummy":
            init_dummy_weights(self.model, seed=config.seed)
        else:
            load_model(self.model, config.model)
        self.model.eval()

        self._sampler = Sampler(config.seed)
        from llmserve_b200.engine.speculative_executor import SpeculativeExecutor
        self.spec = SpeculativeExecutor(self)
        self.draft_model = self.spec.load_draft_model()
        self.speculative_gamma = config.speculative_gamma
        self.speculative_tree_nodes = config.speculative_tree_nodes
        self.speculative_accept_mode = config.speculative_accept_mode
        self.speculative_trace = config.speculative_trace

        if self.is_cuda and self.world_size > 1 and config.fused_collectives:
            from llmserve_b200.parallel.comm import FusedComm
            tp.set_fused_comm(FusedComm.create(self.device, hf.hidden_size, max(config.max_num_seqs, 64)
                                               * (config.speculative_gamma + 1 if config.speculative_model else 1),
                                               timeout_s=config.comm_timeout_s))

        self.graphs = {}
        self.graph_pool = None
        self.decode_workspace = None
        # decode step staging: [ids | positions | slots | lengths | feed rows | block tables]
        self.pack_max_bs = min(config.max_num_seqs, 512)
        self.graph_W = -(-(config.max_model_len + config.speculative_gamma + 2) // self.block_size)
        n = self.pack_max_bs * (5 + self.graph_W)
        self.graph_pack_nps = [np.zeros(n, dtype=np.int32) for _ in range(2)]
        self.graph_pack_hosts = [None, None]
        self.graph_pack_turn = 0
        self.inflight_bs = 0
        self.warmup_model()
        self.allocate_kv_cache()
        if self.is_cuda and not self.enforce_eager:
            self.capture_cudagraph()
        self.spec.setup_graphs()

        if self.world_size > 1:
            name = channel_name or "llmserve_b200"
            if rank == 0:
                self.channel = RpcChannel(name, self.world_size - 1, create=True, ack_timeout_s=config.comm_timeout_s)
                tp.barrier()
            else:
                tp.barrier()
                self.channel = RpcChannel(name, self.world_size - 1, create=False)
                self._parent_pid = parent_pid or os.getppid()
                self.loop()

    # ---- sampler (settable on rank 0, mirrored to the workers) -------------------------------
    @property
    def sampler(self):
        return self._sampler

    @sampler.setter
    def sampler(self, value):
        if self.channel is not None and self.rank == 0:
            self.channel.send("_set_sampler", value)
        self._sampler = value

    def _set_sampler(self, value):
        self._sampler = value

    # ---- control plane -----------------------------------------------------------------------
    def exit(self):
        if self.step_profile:
            import sys
            print(f"[llmserve_b200 rank {self.rank}] step profile: "
                  + ", ".join(f"{k}={v:.4f}" for k, v in sorted(self.step_profile.items())), file=sys.stderr)
        if self.channel is not None and self.rank == 0:
            try:
                self.channel.wait_acks(self.config.comm_timeout_s)
            except Exception:
                pass
        self.graphs = {}
        self.graph_pool = None
        self.spec.graphs = None
        if self.is_cuda:
            torch.cuda.synchronize()
        if self.world_size > 1:
            try:
                tp.barrier()
            except Exception:
                pass
        if self.channel is not None:
            self.channel.close()
        tp.destroy_tensor_parallel()
        # release device memory so another engine can be built in this process
        self._bind_pools(None, None)
        self.k_cache = self.v_cache = self.draft_k_cache = self.draft_v_cache = None
        self.peer_k = self.peer_v = self.peer_dk = self.peer_dv = None
        self.decode_workspace = None
        self._release_pd()
        self.graph_vars = None
        if self.is_cuda:
            import gc
            self.model = self.model.to("meta") if hasattr(self.model, "to") else None
            if self.draft_model is not None:
                self.draft_model = self.draft_model.to("meta")
            gc.collect()
            torch.cuda.empty_cache()

    def _prof(self, key: str, dt: float):
        p = self.step_profile
        p[key] = p.get(key, 0.0) + dt

    def loop(self):
        worker = self.rank - 1
        while True:
            t0 = time.perf_counter()
            try:
                method, args = self.channel.recv(worker, idle_timeout_s=5.0, parent_pid=self._parent_pid)
            except RpcTimeout:
                break
            if self.step_profile is not None and method == "run":
                self._prof("worker_recv_wait_s", time.perf_counter() - t0)
            if method == "exit":
                self.channel.ack(worker, True)
                self.exit()
                break
            try:
                t1 = time.perf_counter()
                getattr(self, method)(*args)
                if self.step_profile is not None and method == "run":
                    self._prof("run_s", time.perf_counter() - t1)
                self.channel.ack(worker, True)
            except Exception as e:
                self.channel.ack(worker, False, f"{type(e).__name__}: {e}")
                raise

    def call(self, method: str, *args):
        if self.channel is not None and self.rank == 0:
            self.channel.check_workers()
            self.channel.send(method, *args)
        if self.step_profile is not None and method == "run":
            t1 = time.perf_counter()
            out = getattr(self, method)(*args)
            self._prof("run_s", time.perf_counter() - t1)
            return out
        return getattr(self, method)(*args)

    def get_step_profile(self) -> dict:
        """Host-side phase totals recorded when ``LLMSERVE_STEP_PROFILE=1`` (diagnostics)."""
        return dict(self.step_profile or {})

    # ---- memory ------------------------------------------------------------------------------
    def _kv_block_bytes(self) -> int:
        hf = self.hf_config
        nkv = hf.num_key_value_heads // self.world_size
        esize = torch.tensor([], dtype=self.dtype).element_size()
        per = 2 * hf.num_hidden_layers * self.block_size * nkv * hf.head_dim * esize
        if self.draft_model is not None:
            d = self.draft_model
            per += 2 * self.block_size * d.num_kv_heads * d.head_dim * esize
        return per

    def _bind_pools(self, k_cache, v_cache, dk=None, dv=None):
        empty = torch.tensor([])
        for i, layer in enumerate(self.model.model.layers):
            layer.self_attn.attn.k_cache = k_cache[i] if k_cache is not None else empty
            layer.self_attn.attn.v_cache = v_cache[i] if v_cache is not None else empty
        if self.draft_model is not None:
            self.draft_model.bind_kv_cache(dk if dk is not None else empty, dv if dv is not None else empty)

    @torch.inference_mode()
    def warmup_model(self):
        """One maximal prefill on a scratch pool to measure peak activation memory."""
        self.warmup_pool_bytes = 0
        if not self.is_cuda:
            return
        torch.cuda.empty_cache()
        torch.cuda.reset_peak_memory_stats(self.device)
        cfg, hf = self.config, self.hf_config
        seq_len = min(cfg.max_num_batched_tokens, cfg.max_model_len)
        num_seqs = max(1, min(cfg.max_num_batched_tokens // seq_len, cfg.max_num_seqs))
        need = -(-seq_len // self.block_size)
        nkv = hf.num_key_value_heads // self.world_size
        shape = (hf.num_hidden_layers, need * num_seqs, nkv, self.block_size, hf.head_dim)
        k = torch.zeros(shape, dtype=self.dtype, device=self.device)
        v = torch.zeros_like(k)
        dk = dv = None
        if self.draft_model is not None:
            d = self.draft_model
            dk = torch.zeros(need * num_seqs, d.num_kv_heads, self.block_size, d.head_dim,
                             dtype=self.dtype, device=self.device)
            dv = torch.zeros_like(dk)
        self.warmup_pool_bytes = sum(t.numel() * t.element_size() for t in (k, v, dk, dv) if t is not None)
        self._bind_pools(k, v, dk, dv)
        seqs = [Sequence([0] * seq_len) for _ in range(num_seqs)]
        for i, s in enumerate(seqs):
            s.num_scheduled_tokens = seq_len
            s.block_table = list(range(i * need, (i + 1) * need))
        self.run(SchedulerOutput(seqs, seqs, [], seq_len * num_seqs), warmup=True)
        self.spec.clear_all()
        torch.cuda.synchronize()
        self._bind_pools(None, None)
        del k, v, dk, dv
        torch.cuda.empty_cache()

    def allocate_kv_cache(self):
        cfg, hf = self.config, self.hf_config
        block_bytes = self._kv_block_bytes()
        if self.is_cuda:
            free, total = torch.cuda.mem_get_info(self.device)
            used = total - free
            stats = torch.cuda.memory_stats(self.device)
            peak = stats["allocated_bytes.all.peak"] - self.warmup_pool_bytes
            current = stats["allocated_bytes.all.current"]
            budget = int(total * cfg.gpu_memory_utilization - used - peak + current)
            blocks = budget // block_bytes
            if cfg.num_kvcache_blocks > 0:
                blocks = min(blocks, cfg.num_kvcache_blocks)
            if self.world_size > 1:
                t = torch.tensor([blocks], device=self.device)
                torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MIN)
                blocks = int(t.item())
        else:
            blocks = cfg.num_kvcache_blocks if cfg.num_kvcache_blocks > 0 else 64
        if cfg.max_kvcache_blocks > 0:
            blocks = min(blocks, cfg.max_kvcache_blocks)
        if blocks <= 0:
            raise RuntimeError("no memory left for the KV cache")
        cfg.num_kvcache_blocks = blocks
        nkv = hf.num_key_value_heads // self.world_size
        shape = (hf.num_hidden_layers, blocks, nkv, self.block_size, hf.head_dim)
        if cfg.pd_role == "decode":
            self.k_cache, self.v_cache = self._exportable_pools(shape, "kv")
        else:
            self.k_cache = torch.zeros(shape, dtype=self.dtype, device=self.device)
            self.v_cache = torch.zeros(shape, dtype=self.dtype, device=self.device)
        self.draft_k_cache = self.draft_v_cache = None
        if self.draft_model is not None:
            d = self.draft_model
            dshape = (blocks, d.num_kv_heads, self.block_size, d.head_dim)
            if cfg.pd_role == "decode":
                self.draft_k_cache, self.draft_v_cache = self._exportable_pools(dshape, "draft")
            else:
                self.draft_k_cache = torch.zeros(dshape, dtype=self.dtype, device=self.device)
                self.draft_v_cache = torch.zeros(dshape, dtype=self.dtype, device=self.device)
        self._bind_pools(self.k_cache, self.v_cache, self.draft_k_cache, self.draft_v_cache)
        if self.is_cuda:
            # the block tables the decode graphs pass cover whole blocks: size the split-KV
            # workspace for that capacity so the graph never builds a fresh one
            max_ctx = -(-(cfg.max_model_len + cfg.speculative_gamma + 16) // self.block_size) * self.block_size
            heads = max(hf.num_attention_heads // self.world_size,
                        self.draft_model.num_heads if self.draft_model is not None else 0)
            # rows: one per sequence for decode, gamma + 1 per sequence for a packed EAGLE3 verify
            rows = cfg.max_num_seqs * (cfg.speculative_gamma + 1 if self.draft_model is not None else 1)
            self.decode_workspace = attn_ops.DecodeWorkspace(max(rows, 16), heads, hf.head_dim, max_ctx, self.device)

    # ---- prefill/decode disaggregation: KV pools shared across processes ---------------------
    def _exportable_pools(self, shape, key: str):
        """K and V pools another process can map: ordinary device tensors shared through CUDA IPC
        (torch's tensor reduction) on the GPU, a named shared-memory segment on the CPU tier.
        ``key`` names the pair in the descriptor (``"kv"`` target, ``"draft"`` EAGLE3 draft)."""
        if not hasattr(self, "_pd_descs"):
            self._pd_descs, self._pd_pools, self._pd_shms = {}, [], []
        if self.is_cuda:
            from torch.multiprocessing.reductions import reduce_tensor
            pools = torch.zeros((2, *shape), dtype=self.dtype, device=self.device)
            desc = {"kind": "cuda", "ipc": reduce_tensor(pools)}
        else:
            from multiprocessing.shared_memory import SharedMemory
            esize = torch.tensor([], dtype=self.dtype).element_size()
            nbytes = 2 * esize
            for d in shape:
                nbytes *= d
            shm = SharedMemory(create=True, size=nbytes)
            self._pd_shms.append(shm)
            raw = torch.frombuffer(shm.buf, dtype=torch.uint8)
            raw.zero_()
            pools = raw.view(self.dtype).view(2, *shape)
            desc = {"kind": "shm", "name": shm.name}
        desc.update(shape=tuple(shape), dtype=str(self.dtype).replace("torch.", ""))
        self._pd_descs[key] = desc
        self._pd_pools.append(pools)
        return pools[0], pools[1]

    def export_kv(self):
        """Every rank's pool descriptors (``{"kv": ..., "draft": ...}``), gathered on rank 0 (the
        decode side of a disaggregated pair)."""
        mine = getattr(self, "_pd_descs", None)
        if self.world_size == 1:
            return [mine]
        out = [None] * self.world_size
        torch.distributed.all_gather_object(out, mine)
        return out

    def _map_pools(self, d):
        if d["kind"] == "cuda":
            fn, args = d["ipc"]
            return fn(*args)
        from multiprocessing import resource_tracker
        from multiprocessing.shared_memory import SharedMemory
        shm = SharedMemory(name=d["name"])
        try:     # the decode process owns (and unlinks) the segment, not this one
            resource_tracker.unregister(shm._name, "shared_memory")
        except Exception:
            pass
        self._peer_shms.append(shm)
        raw = torch.frombuffer(shm.buf, dtype=torch.uint8)
        return raw.view(getattr(torch, d["dtype"])).view(2, *d["shape"])

    def open_peer_kv(self, descs):
        """Prefill side: map the decode rank with this rank's index (same KV-head shard; the draft's
        pools are replicated).  On the GPU a mapping is a tensor on the decode GPU; the push kernel
        stores into it over NVLink."""
        d = descs[self.rank]
        self._peer_shms, self._peer_pools = [], []
        pools = self._map_pools(d["kv"])
        if tuple(pools.shape[3:]) != tuple(self.k_cache.shape[2:]) or pools.shape[1] != self.k_cache.shape[0]:
            raise ValueError("prefill and decode KV pools have different block shapes")
        self._peer_pools.append(pools)
        self.peer_k, self.peer_v = pools[0], pools[1]
        self.peer_dk = self.peer_dv = None
        if self.draft_model is not None:
            if "draft" not in d:
                raise ValueError("the decode side has no draft pools")
            dpools = self._map_pools(d["draft"])
            if tuple(dpools.shape[2:]) != tuple(self.draft_k_cache.shape[1:]):
                raise ValueError("prefill and decode draft pools have different block shapes")
            self._peer_pools.append(dpools)
            self.peer_dk, self.peer_dv = dpools[0], dpools[1]

    def push_kv(self, src_ids, dst_ids):
        """Copy blocks of this rank's pools (target, and draft when present) into the mapped decode
        pools; returns when they landed."""
        from llmserve_b200.ops import kv as kv_ops
        kv_ops.push_blocks(self.k_cache, self.v_cache, self.peer_k, self.peer_v, src_ids, dst_ids)
        if getattr(self, "peer_dk", None) is not None:
            kv_ops.push_blocks(self.draft_k_cache.unsqueeze(0), self.draft_v_cache.unsqueeze(0),
                               self.peer_dk.unsqueeze(0), self.peer_dv.unsqueeze(0), src_ids, dst_ids)
        if self.is_cuda:
            torch.cuda.current_stream(self.device).synchronize()

    def set_draft_lengths(self, lengths: dict):
        """Decode side of a disaggregated pair: the draft K/V length of each handed-off sequence."""
        self.spec.draft_kv_len.update(lengths)

    def _release_pd(self):
        import gc
        self._peer_pools = self._pd_pools = None
        self.peer_k = self.peer_v = self.peer_dk = self.peer_dv = None
        gc.collect()                       # drop the tensors that view the shared segments
        for shms, unlink in ((getattr(self, "_peer_shms", None) or [], False),
                             (getattr(self, "_pd_shms", None) or [], True)):
            for shm in shms:
                try:
                    shm.close()
                except BufferError:        # a view is still alive; the OS reclaims it at exit
                    pass
                if unlink:
                    try:
                        shm.unlink()
                    except FileNotFoundError:
                        pass
        self._peer_shms, self._pd_shms = [], []

    def get_memory_metrics(self) -> dict:
        seen, model_bytes = set(), 0
        for t in list(self.model.parameters()) + list(self.model.buffers()):
            if t.numel() == 0:
                continue
            key = (str(t.device), t.untyped_storage().data_ptr())
            if key not in seen:
                seen.add(key)
                model_bytes += t.untyped_storage().nbytes()
        kv_bytes = (self.k_cache.numel() + self.v_cache.numel()) * self.k_cache.element_size()
        out = {
            "model_runtime_bytes": model_bytes,
            "kv_cache_bytes": kv_bytes,
            "kv_block_bytes": kv_bytes // max(self.config.num_kvcache_blocks, 1),
        }
        if self.is_cuda:
            _, total = torch.cuda.mem_get_info(self.device)
            out.update({
                "cuda_allocated_bytes": torch.cuda.memory_allocated(self.device),
                "cuda_reserved_bytes": torch.cuda.memory_reserved(self.device),
                "cuda_peak_allocated_bytes": torch.cuda.max_memory_allocated(self.device),
                "cuda_total_bytes": total,
            })
        return out

    # ---- step metadata -----------------------------------------------------------------------
    def check_bounds(self, seqs: list[Sequence], positions, slots):
        """``Config.debug_bounds_checks``: validate a step's metadata on the host before any
        kernel sees it -- every block id inside the pool, every position inside the sequence's
        blocks, every slot either -1 (skip) or inside the pool and equal to the block-table slot of
        its position.  Raises ValueError naming the sequence; a no-op when the option is off."""
        if not self.config.debug_bounds_checks:
            return
        nb, bsz = self.config.num_kvcache_blocks, self.block_size
        positions = np.asarray(positions, dtype=np.int64).reshape(-1)
        slots = np.asarray(slots, dtype=np.int64).reshape(-1)
        if positions.shape != slots.shape:
            raise ValueError("bounds check: positions and slots differ in length")
        per = len(positions) // max(len(seqs), 1) if len(seqs) and len(positions) % len(seqs) == 0 else None
        for s in seqs:
            bad = [b for b in s.block_table if not 0 <= b < nb]
            if bad:
                raise ValueError(f"bounds check: sequence {s.seq_id} holds block ids {bad} outside 0..{nb - 1}")
        if ((slots < -1) | (slots >= nb * bsz)).any():
            raise ValueError(f"bounds check: slot outside the pool of {nb * bsz} slots: {slots.min()}..{slots.max()}")
        if per is not None:
            for i, s in enumerate(seqs):
                for p, sl in zip(positions[i * per:(i + 1) * per], slots[i * per:(i + 1) * per]):
                    if p < 0 or p // bsz >= len(s.block_table):
                        raise ValueError(f"bounds check: sequence {s.seq_id} position {p} beyond its "
                                         f"{len(s.block_table)} blocks")
                    if sl >= 0 and sl != s.block_table[p // bsz] * bsz + p % bsz:
                        raise ValueError(f"bounds check: sequence {s.seq_id} position {p} maps to slot {sl}")

    def prepare_block_tables(self, seqs: list[Sequence]) -> torch.Tensor:
        width = max(1, max(len(s.block_table) for s in seqs))
        rows = np.zeros((len(seqs), width), dtype=np.int32)
        for i, s in enumerate(seqs):
            rows[i, :len(s.block_table)] = s.block_table
        self.h2d_bytes += rows.nbytes
        return _to_device(rows, torch.int32, self.device)

    def _slots(self, seq: Sequence, start: int, end: int) -> np.ndarray:
        pos = np.arange(start, end, dtype=np.int64)
        table = np.asarray(seq.block_table, dtype=np.int64)
        return table[pos // self.block_size] * self.block_size + pos % self.block_size

    def prepare_prefill(self, seqs: list[Sequence], decode_seqs: list[Sequence] | None = None):
        decode_ids = {s.seq_id for s in (decode_seqs or [])}
        ids, pos, slots = [], [], []
        cu_q, cu_k, lens_k, last = [0], [0], [], []
        max_q = max_k = 0
        for s in seqs:
            if s.seq_id in decode_ids:
                start, q = len(s) - 1, 1
            else:
                start, q = min(s.num_cached_tokens, len(s) - 1), s.num_scheduled_tokens
            end = start + q
            ids.extend(s.token_ids[start:end])
            pos.extend(range(start, end))
            slots.append(self._slots(s, start, end))
            cu_q.append(cu_q[-1] + q)
            cu_k.append(cu_k[-1] + end)
            lens_k.append(end)
            last.append(cu_q[-1] - 1)
            max_q, max_k = max(max_q, q), max(max_k, end)
        d = self.device
        slot_arr = np.concatenate(slots)
        if self.config.debug_bounds_checks:
            for s, sl, end in zip(seqs, slots, lens_k):
                self.check_bounds([s], np.arange(end - len(sl), end), sl)
        self.h2d_bytes += 16 * len(ids) + 4 * len(slot_arr) + 16 * len(seqs) + 8
        set_context(
            True,
            cu_seqlens_q=_to_device(cu_q, torch.int32, d),
            cu_seqlens_k=_to_device(cu_k, torch.int32, d),
            max_seqlen_q=max_q, max_seqlen_k=max_k,
            slot_mapping=_to_device(slot_arr, torch.int32, d),
            block_tables=self.prepare_block_tables(seqs),
            seqlens_k=_to_device(lens_k, torch.int32, d),
            last_token_indices=_to_device(last, torch.int64, d),
            decode_workspace=self.decode_workspace,
        )
        return _to_device(ids, torch.int64, d), _to_device(pos, torch.int64, d)

    def prepare_decode(self, seqs: list[Sequence]):
        n = len(seqs)
        ids = np.empty(n, dtype=np.int64)
        pos = np.empty(n, dtype=np.int64)
        slots = np.empty(n, dtype=np.int32)
        lens = np.empty(n, dtype=np.int32)
        for i, s in enumerate(seqs):
            L = len(s)
            ids[i], pos[i], lens[i] = s.last_token, L - 1, L
            slots[i] = s.block_table[(L - 1) // self.block_size] * self.block_size + (L - 1) % self.block_size
        d = self.device
        self.check_bounds(seqs, pos, slots)
        self.h2d_bytes += ids.nbytes + pos.nbytes + slots.nbytes + lens.nbytes
        set_context(False, slot_mapping=_to_device(slots, torch.int32, d), context_lens=_to_device(lens, torch.int32, d),
                    block_tables=self.prepare_block_tables(seqs), decode_workspace=self.decode_workspace)
        return _to_device(ids, torch.int64, d), _to_device(pos, torch.int64, d)

    def prepare_sample(self, seqs: list[Sequence]) -> torch.Tensor:
        self.h2d_bytes += 4 * len(seqs)
        return _to_device([s.temperature for s in seqs], torch.float32, self.device)

    # ---- forward -----------------------------------------------------------------------------
    @torch.inference_mode()
    def run_model(self, input_ids, positions, is_prefill: bool) -> torch.Tensor:
        """Hidden states -> this rank's logit shard (eager path; decode graphs go through
        ``_decode_graph_step``)."""
        return self.model.compute_logits(self.model(input_ids, positions))

    def _use_graph(self, decodes, is_prefill) -> bool:
        return (not is_prefill and bool(self.graphs) and len(decodes) <= self.graph_bs[-1]
                and max(len(s.block_table) for s in decodes) <= self.graph_W)

    def _greedy_from_shards(self, vals: torch.Tensor, idx: torch.Tensor, out: torch.Tensor | None = None):
        """Global greedy ids from every rank's per-shard (max, local index): the NVLink exchange
        kernel when the fused collectives are up (no NCCL call, capturable), else NCCL."""
        fused = tp.get_fused_comm()
        if self.world_size > 1 and fused is not None and vals.shape[0] <= 512:
            if out is None:
                out = torch.empty(vals.shape[0], dtype=torch.int64, device=vals.device)
            return fused.argmax(vals.contiguous(), idx.to(torch.int64).contiguous(), self.model.lm_head.vocab_start,
                                out)
        tokens = tp.vocab_parallel_argmax(vals, idx, self.model.lm_head.vocab_start)
        if out is not None:
            out.copy_(tokens)
            return out
        return tokens

    def sample_tokens(self, logits: torch.Tensor, temperatures: torch.Tensor) -> torch.Tensor:
        """Token ids on every rank from the local logit shard."""
        if getattr(self.sampler, "is_greedy", False):
            vals, idx = sampling_ops.local_argmax(logits)
            return self._greedy_from_shards(vals, idx)
        full = tp.gather_logits(logits)
        tokens = self.sampler(full, temperatures).to(torch.int64).reshape(-1)
        return tp.broadcast(tokens.contiguous(), 0)

    @torch.inference_mode()
    def run(self, scheduler_output: SchedulerOutput, warmup: bool = False) -> list[int] | None:
        seqs = scheduler_output.scheduled_seqs
        prefill, decodes = scheduler_output.prefill_seqs, scheduler_output.decode_seqs
        is_prefill = bool(prefill)
        if self.draft_model is not None and not warmup:
            self.spec.note_plain_step(decodes)
        if self._use_graph(decodes, is_prefill):
            t_run = time.perf_counter()
            logits, vals, idx = self._decode_graph_step(decodes)
            if getattr(self.sampler, "is_greedy", False):
                if self._graph_exchanges_argmax:
                    tokens = self.graph_vars["feed_src"][:len(decodes)]
                else:
                    tokens = tp.vocab_parallel_argmax(vals, idx, self.model.lm_head.vocab_start)
            else:
                tokens = self.sample_tokens(logits, self.prepare_sample(seqs))
            host = self.graph_tokens_host[:len(decodes)]
            t_sync = time.perf_counter()
            host.copy_(tokens)
            token_list = host.tolist()
            if self.step_profile is not None:
                now = time.perf_counter()
                self._prof("decode_launch_s", t_sync - t_run)
                self._prof("decode_sync_wait_s", now - t_sync)
                self._prof("decode_steps", 1)
            self.d2h_bytes += 8 * len(token_list)
            return token_list if self.rank == 0 else None
        input_ids, positions = self.prepare_prefill(seqs, decodes) if is_prefill else self.prepare_decode(decodes)
        temperatures = self.prepare_sample(seqs)
        use_draft = self.draft_model is not None and not warmup
        if is_prefill and use_draft:
            hidden, aux = self.model.forward_with_eagle3_aux(input_ids, positions)
            logits = self.model.compute_logits(hidden)
        else:
            aux = None
            logits = self.run_model(input_ids, positions, is_prefill)
        tokens = self.sample_tokens(logits, temperatures)
        token_list = tokens.tolist()
        self.d2h_bytes += 8 * len(token_list)
        if aux is not None:
            self.spec.after_prefill(seqs, decodes, aux, token_list)
        reset_context()
        return token_list if self.rank == 0 else None

    # ---- CUDA graphs -------------------------------------------------------------------------
    @torch.inference_mode()
    def capture_cudagraph(self):
        """Decode graphs per batch bucket.  All step inputs live in ONE packed int32 device buffer
        (ids, positions, slots, context lengths, feed rows, block tables) filled by one
        host-to-device copy from a pinned staging buffer (two of them, used alternately, so the
        host can fill one while the other's copy is still queued); the graph also holds the LM
        head and the greedy argmax.  ``feed[i] >= 0`` makes row i take the token the previous
        step sampled for row ``feed[i]`` straight from the device (overlapped decode)."""
        max_bs, W = self.pack_max_bs, self.graph_W
        d = self.device
        n = max_bs * (5 + W)                       # ids, pos, slots, lens, feed, tables (int32 each)
        self.graph_pack = torch.zeros(n, dtype=torch.int32, device=d)
        self.graph_pack_hosts = [torch.zeros(n, dtype=torch.int32, pin_memory=True) for _ in range(2)]
        self.graph_pack_nps = [h.numpy() for h in self.graph_pack_hosts]
        self.graph_tokens_host = torch.zeros(max_bs, dtype=torch.int64, pin_memory=True)
        pk = self.graph_pack
        v = {
            "ids32": pk[0:max_bs], "pos32": pk[max_bs:2 * max_bs],
            "slot_mapping": pk[2 * max_bs:3 * max_bs], "context_lens": pk[3 * max_bs:4 * max_bs],
            "feed32": pk[4 * max_bs:5 * max_bs],
            "block_tables": pk[5 * max_bs:].view(max_bs, W),
            "logits": torch.zeros(max_bs, self.model.lm_head.shard_size, dtype=self.dtype, device=d),
            "tok_val": torch.zeros(max_bs, dtype=torch.float32, device=d),
            "tok_idx": torch.zeros(max_bs, dtype=torch.int64, device=d),
        }
        # the sampled global ids of the last decode step: the argmax itself at TP = 1, a copy of
        # the vocab-parallel reduction at TP > 1
        v["feed_src"] = v["tok_idx"] if self.world_size == 1 else torch.zeros(max_bs, dtype=torch.int64, device=d)
        self.graph_bs = [b for b in (1, 2, 4, 8) if b <= max_bs] + list(range(16, max_bs + 1, 16))
        self.graphs, self.graph_pool, self.graph_launches = {}, None, {}
        self.graph_vars = v
        # at TP > 1 with the fused collectives the graph ends with the vocab-parallel argmax
        # exchange, writing the global ids straight into feed_src
        self._graph_exchanges_argmax = self.world_size > 1 and tp.get_fused_comm() is not None
        self._tokens_event = None
        v["context_lens"].fill_(1)
        v["feed32"].fill_(-1)
        for bs in reversed(self.graph_bs):
            g = torch.cuda.CUDAGraph()
            self._graph_body(bs)                   # warm-up outside capture
            before = LaunchCounter.launches
            with torch.cuda.graph(g, self.graph_pool, stream=self.capture_stream()):
                self._graph_body(bs)
            self.graph_launches[bs] = LaunchCounter.launches - before
            if self.graph_pool is None:
                self.graph_pool = g.pool()
            self.graphs[bs] = g
            torch.cuda.synchronize()
            reset_context()

    def capture_stream(self) -> torch.cuda.Stream:
        """This runner's side stream for graph capture.  ``torch.cuda.graph`` would otherwise use
        one class-wide stream created on whichever device captured first; a second runner of the
        same process on another GPU (prefill/decode disaggregation) would then capture on the first
        GPU's stream while its kernels run eagerly on its own, leaving an empty graph."""
        if getattr(self, "_capture_stream", None) is None:
            self._capture_stream = torch.cuda.Stream(device=self.device)
        return self._capture_stream

    def _graph_body(self, bs: int):
        v = self.graph_vars
        set_context(False, slot_mapping=v["slot_mapping"][:bs], context_lens=v["context_lens"][:bs],
                    block_tables=v["block_tables"][:bs], decode_workspace=self.decode_workspace)
        ids = sampling_ops.feed_ids(v["ids32"][:bs], v["feed32"][:bs], v["feed_src"])
        pos = v["pos32"][:bs].long()
        v["logits"][:bs] = self.model.compute_logits(self.model(ids, pos))
        sampling_ops.local_argmax_into(v["logits"][:bs], v["tok_val"][:bs], v["tok_idx"][:bs])
        if self._graph_exchanges_argmax:
            self._greedy_from_shards(v["tok_val"][:bs], v["tok_idx"][:bs], v["feed_src"][:bs])

    def _next_pack(self):
        """The pinned staging buffer to fill next (alternating)."""
        self.graph_pack_turn ^= 1
        return self.graph_pack_hosts[self.graph_pack_turn], self.graph_pack_nps[self.graph_pack_turn]

    def fill_decode_pack(self, a: np.ndarray, seqs: list[Sequence], positions: np.ndarray, ids, feed) -> tuple[int, int]:
        """Write one decode step into staging array ``a``: row i runs token ``ids[i]`` (or the
        previous step's row ``feed[i]``) at ``positions[i]`` of ``seqs[i]``.  Returns (bs, graph bs)."""
        bs = len(seqs)
        gbs = next(x for x in self.graph_bs if x >= bs) if self.graphs else bs
        max_bs, W, bsz = self.pack_max_bs, self.graph_W, self.block_size
        a[0:bs] = ids
        a[max_bs:max_bs + bs] = positions
        blocks = np.fromiter((s.block_table[p // bsz] for s, p in zip(seqs, positions.tolist())), dtype=np.int32,
                             count=bs)
        a[2 * max_bs:2 * max_bs + bs] = blocks * bsz + positions % bsz
        self.check_bounds(seqs, positions, a[2 * max_bs:2 * max_bs + bs])
        a[3 * max_bs:3 * max_bs + bs] = positions + 1
        a[4 * max_bs:4 * max_bs + bs] = feed
        tables = a[5 * max_bs:].reshape(max_bs, W)
        for i, s in enumerate(seqs):
            t = s.block_table
            tables[i, :len(t)] = t
        if gbs > bs:
            a[bs:gbs] = 0
            a[max_bs + bs:max_bs + gbs] = 0
            a[2 * max_bs + bs:2 * max_bs + gbs] = -1
            a[3 * max_bs + bs:3 * max_bs + gbs] = 1
            a[4 * max_bs + bs:4 * max_bs + gbs] = -1
        return bs, gbs

    def _replay(self, host: torch.Tensor, bs: int, gbs: int):
        max_bs, W = self.pack_max_bs, self.graph_W
        n = 5 * max_bs + gbs * W
        self.h2d_bytes += n * 4
        self.graph_pack[:n].copy_(host[:n], non_blocking=True)
        self.graphs[gbs].replay()
        LaunchCounter.launches += self.graph_launches[gbs]
        v = self.graph_vars
        if self.world_size > 1 and not self._graph_exchanges_argmax:
            tokens = tp.vocab_parallel_argmax(v["tok_val"][:bs], v["tok_idx"][:bs], self.model.lm_head.vocab_start)
            v["feed_src"][:bs].copy_(tokens)

    def _decode_graph_step(self, seqs: list[Sequence]):
        """Pack the step inputs, one H2D copy, replay; returns the logits shard view and the
        per-shard argmax (value, index) views of the graph outputs."""
        host, a = self._next_pack()
        lens = np.fromiter((len(s) for s in seqs), dtype=np.int32, count=len(seqs))
        ids = np.fromiter((s.last_token for s in seqs), dtype=np.int32, count=len(seqs))
        bs, gbs = self.fill_decode_pack(a, seqs, lens - 1, ids, -1)
        max_bs, W = self.pack_max_bs, self.graph_W
        n = 5 * max_bs + gbs * W
        self.h2d_bytes += n * 4
        self.graph_pack[:n].copy_(host[:n], non_blocking=True)
        self.graphs[gbs].replay()
        LaunchCounter.launches += self.graph_launches[gbs]
        v = self.graph_vars
        return v["logits"][:bs], v["tok_val"][:bs], v["tok_idx"][:bs]

    # ---- overlapped decode: step N+1 is launched before step N's tokens reach the host -----------
    def can_overlap(self) -> bool:
        """Greedy decode through CUDA graphs (or the CPU tier's eager emulation), no draft model."""
        return (getattr(self.sampler, "is_greedy", False) and self.draft_model is None
                and (bool(self.graphs) or not self.is_cuda))

    def overlap_fits(self, bs: int, max_blocks: int) -> bool:
        if not self.is_cuda:
            return True
        return bool(self.graphs) and bs <= self.graph_bs[-1] and max_blocks <= self.graph_W

    def overlap_launch(self, seqs: list[Sequence], positions: np.ndarray, ids, feed, read_previous: bool) -> int:
        """Rank 0: stage one overlapped decode step of ``seqs`` and launch it on every rank."""
        host, a = self._next_pack()
        bs, gbs = self.fill_decode_pack(a, seqs, positions, ids, feed)
        if self.channel is not None:
            n = 5 * self.pack_max_bs + gbs * self.graph_W
            self.channel.check_workers()
            self.channel.send("launch_decode", a[:n].copy(), bs, gbs, read_previous)
        self.launch_decode(None, bs, gbs, read_previous)
        return bs

    @torch.inference_mode()
    def launch_decode(self, pack: np.ndarray | None, bs: int, gbs: int, read_previous: bool):
        """Run one overlapped decode step.  Rank 0 fills ``pack`` itself (``None`` is passed to it)
        and sends its used prefix to the workers.  With ``read_previous`` rank 0 first queues the
        device->host copy of the in-flight step's tokens (so it lands before this step overwrites
        them); :meth:`collect_decode` waits for it."""
        if not self.is_cuda:
            if pack is not None:
                _, a = self._next_pack()
                a[:pack.shape[0]] = pack
            return self._launch_decode_cpu(bs, read_previous)
        if pack is None:
            host = self.graph_pack_hosts[self.graph_pack_turn]
        else:
            host, a = self._next_pack()
            a[:pack.shape[0]] = pack
        v = self.graph_vars
        if read_previous and self.rank == 0:
            nb = self.inflight_bs
            self.graph_tokens_host[:nb].copy_(v["feed_src"][:nb], non_blocking=True)
            self.d2h_bytes += 8 * nb
            self._tokens_event = torch.cuda.Event()
            self._tokens_event.record()
            self._tokens_bs = nb
        self._replay(host, bs, gbs)
        self.inflight_bs = bs

    def collect_decode(self) -> list[int]:
        """Rank 0: the previous in-flight step's tokens (queued by :meth:`launch_decode`)."""
        if not self.is_cuda:
            return self._cpu_collected
        self._tokens_event.synchronize()
        return self.graph_tokens_host[:self._tokens_bs].tolist()

    @torch.inference_mode()
    def drain_decode(self) -> list[int]:
        """Rank 0: the current in-flight step's tokens; nothing is in flight afterwards."""
        nb = self.inflight_bs
        self.inflight_bs = 0
        if not self.is_cuda:
            return self._cpu_next.tolist()
        host = self.graph_tokens_host[:nb]
        host.copy_(self.graph_vars["feed_src"][:nb])
        self.d2h_bytes += 8 * nb
        return host.tolist()

    def _launch_decode_cpu(self, bs, read_previous):
        """CPU tier: the same protocol computed eagerly (the tokens stay in a tensor until read)."""
        a = self.graph_pack_nps[self.graph_pack_turn]
        max_bs, W = self.pack_max_bs, self.graph_W
        ids, pos = a[0:bs].astype(np.int64), a[max_bs:max_bs + bs].astype(np.int64)
        slots, lens, feed = a[2 * max_bs:2 * max_bs + bs], a[3 * max_bs:3 * max_bs + bs], a[4 * max_bs:4 * max_bs + bs]
        tables = a[5 * max_bs:].reshape(max_bs, W)[:bs]
        prev = getattr(self, "_cpu_next", None)
        if read_previous:
            self._cpu_collected = prev.tolist()
        ids_t = torch.as_tensor(ids)
        fed = torch.as_tensor(feed) >= 0
        if bool(fed.any()):
            ids_t[fed] = prev[torch.as_tensor(feed)[fed].long()]
        set_context(False, slot_mapping=torch.as_tensor(slots), context_lens=torch.as_tensor(lens),
                    block_tables=torch.as_tensor(np.ascontiguousarray(tables)), decode_workspace=None)
        logits = self.model.compute_logits(self.model(ids_t, torch.as_tensor(pos)))
        reset_context()
        self._cpu_next = self.sample_tokens(logits, None).cpu()
        self.inflight_bs = bs

    # ---- device timing (benchmarks): every rank records, rank 0 gathers -------------------------
    def mark_event(self, tag: str, fence: str = ""):
        """Record a CUDA event ``tag`` on this rank's stream.  ``fence="before"`` first drains this
        GPU and meets every rank at a barrier (a window opened this way starts with nothing in
        flight on any rank); ``fence="after"`` drains and meets after recording."""
        if not hasattr(self, "_events"):
            self._events = {}
        if fence == "before" and self.is_cuda:
            torch.cuda.synchronize()
            tp.barrier()
        if self.is_cuda:
            e = torch.cuda.Event(enable_timing=True)
            e.record()
            self._events[tag] = e
        self._events[tag + ":launches"] = LaunchCounter.launches
        if fence == "after" and self.is_cuda:
            torch.cuda.synchronize()
            tp.barrier()

    def gather_elapsed(self, start: str, end: str):
        """Per-rank (device ms between two marks, kernel launches between them)."""
        if self.is_cuda:
            torch.cuda.synchronize()
            ms = self._events[start].elapsed_time(self._events[end])
        else:
            ms = 0.0
        mine = torch.tensor([ms, float(self._events[end + ":launches"] - self._events[start + ":launches"])],
                            dtype=torch.float64, device=self.device)
        if self.world_size > 1:
            parts = [torch.empty_like(mine) for _ in range(self.world_size)]
            torch.distributed.all_gather(parts, mine)
            mine = torch.stack(parts)
        return mine.view(-1, 2).tolist() if self.rank == 0 else None

    # ---- speculative entry points (called through the RPC by name) -----------------------------
    def run_speculative_batch(self, seqs):
        return self.spec.run_speculative_batch(seqs)

    def run_speculative_single(self, seq):
        return self.spec.run_speculative_batch([seq])[0]

    def run_speculative_tree_single(self, seq):
        return self.spec.run_speculative_tree_single(seq)

    def clear_speculative_state(self, seq_ids):
        self.spec.clear_speculative_state(seq_ids)
