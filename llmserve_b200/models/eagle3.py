"""EAGLE3 speculator (one Llama-style decoder layer over [embedding ; fused target hidden]).

Checkpoint parity with ``llmserve/models/eagle3.py`` of the reference: RedHat-style nested
``transformer_layer_config`` and SpecForge flat configs (``normalize_eagle3_config``, ``:34-46``),
``layers.0.*`` -> ``midlayer.*`` renaming (``:49-52``), target compatibility checks (``:55-71``),
``fc`` over the concatenated auxiliary hidden states of three target layers, ``hidden_norm`` with
optional ``norm_before_residual``, its own ``lm_head`` over the draft vocabulary with ``d2t``
offsets (draft id + d2t[id] = target id) and the ``t2d`` mask, and a target embedding borrowed
when the draft checkpoint has none.

Runtime design differs: the draft's K/V live in a *paged* pool indexed by the target's block
tables (draft position ``p`` of a sequence uses the same slot as target position ``p``), so the
batched draft runs ordinary paged decode attention and the reference's per-request
``_pack``/``_compact`` tensors (``llmserve/speculative/draft.py:110-153``) do not exist.  The
q/k/v and gate/up projections are concatenated at load so each is one GEMM.
"""
import json
import os

import torch
from safetensors import safe_open
from torch import nn

from llmserve_b200.ops import activation, gemm, kv as kv_ops, sampling
from llmserve_b200.ops import attention as attn_ops
from llmserve_b200.ops import norm as norm_ops
from llmserve_b200.ops import rope as rope_ops
from llmserve_b200.ops.rope import build_cos_sin_cache
from llmserve_b200.speculative.draft import (  # noqa: F401  (offline API, importable from here as in the reference)
    DraftKVPool, DraftKVRef, generate_eagle3_draft_tokens, generate_eagle3_draft_tokens_batched,
    run_eagle3_offline_step, run_eagle3_speculative_cycle, run_eagle3_target_verify)
from llmserve_b200.speculative.sampling import (  # noqa: F401
    sample_from_logits, speculative_accept_greedy_from_logits, speculative_accept_reject_from_logits)
from llmserve_b200.speculative.types import Eagle3DraftOutput
from llmserve_b200.utils.context import get_context, reset_context, set_context


def normalize_eagle3_config(config: dict) -> dict:
    layer = config.get("transformer_layer_config")
    if layer is None:
        return dict(config)
    for key, value in layer.items():
        if key in config and config[key] != value:
            raise ValueError(f"conflicting EAGLE3 config field: {key}")
    merged = dict(layer)
    for key in ("draft_vocab_size", "target_hidden_size", "norm_before_residual"):
        if key in config:
            merged[key] = config[key]
    return merged


def normalize_eagle3_weight_name(name: str) -> str:
    return "midlayer." + name[len("layers.0."):] if name.startswith("layers.0.") else name


def validate_eagle3_target_config(draft_config: dict, target_config: dict):
    draft_config = normalize_eagle3_config(draft_config)
    want_hidden = draft_config.get("target_hidden_size") or draft_config["hidden_size"]
    if target_config["hidden_size"] != want_hidden:
        raise ValueError(f"target hidden_size {target_config['hidden_size']} does not match "
                         f"draft target_hidden_size {want_hidden}")
    if target_config["vocab_size"] != draft_config["vocab_size"]:
        raise ValueError(f"target vocab_size {target_config['vocab_size']} does not match "
                         f"draft vocab_size {draft_config['vocab_size']}")
    if target_config.get("num_hidden_layers", 0) < 1:
        raise ValueError("EAGLE3 target must have hidden layers")


class _Norm(nn.Module):
    def __init__(self, n, eps):
        super().__init__()
        self.eps = eps
        self.weight = nn.Parameter(torch.ones(n), requires_grad=False)

    def forward(self, x):
        return norm_ops.rms_norm(x, self.weight, self.eps)


class _Lin(nn.Module):
    """Bias-free linear holding ``weight [out, in]`` (checkpoint name ``*.weight``)."""

    def __init__(self, n_in, n_out):
        super().__init__()
        self.weight = nn.Parameter(torch.empty(n_out, n_in), requires_grad=False)

    def forward(self, x):
        return gemm.linear(x, self.weight)


class Eagle3Attention(nn.Module):

    def __init__(self, hidden, num_heads, num_kv_heads, head_dim, max_position, rope_theta):
        super().__init__()
        self.num_heads, self.num_kv_heads, self.head_dim = num_heads, num_kv_heads, head_dim
        self.q_proj = _Lin(2 * hidden, num_heads * head_dim)
        self.k_proj = _Lin(2 * hidden, num_kv_heads * head_dim)
        self.v_proj = _Lin(2 * hidden, num_kv_heads * head_dim)
        self.o_proj = _Lin(num_heads * head_dim, hidden)
        self.register_buffer("cos_sin", build_cos_sin_cache(head_dim, max_position, rope_theta), persistent=False)
        self.qkv_weight = None
        self.k_cache = self.v_cache = torch.tensor([])

    def fuse(self):
        self.qkv_weight = torch.cat([self.q_proj.weight, self.k_proj.weight, self.v_proj.weight], 0).contiguous()

    def forward(self, x, positions):
        ctx = get_context()
        w = self.qkv_weight if self.qkv_weight is not None else torch.cat(
            [self.q_proj.weight, self.k_proj.weight, self.v_proj.weight], 0)
        qkv = gemm.linear(x, w)
        scale = self.head_dim ** -0.5
        cos_sin = self.cos_sin.float()
        if ctx.tree_attention_mask is not None:
            # tree drafting: this depth's nodes go to the side buffer, the prefix stays paged
            q, k, v = rope_ops.qkv_norm_rope_store(qkv, positions, cos_sin, None, None, 0.0, None, None,
                                                   None, self.num_heads, self.num_kv_heads, self.head_dim)
            rows = torch.tensor(ctx.tree_rows, dtype=torch.int64, device=x.device)
            ctx.tree_side_k.index_copy_(0, rows, k.to(ctx.tree_side_k.dtype))
            ctx.tree_side_v.index_copy_(0, rows, v.to(ctx.tree_side_v.dtype))
            o = attn_ops.tree_attention(q, self.k_cache, self.v_cache, ctx.tree_block_table, ctx.tree_prefix_len,
                                        ctx.tree_side_k, ctx.tree_side_v, ctx.tree_attention_mask, scale,
                                        ctx.tree_mask_bits)
            return self.o_proj(o.reshape(x.shape[0], -1))
        q, _, _ = rope_ops.qkv_norm_rope_store(qkv, positions, cos_sin, None, None, 0.0,
                                               self.k_cache, self.v_cache, ctx.slot_mapping,
                                               self.num_heads, self.num_kv_heads, self.head_dim)
        if ctx.is_prefill:
            o = attn_ops.prefill_attention(q, self.k_cache, self.v_cache, ctx.cu_seqlens_q, ctx.seqlens_k,
                                           ctx.block_tables, scale, ctx.max_seqlen_q)
        else:
            o = attn_ops.decode_attention(q, self.k_cache, self.v_cache, ctx.block_tables, ctx.context_lens,
                                          scale, ctx.decode_workspace)
        return self.o_proj(o.reshape(x.shape[0], -1))


class Eagle3MLP(nn.Module):

    def __init__(self, hidden, intermediate):
        super().__init__()
        self.gate_proj = _Lin(hidden, intermediate)
        self.up_proj = _Lin(hidden, intermediate)
        self.down_proj = _Lin(intermediate, hidden)
        self.gate_up_weight = None

    def fuse(self):
        self.gate_up_weight = torch.cat([self.gate_proj.weight, self.up_proj.weight], 0).contiguous()

    def forward(self, x):
        w = self.gate_up_weight if self.gate_up_weight is not None else torch.cat(
            [self.gate_proj.weight, self.up_proj.weight], 0)
        return self.down_proj(activation.silu_and_mul(gemm.linear(x, w)))


class Eagle3DecoderLayer(nn.Module):

    def __init__(self, hidden, num_heads, num_kv_heads, head_dim, intermediate, max_position, rope_theta,
                 eps, norm_before_residual=False):
        super().__init__()
        self.hidden_size = hidden
        self.norm_before_residual = norm_before_residual
        self.input_layernorm = _Norm(hidden, eps)
        self.hidden_norm = _Norm(hidden, eps)
        self.post_attention_layernorm = _Norm(hidden, eps)
        self.self_attn = Eagle3Attention(hidden, num_heads, num_kv_heads, head_dim, max_position, rope_theta)
        self.mlp = Eagle3MLP(hidden, intermediate)

    def forward(self, embeds, fused_hidden, positions):
        if self.norm_before_residual:
            hidden = self.hidden_norm(fused_hidden)
            residual = hidden
        else:
            residual = fused_hidden
            hidden = self.hidden_norm(fused_hidden)
        attn_in = torch.cat([self.input_layernorm(embeds), hidden], dim=-1)
        residual = residual + self.self_attn(attn_in, positions)
        return residual + self.mlp(self.post_attention_layernorm(residual))


class Eagle3Speculator(nn.Module):

    def __init__(self, config: dict):
        super().__init__()
        self.config = dict(config)
        self.hidden_size = config["hidden_size"]
        self.target_hidden_size = config.get("target_hidden_size") or self.hidden_size
        self.draft_vocab_size = config.get("draft_vocab_size", 32000)
        self.target_vocab_size = config["vocab_size"]
        self.num_heads = config["num_attention_heads"]
        self.num_kv_heads = config["num_key_value_heads"]
        self.head_dim = config.get("head_dim", self.hidden_size // self.num_heads)
        self.embed_tokens = nn.Embedding(self.target_vocab_size, self.hidden_size)
        self.embed_tokens.weight.requires_grad_(False)
        self.fc = _Lin(3 * self.target_hidden_size, self.hidden_size)
        self.midlayer = Eagle3DecoderLayer(
            self.hidden_size, self.num_heads, self.num_kv_heads, self.head_dim, config["intermediate_size"],
            config.get("max_position_embeddings", 40960), config.get("rope_theta", 1000000),
            config.get("rms_norm_eps", 1e-6), config.get("norm_before_residual", False))
        self.norm = _Norm(self.hidden_size, config.get("rms_norm_eps", 1e-6))
        self.lm_head = _Lin(self.hidden_size, self.draft_vocab_size)
        self.register_buffer("d2t", torch.zeros(self.draft_vocab_size, dtype=torch.long))
        self.register_buffer("t2d", torch.zeros(self.target_vocab_size, dtype=torch.bool))

    @classmethod
    def read_config(cls, path: str) -> dict:
        with open(os.path.join(path, "config.json")) as f:
            return normalize_eagle3_config(json.load(f))

    @classmethod
    def from_pretrained(cls, path: str, target_model_path: str | None = None, target_embedding=None):
        config = cls.read_config(path)
        if target_model_path is not None:
            with open(os.path.join(target_model_path, "config.json")) as f:
                validate_eagle3_target_config(config, json.load(f))
        model = cls(config)
        state = {}
        for name in sorted(os.listdir(path)):
            if not name.endswith(".safetensors"):
                continue
            with safe_open(os.path.join(path, name), framework="pt", device="cpu") as f:
                for key in f.keys():
                    norm_key = normalize_eagle3_weight_name(key)
                    if norm_key in state:
                        raise RuntimeError(f"duplicate EAGLE3 weight after normalization: {norm_key}")
                    state[norm_key] = f.get_tensor(key)
        missing, unexpected = model.load_state_dict(state, strict=False)
        if unexpected:
            raise RuntimeError(f"unexpected EAGLE3 weights: {unexpected}")
        missing = [m for m in missing if m != "embed_tokens.weight"]
        if missing:
            raise RuntimeError(f"missing EAGLE3 weights: {missing}")
        if "embed_tokens.weight" not in state:
            if target_embedding is not None:
                model.embed_tokens.weight = target_embedding
            elif target_model_path is not None:
                model.load_target_embedding(target_model_path)
            else:
                raise ValueError("target_model_path is required when draft weights do not include "
                                 "embed_tokens.weight")
        return model

    def load_target_embedding(self, target_model_path: str):
        wanted = "model.embed_tokens.weight"
        for name in sorted(os.listdir(target_model_path)):
            if not name.endswith(".safetensors"):
                continue
            with safe_open(os.path.join(target_model_path, name), framework="pt", device="cpu") as f:
                if wanted in f.keys():
                    self.embed_tokens.weight.data.copy_(f.get_tensor(wanted))
                    return
        raise RuntimeError(f"{wanted} not found in {target_model_path}")

    def prepare(self):
        """Concatenate projections once the weights are on their device."""
        self.midlayer.self_attn.fuse()
        self.midlayer.mlp.fuse()

    def bind_kv_cache(self, k_cache, v_cache):
        self.midlayer.self_attn.k_cache = k_cache
        self.midlayer.self_attn.v_cache = v_cache

    def forward(self, input_ids, aux_hidden, positions):
        """input_ids [T], aux_hidden [T, 3*Ht or H], positions [T] -> (hidden [T, H], draft logits)."""
        embeds = kv_ops.embedding(input_ids, self.embed_tokens.weight)
        fused = aux_hidden if aux_hidden.shape[-1] == self.hidden_size else self.fc(aux_hidden)
        hidden = self.midlayer(embeds, fused, positions)
        return hidden, self.lm_head(self.norm(hidden))

    @torch.inference_mode()
    def propose(self, input_ids, aux_hidden, positions, temperature: float, past_kv=None, kv_valid_lens=None):
        """One offline draft step for B requests (``llmserve/models/eagle3.py:345-364`` of the
        reference): ids and positions ``[B, 1]``, ``aux_hidden`` ``[B, 1, 3*Ht or H]``.

        The step's K/V goes to a paged :class:`DraftKVPool` (a new one when ``past_kv`` is None;
        otherwise the rows of the given :class:`DraftKVRef`, first cut to ``kv_valid_lens`` when
        given), and attention runs through the same store and decode-attention kernels as the
        engine's draft.  The engine's own pool binding is restored afterwards.  Tokens are sampled
        from the target-vocabulary logits at ``temperature`` (draft argmax when it is 0)."""
        ids = input_ids.reshape(-1).long()
        B = ids.numel()
        dev = ids.device
        if past_kv is None:
            pool = DraftKVPool.for_model(self, dev)
            past_kv = DraftKVRef(pool, pool.new_rows(B))
        pool, rows = past_kv.pool, list(past_kv.rows)
        if len(rows) != B:
            raise ValueError(f"{B} draft inputs for {len(rows)} K/V rows")
        if kv_valid_lens is not None:
            for r, n in zip(rows, kv_valid_lens.reshape(-1).tolist()):
                pool.set_length(r, int(n))
        slots = pool.append_slots(rows)
        attn = self.midlayer.self_attn
        bound = attn.k_cache, attn.v_cache
        attn.k_cache, attn.v_cache = pool.k, pool.v
        set_context(False, slot_mapping=torch.tensor(slots, dtype=torch.int32, device=dev),
                    context_lens=torch.tensor(past_kv.lengths, dtype=torch.int32, device=dev),
                    block_tables=pool.block_table(rows, dev))
        try:
            hidden, logits = self(ids, aux_hidden.reshape(B, -1), positions.reshape(-1).long())
        finally:
            reset_context()
            attn.k_cache, attn.v_cache = bound
        target_logits = self.map_draft_logits(logits)
        if temperature > 1e-10:
            token_ids = sample_from_logits(target_logits, temperature)
        else:
            token_ids = self.greedy_sample(logits)
        return Eagle3DraftOutput(hidden.unsqueeze(1), logits.unsqueeze(1), target_logits.unsqueeze(1),
                                 token_ids.view(B, 1), DraftKVRef(pool, rows))

    def compute_logits(self, hidden_states: torch.Tensor) -> torch.Tensor:
        """Draft logits of ``hidden_states`` scattered into the target vocabulary (``-inf`` outside
        the draft vocabulary), as ``llmserve/models/eagle3.py:330-332`` of the reference."""
        return self.map_draft_logits(self.lm_head(self.norm(hidden_states)))

    def map_draft_logits(self, draft_logits: torch.Tensor) -> torch.Tensor:
        """Scatter draft-vocab logits into a -inf target-vocab row (rejection sampling)."""
        idx = torch.arange(self.draft_vocab_size, device=draft_logits.device) + self.d2t
        out = draft_logits.new_full((*draft_logits.shape[:-1], self.target_vocab_size), float("-inf"))
        out[..., idx] = draft_logits
        return out

    def greedy_sample(self, draft_logits: torch.Tensor) -> torch.Tensor:
        ids = sampling.argmax(draft_logits.reshape(-1, draft_logits.shape[-1])).view(draft_logits.shape[:-1])
        return ids + self.d2t[ids]

    def greedy_topk(self, draft_logits: torch.Tensor, k: int) -> torch.Tensor:
        ids = torch.topk(draft_logits.float(), k=k, dim=-1).indices
        return ids + self.d2t[ids]
