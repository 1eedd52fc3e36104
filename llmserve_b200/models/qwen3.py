"""Qwen3 dense decoder, tensor parallel.

Architecture parity with ``llmserve/models/qwen3.py`` of the reference: GQA with per-head QK
RMSNorm when ``attention_bias`` is false, neox RoPE, fused ``qkv_proj`` / ``gate_up_proj``
(checkpoint ``q/k/v_proj`` and ``gate/up_proj`` are merged at load), residual-carrying RMSNorm,
and EAGLE3 auxiliary capture of the residual stream *entering* layers
``{2, L/2, L-3}`` (``qwen3.py:16-18``, ``:203-211``).

The forward pass is arranged around the fusions of the sm_100a path: the residual add and the
*next* RMSNorm are applied by the row-parallel projections themselves (``forward_add_norm``), so
one kernel per row-parallel layer does split-K reduction + TP all-reduce + residual + norm.  The
value stream is identical to the reference's ``layer(h, residual)`` formulation.
"""
import torch
from torch import nn

from llmserve_b200.layers.attention import Attention
from llmserve_b200.layers.embed_head import ParallelLMHead, ReplicatedEmbedding
from llmserve_b200.layers.linear import MergedColumnParallelLinear, QKVParallelLinear, RowParallelLinear
from llmserve_b200.layers.norm import RMSNorm
from llmserve_b200.ops import norm as norm_ops
from llmserve_b200.ops.rope import build_cos_sin_cache
from llmserve_b200.parallel import state as tp


def get_eagle3_aux_layer_ids(num_hidden_layers: int) -> tuple[int, int, int]:
    """Layers whose *input* residual stream feeds the EAGLE3 draft, in concatenation order.

    ``(2, L/2, L-3)`` as in the reference (``qwen3.py:16-18``; {2, 18, 33} for Qwen3-8B).  Targets
    shallower than 6 layers (test models) use ``(0, L/2, L-1)`` -- {0, 1, 1} for two layers.
    Duplicates are kept: the draft's ``fc`` always sees three hidden states (the reference turns
    the tuple into a set, which loses the duplicate of a 6-layer target)."""
    if num_hidden_layers < 1:
        raise ValueError("target needs at least one layer")
    if num_hidden_layers < 6:
        return (0, num_hidden_layers // 2, num_hidden_layers - 1)
    return (2, num_hidden_layers // 2, num_hidden_layers - 3)


class Qwen3Attention(nn.Module):

    def __init__(self, config, quant_config=None):
        super().__init__()
        world = tp.get_tp_size()
        self.total_num_heads = config.num_attention_heads
        self.total_num_kv_heads = config.num_key_value_heads
        if self.total_num_heads % world or self.total_num_kv_heads % world:
            raise ValueError("attention heads must divide evenly over the tensor-parallel ranks")
        self.num_heads = self.total_num_heads // world
        self.num_kv_heads = self.total_num_kv_heads // world
        self.head_dim = config.head_dim
        self.qkv_bias = bool(getattr(config, "attention_bias", False))
        self.eps = config.rms_norm_eps
        self.qkv_proj = QKVParallelLinear(config.hidden_size, self.head_dim, self.total_num_heads,
                                          self.total_num_kv_heads, bias=self.qkv_bias, quant_config=quant_config)
        self.o_proj = RowParallelLinear(self.total_num_heads * self.head_dim, config.hidden_size, bias=False,
                                        quant_config=quant_config)
        theta = config.rope_theta
        if isinstance(config.rope_scaling, dict):
            theta = config.rope_scaling.get("rope_theta", theta)
        self.register_buffer("cos_sin", build_cos_sin_cache(self.head_dim, config.max_position_embeddings, theta)
                             .float(), persistent=False)
        self.attn = Attention(self.num_heads, self.head_dim, self.head_dim ** -0.5, self.num_kv_heads)
        if not self.qkv_bias:
            self.q_norm = RMSNorm(self.head_dim, eps=self.eps)
            self.k_norm = RMSNorm(self.head_dim, eps=self.eps)

    def attention_core(self, positions, h):
        qkv = self.qkv_proj.forward_partials(h)
        qw = None if self.qkv_bias else self.q_norm.weight
        kw = None if self.qkv_bias else self.k_norm.weight
        return self.attn(qkv, positions, self.cos_sin, qw, kw, self.eps)


class Qwen3MLP(nn.Module):

    def __init__(self, config, quant_config=None):
        super().__init__()
        if config.hidden_act != "silu":
            raise ValueError("Qwen3 MLP expects silu")
        self.gate_up_proj = MergedColumnParallelLinear(config.hidden_size, [config.intermediate_size] * 2,
                                                       bias=False, quant_config=quant_config)
        self.down_proj = RowParallelLinear(config.intermediate_size, config.hidden_size, bias=False,
                                           quant_config=quant_config)

    def up(self, h):
        return self.gate_up_proj.forward_silu(h)


class Qwen3DecoderLayer(nn.Module):

    def __init__(self, config, quant_config=None):
        super().__init__()
        self.self_attn = Qwen3Attention(config, quant_config)
        self.mlp = Qwen3MLP(config, quant_config)
        self.input_layernorm = RMSNorm(config.hidden_size, eps=config.rms_norm_eps)
        self.post_attention_layernorm = RMSNorm(config.hidden_size, eps=config.rms_norm_eps)

    def forward_fused(self, positions, h, residual, next_norm: RMSNorm):
        """``h`` is this layer's normalised input and ``residual`` the stream entering it.
        Returns ``(next_norm(stream_out), stream_out)``."""
        o = self.self_attn.attention_core(positions, h)
        pn = self.post_attention_layernorm
        h, residual = self.self_attn.o_proj.forward_add_norm(o, residual, pn.weight, pn.eps)
        a = self.mlp.up(h)
        return self.mlp.down_proj.forward_add_norm(a, residual, next_norm.weight, next_norm.eps)


class Qwen3Model(nn.Module):

    def __init__(self, config, quant_config=None):
        super().__init__()
        self.embed_tokens = ReplicatedEmbedding(config.vocab_size, config.hidden_size)
        self.layers = nn.ModuleList([Qwen3DecoderLayer(config, quant_config)
                                     for _ in range(config.num_hidden_layers)])
        self.norm = RMSNorm(config.hidden_size, eps=config.rms_norm_eps)

    def forward(self, input_ids, positions, aux_layer_ids=None):
        x = self.embed_tokens(input_ids)
        residual = x
        first = self.layers[0].input_layernorm
        h = norm_ops.rms_norm(x, first.weight, first.eps)
        aux = [None] * len(aux_layer_ids) if aux_layer_ids is not None else None
        n = len(self.layers)
        for i, layer in enumerate(self.layers):
            if aux_layer_ids is not None:
                for j, want in enumerate(aux_layer_ids):
                    if want == i:
                        # fused collectives return views of reusable buffers: keep a copy
                        aux[j] = residual.clone()
            next_norm = self.layers[i + 1].input_layernorm if i + 1 < n else self.norm
            h, residual = layer.forward_fused(positions, h, residual, next_norm)
        if aux_layer_ids is not None:
            if any(a is None for a in aux):
                raise ValueError(f"invalid aux_layer_ids: {aux_layer_ids}")
            return h, torch.cat(aux, dim=-1)
        return h


class Qwen3ForCausalLM(nn.Module):
    packed_modules_mapping = {
        "q_proj": ("qkv_proj", "q"),
        "k_proj": ("qkv_proj", "k"),
        "v_proj": ("qkv_proj", "v"),
        "gate_proj": ("gate_up_proj", 0),
        "up_proj": ("gate_up_proj", 1),
    }

    def __init__(self, config, quant_config=None):
        super().__init__()
        self.config = config
        self.model = Qwen3Model(config, quant_config)
        self.lm_head = ParallelLMHead(config.vocab_size, config.hidden_size)
        self.tie_word_embeddings = bool(config.tie_word_embeddings)
        self.eagle3_aux_layer_ids = tuple(get_eagle3_aux_layer_ids(config.num_hidden_layers))

    def post_load(self):
        """After weights are loaded: optional SiLU interleave of gate_up, then tile-pack every dense
        projection (and the untied LM head) for the sm_100a GEMM."""
        from llmserve_b200.layers.linear import LinearBase
        for layer in self.model.layers:
            layer.mlp.gate_up_proj.interleave_for_silu()
        for m in self.modules():
            if isinstance(m, LinearBase):
                m.pack_for_gemm()
        if not self.tie_word_embeddings:
            self.lm_head.pack_for_gemm()
        if torch.cuda.is_available():
            torch.cuda.empty_cache()

    def tie_weights(self):
        if self.tie_word_embeddings:
            w = self.model.embed_tokens.weight
            self.lm_head.weight.data = w.data.narrow(0, self.lm_head.vocab_start, self.lm_head.shard_size)

    def forward(self, input_ids, positions, aux_layer_ids=None):
        return self.model(input_ids, positions, aux_layer_ids=aux_layer_ids)

    def forward_with_eagle3_aux(self, input_ids, positions):
        return self.model(input_ids, positions, aux_layer_ids=self.eagle3_aux_layer_ids)

    def compute_logits(self, hidden_states, all_tokens: bool = False):
        """This rank's vocab shard of the logits."""
        return self.lm_head(hidden_states, all_tokens=all_tokens)
