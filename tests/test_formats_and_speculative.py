"""Checkpoint formats (AutoAWQ GEMM g128, EAGLE3 RedHat / SpecForge, HF Qwen3 loading with TP
slicing) and the speculative acceptance algorithms, against the reference where importable."""
import json
import os
from types import SimpleNamespace

import pytest
import torch

from llmserve_b200.models.eagle3 import (Eagle3Speculator, normalize_eagle3_config, normalize_eagle3_weight_name,
                                         validate_eagle3_target_config)
from llmserve_b200.models.synthetic import TINY, awq_quantize_dense, write_eagle3_checkpoint
from llmserve_b200.quantization.awq import (AWQRuntimeConfig, awq_reference_linear, dequantize_awq_gemm,
                                            pack_awq_int4, unpack_awq_int4)
from llmserve_b200.speculative.sampling import (greedy_accept_batch, greedy_accept_from_ids,
                                                speculative_accept_greedy_from_logits, speculative_accept_reject)
from llmserve_b200.speculative.tree import build_fixed_tree_topology, select_greedy_tree_path
from tests.support import reference_module


# ---- AWQ -------------------------------------------------------------------------------------
def test_awq_pack_unpack_roundtrip_and_reference_order():
    ref = reference_module("llmserve.layers.quantization.awq")
    codes = torch.randint(0, 16, (32, 64), dtype=torch.int32)
    packed = pack_awq_int4(codes)
    assert torch.equal(unpack_awq_int4(packed), codes)
    assert torch.equal(ref.unpack_awq_int4(packed), codes)
    qz = pack_awq_int4(torch.randint(0, 16, (1, 64), dtype=torch.int32).repeat(1, 1))
    qw = pack_awq_int4(torch.randint(0, 16, (128, 64), dtype=torch.int32))
    sc = torch.rand(1, 64).bfloat16()
    assert torch.equal(dequantize_awq_gemm(qw, qz, sc, group_size=128), ref.dequantize_awq_gemm(qw, qz, sc, group_size=128))


def test_awq_rtn_quantization_is_close():
    w = torch.randn(256, 512) * 0.02
    qw, qz, sc = awq_quantize_dense(w)
    deq = dequantize_awq_gemm(qw, qz, sc, group_size=128).float().t()
    assert ((deq - w).norm() / w.norm()).item() < 0.12
    x = torch.randn(4, 512).bfloat16()
    y = awq_reference_linear(x, qw, qz, sc, group_size=128)
    assert y.shape == (4, 256)


def test_awq_config_validation():
    good = SimpleNamespace(dtype=torch.bfloat16, quantization_config=dict(
        quant_method="awq", backend="autoawq", bits=4, group_size=128, version="gemm", zero_point=True))
    assert AWQRuntimeConfig.from_hf_config(good).pack_factor == 8
    for key, bad in (("bits", 8), ("group_size", 64), ("version", "gemv"), ("zero_point", False)):
        cfg = SimpleNamespace(dtype=torch.bfloat16, quantization_config=dict(good.quantization_config, **{key: bad}))
        with pytest.raises(ValueError, match=key):
            AWQRuntimeConfig.from_hf_config(cfg)


def test_awq_checkpoint_loads_with_tp_slicing_on_cpu(tmp_path):
    """AutoAWQ checkpoint through the engine loader; TP=2 shards of a packed layer concatenate back."""
    from llmserve_b200.layers.linear import RowParallelLinear
    from llmserve_b200.parallel import state as tp
    cfg = AWQRuntimeConfig(4, 128, True, "gemm", "autoawq", torch.bfloat16)
    w = torch.randn(512, 256) * 0.02
    qw, qz, sc = awq_quantize_dense(w)
    shards = []
    for rank in range(2):
        tp._tp.rank, tp._tp.world_size = rank, 2
        try:
            lin = RowParallelLinear(256, 512, quant_config=cfg)
            for name, t in (("qweight", qw), ("qzeros", qz), ("scales", sc)):
                p = getattr(lin, name)
                p.weight_loader(p, t)
            shards.append(lin.qweight.data.clone())
        finally:
            tp._tp.rank, tp._tp.world_size = 0, 1
    assert torch.equal(torch.cat(shards, 0), qw)


# ---- EAGLE3 ----------------------------------------------------------------------------------
def test_eagle3_config_and_name_normalization_match_reference():
    ref = reference_module("llmserve.models.eagle3")
    nested = json.load(open(os.path.join(write_eagle3_checkpoint("/tmp/lsb_e3_nested", TINY, 512), "config.json")))
    assert normalize_eagle3_config(nested) == ref.normalize_eagle3_config(nested)
    with pytest.raises(ValueError, match="conflicting"):
        normalize_eagle3_config({"hidden_size": 1, "transformer_layer_config": {"hidden_size": 2}})
    for name in ("layers.0.self_attn.q_proj.weight", "fc.weight", "midlayer.mlp.up_proj.weight"):
        assert normalize_eagle3_weight_name(name) == ref.normalize_eagle3_weight_name(name)
    with pytest.raises(ValueError, match="vocab_size"):
        validate_eagle3_target_config(normalize_eagle3_config(nested), dict(TINY, vocab_size=5))


@pytest.mark.parametrize("nested", [True, False])
def test_eagle3_loads_redhat_and_specforge_layouts(tmp_path, nested):
    from llmserve_b200.models.synthetic import write_qwen3_checkpoint
    tgt = write_qwen3_checkpoint(str(tmp_path / "t"), TINY)
    d = write_eagle3_checkpoint(str(tmp_path / "d"), TINY, 512, nested=nested)
    m = Eagle3Speculator.from_pretrained(d, target_model_path=tgt)
    from safetensors import safe_open
    with safe_open(os.path.join(tgt, "model-00001-of-00001.safetensors"), "pt") as f:
        assert torch.equal(m.embed_tokens.weight.data, f.get_tensor("model.embed_tokens.weight"))
    logits = torch.zeros(2, 512)
    logits[0, 5] = 1
    logits[1, 100] = 1
    ids = m.greedy_sample(logits)
    assert ids.tolist() == [5 + int(m.d2t[5]), 100 + int(m.d2t[100])]
    mapped = m.map_draft_logits(logits)
    assert mapped.shape == (2, 1024) and torch.isinf(mapped).sum() == 2 * (1024 - 512)


def test_eagle3_missing_embedding_without_target_raises(tmp_path):
    d = write_eagle3_checkpoint(str(tmp_path / "d"), TINY, 512)
    with pytest.raises(ValueError, match="target_model_path"):
        Eagle3Speculator.from_pretrained(d)


# ---- acceptance ------------------------------------------------------------------------------
def test_greedy_acceptance_matches_reference():
    ref = reference_module("llmserve.speculative.sampling")
    g = torch.Generator().manual_seed(0)
    for _ in range(50):
        logits = torch.randn(4, 9, generator=g)
        target = logits.argmax(-1)
        drafts = target[:3].clone()
        k = int(torch.randint(0, 4, (1,), generator=g))
        if k < 3:
            drafts[k] = (drafts[k] + 1) % 9
        a = speculative_accept_greedy_from_logits(logits, drafts)
        b = ref.speculative_accept_greedy_from_logits(logits, drafts)
        assert (a.token_ids, a.num_accepted, a.accepted_all) == (b.token_ids, b.num_accepted, b.accepted_all)
        acc, fin = greedy_accept_batch(target.view(1, 4), drafts.view(1, 3))
        assert int(acc[0]) == a.num_accepted and int(fin[0]) == a.final_token_id


def test_rejection_sampling_preserves_target_distribution():
    torch.manual_seed(0)
    p = torch.tensor([[0.5, 0.3, 0.2], [0.2, 0.2, 0.6]])
    q = torch.tensor([[0.2, 0.6, 0.2]])
    counts = torch.zeros(3)
    n = 20000
    for _ in range(n):
        draft = torch.multinomial(q[0], 1)
        res = speculative_accept_reject(p, q, draft)
        counts[res.token_ids[0]] += 1
    assert torch.allclose(counts / n, p[0], atol=0.015)


def test_tree_path_selection_matches_reference():
    ref = reference_module("llmserve.speculative.tree")
    for nodes in (6, 10):
        topo = build_fixed_tree_topology(nodes)
        rt = ref.build_fixed_tree_topology(nodes)
        assert torch.equal(topo.attention_mask(), rt.attention_mask())
        g = torch.Generator().manual_seed(nodes)
        for _ in range(30):
            logits = torch.randn(len(topo.parents), 5, generator=g)
            drafts = torch.randint(0, 5, (nodes,), generator=g).tolist()
            a = select_greedy_tree_path(topo, drafts, logits.argmax(-1).tolist())
            b = ref.select_greedy_tree_path(rt, drafts, logits)
            assert (a.token_ids, a.commit_node_indices, a.final_node_index, a.accepted_all) == \
                (b.token_ids, b.commit_node_indices, b.final_node_index, b.accepted_all)


def test_greedy_from_ids_bonus():
    r = greedy_accept_from_ids([1, 2, 3, 4], [1, 2, 3])
    assert r.token_ids == [1, 2, 3, 4] and r.accepted_all


def test_pack_weight_layout_roundtrip():
    """Packed GEMM weights: tile (m, kt) is 128 rows of 64 elements whose 16-byte chunks are
    XOR-swizzled by row; unpacking restores the weight exactly (padding dropped)."""
    from llmserve_b200.ops import gemm
    w = torch.arange(300 * 136, dtype=torch.float32).view(300, 136).to(torch.bfloat16)
    pw = gemm.pack_weight(w)
    assert pw.shape == (300, 136)
    assert pw.data.shape == (512 // 128 * 3 * 128, 64)        # rows padded to 512, K to 192
    assert torch.equal(pw.unpack(), w)
    wp = torch.zeros(512, 192, dtype=torch.bfloat16)
    wp[:300, :136] = w
    kt_count = 3
    for m, kt, r, p in [(0, 0, 0, 0), (1, 2, 5, 3), (2, 1, 127, 7), (3, 0, 9, 1)]:
        row = (m * kt_count + kt) * 128 + r
        logical_chunk = p ^ (r & 7)
        expect = wp[m * 128 + r, kt * 64 + logical_chunk * 8: kt * 64 + logical_chunk * 8 + 8]
        assert torch.equal(pw.data[row, p * 8: p * 8 + 8], expect)


def test_awq_repack_matches_autoawq_dequant():
    """The load-time repack for the W4A16 kernel keeps every (q - z) * s of the AutoAWQ tensors."""
    from llmserve_b200.ops import awq as awq_ops
    from llmserve_b200.quantization.awq import dequantize_awq_gemm
    g = torch.Generator().manual_seed(3)
    w = torch.randn(200, 384, generator=g) * 0.05
    qw, qz, sc = awq_quantize_dense(w)
    ref = dequantize_awq_gemm(qw, qz, sc.bfloat16(), group_size=128)
    packed = awq_ops.prepare_awq_weights(qw, qz, sc.bfloat16(), 128)
    assert packed.qtiles.shape == (2, 6, 128, 8) and packed.sztiles.shape == (2, 3, 128, 2)
    assert torch.equal(awq_ops.dequantize_packed(packed), ref.t().contiguous())


def test_packed_greedy_accept_matches_per_sequence_rule():
    from llmserve_b200.speculative.sampling import greedy_accept_packed
    g = torch.Generator().manual_seed(4)
    draft = torch.randint(0, 4, (50, 3), generator=g)
    target = torch.randint(0, 4, (50, 4), generator=g)
    start = torch.arange(50)
    packed = greedy_accept_packed(target, draft, start)
    for i in range(50):
        r = greedy_accept_from_ids(target[i].tolist(), draft[i].tolist())
        assert packed[i, 0] == r.num_accepted and packed[i, 1] == r.final_token_id
        assert packed[i, 2] == i and packed[i, 3:].tolist() == draft[i].tolist()


def test_nvtx_ranges_are_noops_when_disabled_or_without_cuda(monkeypatch):
    from llmserve_b200.utils import nvtx
    with nvtx.nvtx_range("x"):
        pass
    monkeypatch.setattr(nvtx, "ENABLED", True)
    with nvtx.nvtx_range("x"):          # no CUDA here: still a no-op
        pass


def test_engine_imports_without_triton_flash_attn_or_vllm():
    """The engine never needs Triton, flash-attn, FlashInfer or vLLM (reference test:
    ``tests/test_optional_dependencies.py``)."""
    import subprocess
    import sys
    code = ("import sys\n"
            "for m in ('triton', 'flash_attn', 'flashinfer', 'vllm'): sys.modules[m] = None\n"
            "import llmserve_b200, llmserve_b200.engine.llm_engine, llmserve_b200.engine.pd_engine\n"
            "import llmserve_b200.quantization.awq_calibration, benchmarks.serve\n"
            "from llmserve_b200 import LLM, SamplingParams\n")
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    r = subprocess.run([sys.executable, "-c", code], cwd=root, capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr[-2000:]


# ---- tree K/V commit manager -------------------------------------------------------------------
class _TreeLayer:
    def __init__(self, values):
        self.tree_k = torch.tensor(values, dtype=torch.float32).view(-1, 1, 1)
        self.tree_v = self.tree_k + 10


def test_tree_kv_manager_validates_and_always_clears():
    from llmserve_b200.speculative.tree_kv import TreeKVCacheManager
    layers = [_TreeLayer([1, 2, 3]), _TreeLayer([4, 5])]
    with pytest.raises(ValueError, match="same shape"):
        TreeKVCacheManager(layers).commit([0], torch.tensor([4], dtype=torch.int32))
    assert all(layer.tree_k.numel() == 0 and layer.tree_v.numel() == 0 for layer in layers)
    layer = _TreeLayer([1, 2, 3])
    manager = TreeKVCacheManager([layer])
    with pytest.raises(ValueError, match="slot count"):
        manager.commit([0, 2], torch.tensor([4], dtype=torch.int32))
    layer.tree_k = torch.tensor([1.0, 2.0, 3.0]).view(-1, 1, 1)
    layer.tree_v = layer.tree_k + 10
    with pytest.raises(ValueError, match="node index"):
        manager.commit([0, 3], torch.tensor([4, 5], dtype=torch.int32))
    assert layer.tree_k.numel() == 0
    with pytest.raises(ValueError, match="capture"):
        manager.commit([0], torch.tensor([4], dtype=torch.int32))
    with pytest.raises(ValueError):
        TreeKVCacheManager([])


def test_tree_kv_manager_commits_selected_nodes_of_every_layer():
    from llmserve_b200.speculative.tree_kv import TreeKVCacheManager
    layers = [_TreeLayer([1, 2, 3]), _TreeLayer([4, 5, 6])]
    k_cache = torch.zeros(2, 2, 1, 4, 1)                 # [layers, blocks, kv_heads, block_size, head_dim]
    v_cache = torch.zeros_like(k_cache)
    TreeKVCacheManager(layers, k_cache=k_cache, v_cache=v_cache).commit([0, 2], torch.tensor([5, 6], dtype=torch.int32))
    assert k_cache[:, 1, 0, 1:3, 0].tolist() == [[1.0, 3.0], [4.0, 6.0]]
    assert v_cache[:, 1, 0, 1:3, 0].tolist() == [[11.0, 13.0], [14.0, 16.0]]
    assert k_cache[:, 0].abs().sum() == 0
    assert all(layer.tree_k.numel() == 0 for layer in layers)


# ---- Qwen3 auxiliary hidden states for EAGLE3 ----------------------------------------------------
def test_eagle3_aux_layers_are_the_residual_streams_entering_the_chosen_layers():
    from torch import nn

    from llmserve_b200.models.qwen3 import Qwen3Model, get_eagle3_aux_layer_ids
    assert get_eagle3_aux_layer_ids(36) == (2, 18, 33)
    assert get_eagle3_aux_layer_ids(2) == (0, 1, 1)

    class Norm(nn.Module):
        def __init__(self):
            super().__init__()
            self.weight, self.eps = nn.Parameter(torch.ones(4), requires_grad=False), 1e-6

    class Layer(nn.Module):
        def __init__(self, i):
            super().__init__()
            self.i, self.input_layernorm = i, Norm()

        def forward_fused(self, positions, h, residual, next_norm):
            stream = residual + (self.i + 1)              # layer i adds i + 1 to the stream
            return h * 0 + self.i, stream

    model = Qwen3Model.__new__(Qwen3Model)
    nn.Module.__init__(model)
    model.embed_tokens = lambda ids: torch.full((ids.numel(), 4), 100.0)
    model.layers = nn.ModuleList(Layer(i) for i in range(8))
    model.norm = Norm()
    ids, pos = torch.tensor([1, 2, 3]), torch.tensor([0, 1, 2])
    plain = model(ids, pos)
    hidden, aux = model(ids, pos, aux_layer_ids=(2, 5, 5))
    assert torch.equal(hidden, plain)
    entering = {i: 100.0 + sum(k + 1 for k in range(i)) for i in range(8)}
    expected = torch.cat([torch.full((3, 4), entering[i]) for i in (2, 5, 5)], dim=-1)
    assert torch.equal(aux, expected)                      # concatenation order kept, duplicates kept
    with pytest.raises(ValueError, match="aux_layer_ids"):
        model(ids, pos, aux_layer_ids=(2, 5, 9))


def test_config_fields_and_defaults_cover_the_reference():
    """Every ``Config`` field of the reference exists here with the same default, so the same
    ``LLM(model, **kwargs)`` calls work.  The one deliberate difference: the default rendezvous
    address is 127.0.0.1 instead of ``localhost`` (a container's host name may not resolve)."""
    import dataclasses

    from llmserve_b200.config import Config
    ref = reference_module("llmserve.config")
    ours = {f.name: f for f in dataclasses.fields(Config)}
    for f in dataclasses.fields(ref.Config):
        assert f.name in ours, f.name
        if f.name in ("hf_config", "quant_config"):
            continue
        want = f.default if f.default is not dataclasses.MISSING else None
        got = ours[f.name].default if ours[f.name].default is not dataclasses.MISSING else None
        if f.name == "distributed_init_method":
            assert want == "tcp://localhost:2333" and got == "tcp://127.0.0.1:2333"
            continue
        assert got == want, f.name
        assert ours[f.name].init == f.init, f.name


@pytest.mark.parametrize("nodes", [6, 10])
def test_tree_attention_equals_reference_tree_path(nodes):
    """Prefix in a paged pool (shuffled blocks) + tree nodes under the ancestor mask: the host
    reference of the tree-attention kernel equals the reference engine's masked-SDPA tree path."""
    from llmserve_b200.ops.attention import tree_attention_ref
    ref_attn = reference_module("llmserve.layers.attention")
    ref_ctx = reference_module("llmserve.utils.context")
    topo = build_fixed_tree_topology(nodes)
    n, nh, nkv, hd, bs, P = len(topo.parents), 8, 2, 16, 16, 37
    g = torch.Generator().manual_seed(nodes)
    pk, pv = torch.randn(P, nkv, hd, generator=g), torch.randn(P, nkv, hd, generator=g)
    q = torch.randn(n, nh, hd, generator=g)
    tk, tv = torch.randn(n, nkv, hd, generator=g), torch.randn(n, nkv, hd, generator=g)
    nblocks = 6
    table = torch.tensor([4, 1, 3], dtype=torch.int32)
    ours_k = torch.zeros(nblocks, nkv, bs, hd)
    ours_v = torch.zeros_like(ours_k)
    theirs_k = torch.zeros(nblocks, bs, nkv, hd)
    theirs_v = torch.zeros_like(theirs_k)
    slots = []
    for p in range(P):
        b, o = int(table[p // bs]), p % bs
        ours_k[b, :, o], ours_v[b, :, o] = pk[p], pv[p]
        theirs_k[b, o], theirs_v[b, o] = pk[p], pv[p]
        slots.append(b * bs + o)
    mask = topo.attention_mask()
    ours = tree_attention_ref(q, ours_k, ours_v, table, P, tk, tv, mask, hd ** -0.5)
    layer = ref_attn.Attention(nh, hd, hd ** -0.5, nkv)
    layer.k_cache, layer.v_cache = theirs_k, theirs_v
    ref_ctx.set_context(True, tree_prefix_slots=torch.tensor(slots), tree_attention_mask=mask)
    try:
        theirs = layer(q, tk, tv)
    finally:
        ref_ctx.reset_context()
    torch.testing.assert_close(ours, theirs, atol=1e-5, rtol=1e-5)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_norm_rope_and_silu_host_references_equal_the_reference_layers(dtype):
    """The host references that the sm_100a kernels are tested against compute what the reference's
    layers compute (RMSNorm, fused add + RMSNorm with the bf16 residual, neox RoPE from the
    cos/sin cache, SiLU-mul), run here with the reference's ``torch.compile`` switched off."""
    import torch._dynamo

    from llmserve_b200.ops.activation import silu_and_mul_ref
    from llmserve_b200.ops.norm import add_rms_norm_ref, rms_norm_ref
    from llmserve_b200.ops.rope import apply_rope_ref, build_cos_sin_cache
    ln = reference_module("llmserve.layers.layernorm")
    rope = reference_module("llmserve.layers.rotary_embedding")
    act = reference_module("llmserve.layers.activation")
    g = torch.Generator().manual_seed(3)
    x = torch.randn(5, 64, generator=g).to(dtype)
    res = torch.randn(5, 64, generator=g).to(dtype)
    w = (1 + 0.1 * torch.randn(64, generator=g)).to(dtype)
    norm = ln.RMSNorm(64, eps=1e-6).to(dtype)
    norm.weight.data.copy_(w)
    pos = torch.tensor([0, 3, 17, 200, 4095])
    q = torch.randn(5, 4, 128, generator=g).to(dtype)
    k = torch.randn(5, 2, 128, generator=g).to(dtype)
    emb = rope.RotaryEmbedding(128, 128, 4096, 1000000.0)
    cs = build_cos_sin_cache(128, 4096, 1000000.0)
    gate_up = torch.randn(5, 2 * 96, generator=g).to(dtype)
    saved = torch._dynamo.config.disable
    torch._dynamo.config.disable = True
    try:
        with torch.no_grad():
            ref_n = norm(x.clone())
            ref_an, ref_res = norm(x.clone(), res.clone())
            ref_q, ref_k = emb(pos, q, k)
            ref_act = act.SiluAndMul()(gate_up)
    finally:
        torch._dynamo.config.disable = saved
    tol = dict(atol=1e-5, rtol=1e-5) if dtype == torch.float32 else dict(atol=2e-2, rtol=2e-2)
    torch.testing.assert_close(rms_norm_ref(x, w, 1e-6), ref_n, **tol)
    an, r = add_rms_norm_ref(x, res, w, 1e-6)
    torch.testing.assert_close(an, ref_an, **tol)
    if dtype == torch.bfloat16:
        # (with fp32 activations the reference's in-place ops alias its returned residual with the
        # normalised output -- ``x.float()`` is ``x`` itself -- so only the bf16 residual compares)
        torch.testing.assert_close(r, ref_res, **tol)
    torch.testing.assert_close(apply_rope_ref(q, pos, cs), ref_q, **tol)
    torch.testing.assert_close(apply_rope_ref(k, pos, cs), ref_k, **tol)
    torch.testing.assert_close(silu_and_mul_ref(gate_up), ref_act, **tol)
