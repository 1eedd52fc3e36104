"""Checkpoint loading (HF safetensors) and synthetic weights.

``load_model`` follows ``llmserve/utils/loader.py:12-61`` of the reference: checkpoint names of
``q/k/v_proj`` and ``gate/up_proj`` are routed to the fused parameters with their shard id, each
parameter's ``weight_loader`` slices its tensor-parallel shard, missing tensors or shards raise,
and quantized layers are post-processed (AWQ repack) at the end.  Tied embeddings
(``tie_word_embeddings``) need no ``lm_head.weight`` in the checkpoint.

``init_dummy_weights`` draws N(0, std) weights directly on the device for the synthetic
benchmark configs (norm weights stay 1, AWQ tensors get uniform codes and |N(0,1)|*0.01 scales),
seeded per parameter name so replicated tensors agree across tensor-parallel ranks.
"""
import os
import zlib
from glob import glob

import torch
from safetensors import safe_open
from torch import nn


def default_weight_loader(param: nn.Parameter, loaded: torch.Tensor):
    param.data.copy_(loaded)


def _post_load(model: nn.Module):
    if hasattr(model, "tie_weights"):
        model.tie_weights()
    for module in model.modules():
        qm = getattr(module, "quant_method", None)
        if qm is not None:
            qm.process_weights_after_loading(module)
    if hasattr(model, "post_load"):
        model.post_load()


def load_model(model: nn.Module, path: str):
    packed = getattr(model, "packed_modules_mapping", {})
    tied = getattr(model, "tie_word_embeddings", False)
    loaded_ids: set[int] = set()
    loaded_shards: dict[int, set] = {}
    files = sorted(glob(os.path.join(path, "*.safetensors")))
    if not files:
        raise RuntimeError(f"no *.safetensors under {path}")
    for file in files:
        with safe_open(file, "pt", "cpu") as f:
            for name in f.keys():
                if tied and name == "lm_head.weight":
                    continue
                for src, (dst, shard_id) in packed.items():
                    if src in name:
                        param = model.get_parameter(name.replace(src, dst))
                        param.weight_loader(param, f.get_tensor(name), shard_id)
                        loaded_shards.setdefault(id(param), set()).add(shard_id)
                        break
                else:
                    param = model.get_parameter(name)
                    getattr(param, "weight_loader", default_weight_loader)(param, f.get_tensor(name))
                loaded_ids.add(id(param))
    missing = []
    for pname, param in model.named_parameters():
        if tied and pname == "lm_head.weight":
            continue
        expected = getattr(param, "expected_shard_ids", None)
        if expected is not None:
            got = loaded_shards.get(id(param), set())
            missing += [f"{pname}[{s}]" for s in expected if s not in got]
        elif id(param) not in loaded_ids:
            missing.append(pname)
    if missing:
        raise RuntimeError(f"missing checkpoint parameters or shards: {missing}")
    _post_load(model)


def seed_for(name: str, base: int) -> int:
    return (zlib.crc32(name.encode()) + 7919 * base) & 0x7FFFFFFF


@torch.no_grad()
def init_dummy_weights(model: nn.Module, seed: int = 0, std: float = 0.02):
    """Random-init every parameter on its current device (synthetic benchmarks)."""
    tied = getattr(model, "tie_word_embeddings", False)
    for name, p in model.named_parameters():
        if tied and name == "lm_head.weight":
            continue
        gen = torch.Generator(device=p.device)
        gen.manual_seed(seed_for(name, seed))
        if name.endswith("norm.weight"):
            p.data.fill_(1.0)
        elif p.dtype == torch.int32:
            lo = torch.randint(0, 1 << 16, p.shape, generator=gen, device=p.device, dtype=torch.int32)
            hi = torch.randint(0, 1 << 16, p.shape, generator=gen, device=p.device, dtype=torch.int32)
            p.data.copy_(lo | (hi << 16))
        elif name.endswith("scales"):
            p.data.copy_(torch.randn(p.shape, generator=gen, device=p.device, dtype=torch.float32)
                         .abs_().mul_(0.01).to(p.dtype))
        else:
            p.data.copy_(torch.randn(p.shape, generator=gen, device=p.device, dtype=torch.float32)
                         .mul_(std).to(p.dtype))
    _post_load(model)
