"""Engine configuration.

Field names and defaults follow ``llmserve/config.py:8-33`` of the reference so that
``LLM(model, **kwargs)`` accepts the same keyword set.  Fields added by this framework
are grouped at the end:

* ``device``               -- ``"cuda"`` (B200 path) or ``"cpu"`` (fp32 oracle path used by
                              the CPU test tier; runs TP over gloo ranks).
* ``load_format``          -- ``"auto"`` reads HF safetensors; ``"dummy"`` draws random
                              N(0, 0.02) weights on the device (synthetic benchmarks).
* ``fused_collectives``    -- use the in-kernel NVLink all-reduce (+residual+RMSNorm) instead
                              of NCCL for the row-parallel layers; NCCL stays as the baseline.
* ``comm_timeout_s``       -- bound on every host RPC wait and on the process-group timeout.
* ``debug_bounds_checks``  -- validate slot mappings / block tables on the host before launch.
* ``pd_*``                 -- prefill/decode disaggregation (prefill group pushes KV blocks).
* ``distributed_launcher`` -- ``"spawn"``: rank 0 starts the TP workers itself (reference
                              behaviour); ``"external"``: ranks were started by torchrun and
                              ranks > 0 call :func:`llmserve_b200.engine.llm_engine.run_worker`.
* ``overlap_decode``       -- launch decode step N+1 from device-resident tokens before step N is
                              read on the host (greedy, graph decode); on by default.
* ``speculative_cuda_graphs`` -- capture the greedy EAGLE3 chain step (drafts, packed verify,
                              acceptance) in CUDA graphs per batch bucket; off by default.

``awq_backend="triton"`` is accepted for compatibility and runs the sm_100a W4A16 kernel.
"""
import json
import os
from dataclasses import dataclass, field, replace

import torch

from llmserve_b200.quantization.awq import AWQRuntimeConfig


_DTYPES = {"bfloat16": torch.bfloat16, "float16": torch.float16, "float32": torch.float32}


class HFConfig:
    """Minimal stand-in for ``transformers.AutoConfig`` built from ``config.json``.

    Attribute access mirrors the HF config object for the fields the engine reads, so a
    synthetic checkpoint directory needs nothing but ``config.json``.
    """

    def __init__(self, raw: dict):
        self._raw = dict(raw)
        for key, value in raw.items():
            setattr(self, key, value)
        dtype = raw.get("dtype", raw.get("torch_dtype", "bfloat16"))
        self.dtype = _DTYPES[dtype] if isinstance(dtype, str) else dtype
        self.torch_dtype = self.dtype
        self.head_dim = raw.get("head_dim") or raw["hidden_size"] // raw["num_attention_heads"]
        self.tie_word_embeddings = raw.get("tie_word_embeddings", False)
        self.attention_bias = raw.get("attention_bias", False)
        self.rope_theta = raw.get("rope_theta", 1000000.0)
        self.rope_scaling = raw.get("rope_scaling")
        self.rms_norm_eps = raw.get("rms_norm_eps", 1e-6)
        self.hidden_act = raw.get("hidden_act", "silu")
        self.max_position_embeddings = raw.get("max_position_embeddings", 40960)
        self.quantization_config = raw.get("quantization_config")

    def to_dict(self) -> dict:
        return dict(self._raw)

    @classmethod
    def from_pretrained(cls, path: str) -> "HFConfig":
        with open(os.path.join(path, "config.json")) as f:
            return cls(json.load(f))


@dataclass(slots=True)
class Config:
    model: str
    max_num_batched_tokens: int = 16384
    max_num_seqs: int = 512
    max_model_len: int = 4096
    gpu_memory_utilization: float = 0.9
    tensor_parallel_size: int = 1
    distributed_init_method: str = "tcp://127.0.0.1:2333"
    enforce_eager: bool = False
    awq_backend: str = "cuda"
    enable_chunked_prefill: bool = False
    enable_kv_capacity_admission: bool = False
    speculative_model: str | None = None
    speculative_gamma: int = 3
    speculative_tree_nodes: int = 0
    speculative_accept_mode: str = "greedy"
    speculative_trace: bool = False
    hf_config: HFConfig | None = None
    quant_config: AWQRuntimeConfig | None = field(init=False, default=None)
    eos: int = -1
    kvcache_block_size: int = 256
    num_kvcache_blocks: int = -1
    # ---- additions of this framework ----
    device: str = "cuda"
    load_format: str = "auto"
    seed: int = 0
    fused_collectives: bool = True
    comm_timeout_s: float = 120.0
    debug_bounds_checks: bool = False
    pd_disaggregation: bool = False
    pd_prefill_devices: tuple[int, ...] = ()
    pd_decode_devices: tuple[int, ...] = ()
    device_offset: int = 0
    max_kvcache_blocks: int = -1
    distributed_launcher: str = "spawn"
    rpc_channel: str | None = None
    overlap_decode: bool = True
    speculative_cuda_graphs: bool = False
    pd_role: str = ""          # internal: "decode" exports its KV pools to the prefill ranks

    def __post_init__(self):
        if not os.path.isdir(self.model):
            raise ValueError(f"model path is not a directory: {self.model}")
        if self.kvcache_block_size % 16:
            raise ValueError("kvcache_block_size must be a multiple of 16")
        if not 1 <= self.tensor_parallel_size <= 8:
            raise ValueError("tensor_parallel_size must be in [1, 8]")
        if self.speculative_gamma <= 0:
            raise ValueError("speculative_gamma must be positive")
        if self.speculative_tree_nodes not in (0, 6, 10):
            raise ValueError("speculative_tree_nodes must be 0, 6 or 10")
        if self.speculative_accept_mode not in ("greedy", "rejection"):
            raise ValueError("speculative_accept_mode must be 'greedy' or 'rejection'")
        if self.speculative_tree_nodes:
            if self.speculative_gamma != 3 or self.speculative_accept_mode != "greedy":
                raise ValueError("tree speculation requires gamma=3 and greedy acceptance")
            if self.speculative_model is None:
                raise ValueError("tree speculation requires a speculative_model")
        if self.awq_backend not in ("reference", "triton", "cuda"):
            raise ValueError("awq_backend must be 'reference', 'triton', or 'cuda'")
        if self.awq_backend == "triton":
            # the reference's Triton W4A16 kernels are replaced by the sm_100a kernel here
            self.awq_backend = "cuda"
        if self.device not in ("cuda", "cpu"):
            raise ValueError("device must be 'cuda' or 'cpu'")
        if self.distributed_launcher not in ("spawn", "external"):
            raise ValueError("distributed_launcher must be 'spawn' or 'external'")
        if self.load_format not in ("auto", "dummy"):
            raise ValueError("load_format must be 'auto' or 'dummy'")
        if self.speculative_model is not None and not os.path.isdir(self.speculative_model):
            raise ValueError(f"speculative model path is not a directory: {self.speculative_model}")
        if self.hf_config is None:
            self.hf_config = HFConfig.from_pretrained(self.model)
        if getattr(self.hf_config, "quantization_config", None) is not None:
            self.quant_config = replace(
                AWQRuntimeConfig.from_hf_config(self.hf_config),
                execution_backend=self.awq_backend,
            )
        self.max_model_len = min(self.max_model_len, self.hf_config.max_position_embeddings)
        if self.pd_disaggregation:
            if not self.pd_prefill_devices or not self.pd_decode_devices:
                raise ValueError("pd_disaggregation needs pd_prefill_devices and pd_decode_devices")
            if len(self.pd_prefill_devices) != len(self.pd_decode_devices):
                raise ValueError("prefill and decode groups must have the same TP degree")
