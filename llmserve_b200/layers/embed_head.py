"""Token embedding and the vocab-parallel LM head.

The embedding table is replicated on every rank (1.2 GB for Qwen3-8B in bf16, small next to a
B200's HBM), which removes the reference's per-forward all-reduce of ``[T, H]``
(``llmserve/layers/embed_head.py:34-42``).  The LM head stays vocab-sharded: each rank produces
its logit shard; greedy decoding combines per-shard (max, index) pairs and only temperature
sampling gathers full rows (``embed_head.py:56-66`` gathers every row to rank 0).
"""
import os

import torch
from torch import nn

from llmserve_b200.ops import gemm, kv as kv_ops
from llmserve_b200.parallel import state as tp
from llmserve_b200.utils.context import get_context


class ReplicatedEmbedding(nn.Module):

    def __init__(self, num_embeddings: int, embedding_dim: int):
        super().__init__()
        self.num_embeddings = num_embeddings
        self.weight = nn.Parameter(torch.empty(num_embeddings, embedding_dim), requires_grad=False)
        self.weight.weight_loader = self.weight_loader

    def weight_loader(self, param, loaded):
        param.data.copy_(loaded)

    def forward(self, ids: torch.Tensor) -> torch.Tensor:
        return kv_ops.embedding(ids, self.weight)


class ParallelLMHead(nn.Module):

    def __init__(self, num_embeddings: int, embedding_dim: int):
        super().__init__()
        world, rank = tp.get_tp_size(), tp.get_tp_rank()
        if num_embeddings % world:
            raise ValueError("vocab size must be divisible by the tensor-parallel size")
        self.num_embeddings = num_embeddings
        self.shard_size = num_embeddings // world
        self.vocab_start = rank * self.shard_size
        self.weight = nn.Parameter(torch.empty(self.shard_size, embedding_dim), requires_grad=False)
        self.weight.weight_loader = self.weight_loader

    def weight_loader(self, param, loaded):
        param.data.copy_(loaded.narrow(0, self.vocab_start, self.shard_size))

    packed_weight = None

    @property
    def gemm_weight(self):
        return self.packed_weight if self.packed_weight is not None else self.weight

    def pack_for_gemm(self):
        """Tile-pack the (untied) head for the GEMM; see ``LinearBase.pack_for_gemm``."""
        if os.environ.get("LLMSERVE_PACK_WEIGHTS", "1") == "0" or not self.weight.is_cuda \
                or self.packed_weight is not None:
            return
        pw = gemm.pack_weight(self.weight.data)
        self.register_buffer("weight_tiles", pw.data, persistent=False)
        self.packed_weight = pw
        self.weight.data = torch.empty(0, dtype=self.weight.dtype, device=self.weight.device)

    def forward(self, x: torch.Tensor, all_tokens: bool = False) -> torch.Tensor:
        """Logit shard ``[rows, V / tp]``; in prefill only each sequence's last row."""
        ctx = get_context()
        if not all_tokens and ctx.is_prefill and ctx.last_token_indices is not None:
            x = x.index_select(0, ctx.last_token_indices)
        return gemm.linear(x, self.gemm_weight)
