"""Token embedding and the vocab-parallel LM head.

The embedding table is replicated on every rank (1.2 GB for Qwen3-8B in bf16, small next to a
B200's HBM), which removes the reference's per-forward all-reduce of ``[T, H]``
(``llmserve/layers/embed_head.py:34-42``).  The LM head stays vocab-sharded: each rank produces
its logit shard; greedy decoding combines per-shard (max, index) pairs and only temperature
sampling gathers full rows (``embed_head.py:56-66`` gathers every row to rank 0).
"""
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

    def forward(self, x: torch.Tensor, all_tokens: bool = False) -> torch.Tensor:
        """Logit shard ``[rows, V / tp]``; in prefill only each sequence's last row."""
        ctx = get_context()
        if not all_tokens and ctx.is_prefill and ctx.last_token_indices is not None:
            x = x.index_select(0, ctx.last_token_indices)
        return gemm.linear(x, self.weight)
