"""Per-forward attention metadata, set by the runner and read by the attention layers.

Field set of ``llmserve/utils/context.py:5-18`` of the reference plus what the paged kernels
need: ``seqlens_k`` (keys per sequence, int32), ``decode_workspace`` (split-KV scratch),
``last_token_indices`` (LM-head row selection), the tree-verify / tree-draft inputs and
``uniform_q`` (a verify chunk of equal length per sequence, run on the decode kernel).
"""
from dataclasses import dataclass

import torch


@dataclass(slots=True)
class Context:
    is_prefill: bool = False
    cu_seqlens_q: torch.Tensor | None = None
    cu_seqlens_k: torch.Tensor | None = None
    max_seqlen_q: int = 0
    max_seqlen_k: int = 0
    slot_mapping: torch.Tensor | None = None
    context_lens: torch.Tensor | None = None
    block_tables: torch.Tensor | None = None
    tree_prefix_slots: torch.Tensor | None = None
    tree_attention_mask: torch.Tensor | None = None
    seqlens_k: torch.Tensor | None = None
    last_token_indices: torch.Tensor | None = None
    decode_workspace: object | None = None
    tree_prefix_len: int = 0
    tree_block_table: torch.Tensor | None = None
    tree_mask_bits: torch.Tensor | None = None
    tree_rows: list | None = None
    tree_side_k: torch.Tensor | None = None
    tree_side_v: torch.Tensor | None = None
    # > 0: a packed verify chunk with exactly this many query rows per sequence (prefill mode)
    uniform_q: int = 0


_CONTEXT = Context()


def get_context() -> Context:
    return _CONTEXT


def set_context(is_prefill, cu_seqlens_q=None, cu_seqlens_k=None, max_seqlen_q=0, max_seqlen_k=0,
                slot_mapping=None, context_lens=None, block_tables=None, tree_prefix_slots=None,
                tree_attention_mask=None, **extra):
    global _CONTEXT
    _CONTEXT = Context(is_prefill, cu_seqlens_q, cu_seqlens_k, max_seqlen_q, max_seqlen_k, slot_mapping,
                       context_lens, block_tables, tree_prefix_slots, tree_attention_mask, **extra)
    return _CONTEXT


def reset_context():
    global _CONTEXT
    _CONTEXT = Context()
