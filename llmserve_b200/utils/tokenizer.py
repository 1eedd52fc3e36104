"""Tokenizer access.

Uses ``transformers.AutoTokenizer`` when the model directory carries tokenizer files, as the
reference does (``llmserve/engine/llm_engine.py:36-37``).  Synthetic checkpoints (random weights,
no tokenizer) get :class:`ByteTokenizer`: UTF-8 bytes shifted past the special ids, so prompts
given as strings still work and token-id prompts pass through unchanged.
"""
import os


class ByteTokenizer:
    offset = 3

    def __init__(self, vocab_size: int, eos_token_id: int = 2):
        self.vocab_size = vocab_size
        self.eos_token_id = eos_token_id

    def encode(self, text: str) -> list[int]:
        return [(b + self.offset) % self.vocab_size for b in text.encode("utf-8")]

    def decode(self, ids) -> str:
        data = bytes((int(i) - self.offset) % 256 for i in ids if int(i) >= self.offset)
        return data.decode("utf-8", errors="replace")


def load_tokenizer(model_path: str, hf_config):
    names = ("tokenizer.json", "tokenizer.model", "tokenizer_config.json", "vocab.json")
    if any(os.path.exists(os.path.join(model_path, n)) for n in names):
        from transformers import AutoTokenizer
        return AutoTokenizer.from_pretrained(model_path, use_fast=True)
    eos = getattr(hf_config, "eos_token_id", 2)
    if isinstance(eos, list):
        eos = eos[0]
    return ByteTokenizer(hf_config.vocab_size, eos if eos is not None else 2)
