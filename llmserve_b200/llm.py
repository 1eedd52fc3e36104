from llmserve_b200.engine.llm_engine import LLMEngine


class LLM(LLMEngine):
    """User-facing alias of :class:`LLMEngine` (``llmserve/llm.py:4-5`` of the reference)."""
