"""B200-native LLM serving engine (sm_100a kernels, NVLink tensor parallelism).

Public API parity with HGinkgo/LLM-Serve: ``LLM(model, **config).generate(prompts, params)``.
"""
from llmserve_b200.sampling_params import SamplingParams


def __getattr__(name):
    # The engine pulls in torch.distributed and the runner; import it lazily so that
    # ``from llmserve_b200 import SamplingParams`` stays cheap.
    if name in ("LLM", "LLMEngine"):
        from llmserve_b200.llm import LLM
        from llmserve_b200.engine.llm_engine import LLMEngine
        return {"LLM": LLM, "LLMEngine": LLMEngine}[name]
    raise AttributeError(name)


__all__ = ["LLM", "LLMEngine", "SamplingParams"]
