"""NVTX ranges for timeline tools (``LLMSERVE_NVTX=1``): engine steps and their phases, and the
stages of a speculative step.  A no-op unless the variable is set and CUDA is available."""
import contextlib
import os

ENABLED = os.environ.get("LLMSERVE_NVTX", "0") == "1"


def nvtx_range(name: str):
    if not ENABLED:
        return contextlib.nullcontext()
    import torch
    if not torch.cuda.is_available():
        return contextlib.nullcontext()
    return torch.cuda.nvtx.range(name)
