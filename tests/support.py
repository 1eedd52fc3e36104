"""Test helpers: the reference implementation as an oracle (read-only import), tiny checkpoints."""
import importlib
import os
import sys

import pytest

# the reference checkout named by LLMSERVE_REFERENCE_PATH, else its package installed under baseline/_ref
_REF_CANDIDATES = [os.environ.get("LLMSERVE_REFERENCE_PATH", ""),
                   os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "baseline", "_ref")]


def reference_module(name: str):
    """Import ``llmserve.<name>`` from the reference checkout, or skip the test."""
    for root in _REF_CANDIDATES:
        if root and os.path.isdir(os.path.join(root, "llmserve")):
            if root not in sys.path:
                sys.path.append(root)
            break
    else:
        pytest.skip("reference implementation not available")
    try:
        return importlib.import_module(name)
    except Exception as e:  # pragma: no cover - depends on the environment
        pytest.skip(f"reference module {name} not importable: {e}")
