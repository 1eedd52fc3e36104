"""Loader for the in-tree sm_100a extension ``llmserve_b200/_C*.so``.

The extension is built by ``python setup.py build_ext --inplace`` (or ``__graft_entry__.build``).
There is no silent fallback: a CUDA tensor reaching an op without the extension is an error.
"""
import importlib

_C = None


def C():
    global _C
    if _C is None:
        try:
            _C = importlib.import_module("llmserve_b200._C")
        except ImportError as e:
            raise RuntimeError(
                "llmserve_b200._C (sm_100a kernels) is not built; run "
                "`python setup.py build_ext --inplace` in the repository root") from e
    return _C


def available() -> bool:
    try:
        C()
        return True
    except RuntimeError:
        return False
