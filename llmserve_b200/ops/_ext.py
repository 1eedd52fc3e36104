"""Loader for the in-tree sm_100a extension ``llmserve_b200/_C*.so``.

The extension is built by ``python setup.py build_ext --inplace`` (or ``__graft_entry__.build``).
There is no silent fallback: a CUDA tensor reaching an op without the extension is an error.
"""
import importlib

_C = None
_PROXY = None

# kernels launched per extension call (calls not listed launch one kernel)
_KERNELS_PER_CALL = {}


class LaunchCounter:
    """Counts the extension's kernel launches (graph replays add their captured count)."""
    launches = 0


class _CountingModule:
    def __init__(self, mod):
        self._mod = mod
        self._cache = {}

    def __getattr__(self, name):
        fn = self._cache.get(name)
        if fn is None:
            target = getattr(self._mod, name)
            n = _KERNELS_PER_CALL.get(name, 1)

            def fn(*args, _t=target, _n=n):
                LaunchCounter.launches += _n
                return _t(*args)
            self._cache[name] = fn
        return fn


def C():
    global _C, _PROXY
    if _PROXY is None:
        try:
            import torch  # noqa: F401  (loads libc10 for the extension)
            _C = importlib.import_module("llmserve_b200._C")
        except ImportError as e:
            raise RuntimeError(
                "llmserve_b200._C (sm_100a kernels) is not built; run "
                "`python setup.py build_ext --inplace` in the repository root") from e
        _PROXY = _CountingModule(_C)
    return _PROXY


def raw_module():
    C()
    return _C


def available() -> bool:
    try:
        C()
        return True
    except RuntimeError:
        return False


_STATUS = {}

ERROR_NAMES = {1: "TMA stage wait timed out", 2: "free-stage wait timed out", 3: "accumulator wait timed out",
               4: "peer flag wait timed out", 5: "out-of-range slot/block index skipped"}


def status(device):
    """Per-device int32 word in which kernels record a bounded-wait timeout or a skipped bad
    index instead of trapping; read it with :func:`check_status`."""
    import torch
    d = torch.device(device)
    if d.type == "cuda" and d.index is None:
        d = torch.device("cuda", torch.cuda.current_device())
    key = str(d)
    t = _STATUS.get(key)
    if t is None:
        # a normal tensor even when first asked for inside inference mode: check_status resets it
        # in place from ordinary code
        with torch.inference_mode(False):
            t = torch.zeros(1, dtype=torch.int32, device=d)
        _STATUS[key] = t
    return t


def check_status(device, reset: bool = True):
    """Raise if a kernel on ``device`` recorded an error since the last check (syncs the device)."""
    t = status(device)
    code = int(t.item())
    if code and reset:
        t.zero_()
    if code:
        raise RuntimeError(f"llmserve_b200 kernel error {code}: {ERROR_NAMES.get(code, 'unknown')}")
