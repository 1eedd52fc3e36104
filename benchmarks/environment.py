"""Run provenance stored with every benchmark result: the code revision, the software stack, the
GPU, and the revision of the checkpoint that produced the numbers.

The key names of :func:`build_environment_metadata` form the ``metadata`` block of the result
schema, which the reference harness writes too (``benchmarks/environment.py`` there), so result
files of both engines line up; the probing below is this module's own.
"""
import json
import os
import platform
import re
import subprocess
import tempfile
from datetime import datetime, timezone
from pathlib import Path

REPOSITORY_ROOT = Path(__file__).resolve().parents[1]
_COMMIT_RE = re.compile(r"^[0-9a-f]{40}$")


def _git(*args: str) -> str | None:
    """stdout of a git command run at the repository root, or None when git is missing or fails."""
    try:
        proc = subprocess.run(("git", "-C", str(REPOSITORY_ROOT)) + args, capture_output=True, text=True,
                              timeout=30)
    except (OSError, subprocess.TimeoutExpired):
        return None
    return proc.stdout.strip() if proc.returncode == 0 else None


def _gpu_facts() -> dict:
    import torch
    if not torch.cuda.is_available():
        return {"cuda_available": False, "gpu_name": None, "gpu_memory_bytes": None, "gpu_count": 0}
    props = torch.cuda.get_device_properties(0)
    return {"cuda_available": True, "gpu_name": props.name, "gpu_memory_bytes": props.total_memory,
            "gpu_count": torch.cuda.device_count()}


def build_environment_metadata() -> dict:
    """The ``metadata`` block: UTC time, commit and whether the tree had local changes (untracked
    files included), Python / torch / CUDA versions, and the first GPU."""
    import torch
    changes = _git("status", "--porcelain")
    meta = {
        "generated_at_utc": datetime.now(timezone.utc).isoformat(),
        "git_commit": _git("rev-parse", "HEAD"),
        "git_dirty": None if changes is None else changes != "",
        "python_version": platform.python_version(),
        "torch_version": torch.__version__,
        "cuda_runtime": torch.version.cuda,
    }
    meta.update(_gpu_facts())
    return meta


def discover_model_revision(model_path: str | None) -> str | None:
    """The 40-hex commit of a local checkpoint directory, when the Hugging Face tooling recorded
    one: a snapshot directory of the hub cache (``.../snapshots/<commit>``), or a ``--local-dir``
    download whose metadata file starts with the commit.  None otherwise."""
    if not model_path:
        return None
    path = Path(model_path)
    if path.parent.name == "snapshots" and _COMMIT_RE.match(path.name):
        return path.name
    meta = path / ".cache" / "huggingface" / "download" / "config.json.metadata"
    try:
        with open(meta) as f:
            first = f.readline().strip()
    except OSError:
        return None
    return first if _COMMIT_RE.match(first) else None


def atomic_write_json(path, value: dict) -> None:
    """Write ``value`` as indented JSON so a reader never sees a partial file: a temporary file in
    the same directory, flushed to disk, then renamed over ``path``."""
    path = Path(path)
    path.parent.mkdir(parents=True, exist_ok=True)
    fd, tmp = tempfile.mkstemp(dir=path.parent, prefix=path.name + ".", suffix=".tmp")
    try:
        with os.fdopen(fd, "w") as f:
            f.write(json.dumps(value, indent=2) + "\n")
            f.flush()
            os.fsync(f.fileno())
        os.replace(tmp, path)
    except BaseException:
        try:
            os.unlink(tmp)
        except OSError:
            pass
        raise
