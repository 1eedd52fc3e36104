"""Provenance of a benchmark run (``benchmarks/environment.py`` of the reference)."""
import json
import os
import platform
import subprocess
from datetime import datetime, timezone
from pathlib import Path

REPOSITORY_ROOT = Path(__file__).resolve().parents[1]


def git_output(*args: str):
    try:
        r = subprocess.run(["git", *args], cwd=REPOSITORY_ROOT, check=True, capture_output=True, text=True)
    except (OSError, subprocess.CalledProcessError):
        return None
    return r.stdout.strip()


def build_environment_metadata() -> dict:
    import torch
    cuda = torch.cuda.is_available()
    commit = git_output("rev-parse", "HEAD")
    status = git_output("status", "--porcelain")
    return {
        "generated_at_utc": datetime.now(timezone.utc).isoformat(),
        "git_commit": commit,
        "git_dirty": bool(status) if status is not None else None,
        "python_version": platform.python_version(),
        "torch_version": torch.__version__,
        "cuda_runtime": torch.version.cuda,
        "cuda_available": cuda,
        "gpu_name": torch.cuda.get_device_name(0) if cuda else None,
        "gpu_memory_bytes": torch.cuda.get_device_properties(0).total_memory if cuda else None,
        "gpu_count": torch.cuda.device_count() if cuda else 0,
    }


def discover_model_revision(model_path: str | None):
    """40-hex revision recorded by the HF hub download cache next to a local checkout, if any."""
    if model_path is None:
        return None
    meta = Path(model_path) / ".cache" / "huggingface" / "download" / "config.json.metadata"
    try:
        rev = meta.read_text().splitlines()[0].strip()
    except (OSError, IndexError):
        return None
    if len(rev) != 40:
        return None
    try:
        int(rev, 16)
    except ValueError:
        return None
    return rev


def atomic_write_json(path, value: dict):
    path = Path(path)
    path.parent.mkdir(parents=True, exist_ok=True)
    tmp = path.with_suffix(path.suffix + ".tmp")
    tmp.write_text(json.dumps(value, indent=2) + "\n")
    os.replace(tmp, path)
