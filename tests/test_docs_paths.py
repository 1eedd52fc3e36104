"""Every repository path that the design notes, the README and the benchmark README name exists
(brace lists such as ``benchmarks/{suite,run_suite}.py`` are expanded)."""
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PREFIXES = ("llmserve_b200/", "benchmarks/", "tests/", "profiles/", "baseline/ref_arm", "bench.py", "setup.py",
            "check_speculative_correctness.py", "example.py", "__graft_entry__.py", ".github/")


def _expand(path):
    m = re.search(r"\{([^{}]*)\}", path)
    if not m:
        return [path]
    return [p for alt in m.group(1).split(",") for p in _expand(path[:m.start()] + alt + path[m.end():])]


def _named_paths(text):
    for token in re.findall(r"`([^`\s]+)`", text):
        token = token.rstrip(".,;:")
        if token.startswith(PREFIXES) and "*" not in token and "<" not in token:
            yield from _expand(token)


@pytest.mark.parametrize("doc", ["DESIGN.md", "README.md", "benchmarks/README.md", "profiles/README.md"])
def test_named_paths_exist(doc):
    text = open(os.path.join(ROOT, doc)).read()
    missing = []
    for p in _named_paths(text):
        base = p.split("::")[0].split(":")[0]
        if base.endswith("/"):
            base = base[:-1]
        if not os.path.exists(os.path.join(ROOT, base)):
            missing.append(p)
    assert not missing, missing


def test_package_relative_and_profile_names_exist():
    """``ops/csrc/...``-style names in the design notes are relative to the package; the profile
    index names files of ``profiles/``."""
    design = open(os.path.join(ROOT, "DESIGN.md")).read()
    rel = [p for t in re.findall(r"`((?:ops|engine|models|layers|parallel|quantization|speculative|utils)/[^`\s]+)`",
                                  design) for p in _expand(t.rstrip(".,;:"))]
    assert rel and all(os.path.exists(os.path.join(ROOT, "llmserve_b200", p)) for p in rel), \
        [p for p in rel if not os.path.exists(os.path.join(ROOT, "llmserve_b200", p))]
    index = open(os.path.join(ROOT, "profiles", "README.md")).read()
    names = re.findall(r"`([\w.-]+\.md)`", index)
    assert names and all(os.path.exists(os.path.join(ROOT, "profiles", n)) for n in names)
    listed = set(names)
    assert {f for f in os.listdir(os.path.join(ROOT, "profiles")) if f != "README.md"} <= listed
