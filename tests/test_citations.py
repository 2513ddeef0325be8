"""Every reference citation `file:line` or `file:a-b` in this repository's code and documents points inside the cited
reference file. The reference tree is taken from VLLM_TURING_REFERENCE, else the directory `reference` beside the
repository; the test is skipped where neither exists (e.g. on the GPU box). Citations name a reference file by its
path within the reference project (vllm_turing/w8a8.py, csrc/host_ar.cu, tests/test_hostar.py, ...) or by a base name
that occurs in the reference tree; other `name.ext:n` strings (this repository's own files) are not checked."""
import os
import re

import pytest

HERE = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF = os.environ.get("VLLM_TURING_REFERENCE") or os.path.join(os.path.dirname(HERE), "reference")
CITE = re.compile(r"([A-Za-z0-9_./-]+\.(?:py|cu|cuh|h|c|toml|md))[:](\d+)(?:-(\d+))?")
SCAN_DIRS = ("vllm_turing_b200", "include", "oracle", "tests")
SCAN_FILES = ("bench.py", "__graft_entry__.py", "DESIGN.md", "INTEGRATION.md", "README.md", "BASELINE.md")
OWN_ONLY = {"bench.py", "__graft_entry__.py", "DESIGN.md", "INTEGRATION.md", "README.md", "SURVEY.md",
            "BASELINE.md", "VERDICT.md", "ADVICE.md"}


def _sources():
    for d in SCAN_DIRS:
        for root, _, files in os.walk(os.path.join(HERE, d)):
            if "_ref" in root or "__pycache__" in root or "golden" in root:
                continue
            for f in files:
                if f.endswith((".py", ".cu", ".cuh", ".h", ".c", ".md")):
                    yield os.path.join(root, f)
    for f in SCAN_FILES:
        p = os.path.join(HERE, f)
        if os.path.exists(p):
            yield p


def _ref_index():
    idx = {}
    for root, dirs, files in os.walk(REF):
        dirs[:] = [d for d in dirs if not d.startswith(".")]
        for f in files:
            idx.setdefault(f, []).append(os.path.join(root, f))
    return idx


def _candidates(path, idx):
    path = path.lstrip("./")
    if "/" in path:
        out = [os.path.join(REF, path)]
        tail = path.split("/")
        # a path given from inside the project's package or a sub-directory of it
        for k in range(1, len(tail)):
            out += [p for p in idx.get(tail[-1], []) if p.endswith("/" + "/".join(tail[k:]))]
        return [p for p in out if os.path.isfile(p)]
    return idx.get(path, [])


def _lines(p, cache={}):   # noqa: B006
    if p not in cache:
        with open(p, errors="replace") as f:
            cache[p] = sum(1 for _ in f)
    return cache[p]


@pytest.mark.skipif(not os.path.isdir(REF), reason="the reference tree is not present here")
def test_reference_citations_are_in_range():
    idx = _ref_index()
    bad, checked = [], 0
    for src in _sources():
        with open(src, errors="replace") as f:
            text = f.read()
        for m in CITE.finditer(text):
            path, a, b = m.group(1), int(m.group(2)), int(m.group(3) or m.group(2))
            if os.path.basename(path) in OWN_ONLY:
                continue
            cands = _candidates(path, idx)
            if not cands:
                continue
            checked += 1
            if not any(a >= 1 and a <= b <= _lines(p) for p in cands):
                where = os.path.relpath(src, HERE)
                bad.append(f"{where}: {m.group(0)} (file has {max(_lines(p) for p in cands)} lines)")
    assert checked > 50, f"only {checked} citations found: the scan is broken"
    assert not bad, "citations outside the cited file:\n" + "\n".join(bad)
