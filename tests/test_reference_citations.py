"""Every ``file:line`` citation of the reference in this repository's code
and tests (docstrings and comments) names a file that exists in the
reference checkout and a line range inside it. Skipped when the reference
checkout is absent."""
import os
import re
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF = os.environ.get("IWHISPER_REFERENCE", os.path.join(os.path.dirname(ROOT), "reference"))
CITE = re.compile(r"([A-Za-z_][A-Za-z0-9_./-]*\.(?:py|cpp|h|hpp|csv|report|toml)):(\d+)(?:-(\d+))?")
SOURCES = (".py", ".cu", ".cuh", ".h", ".c", ".cpp")

pytestmark = pytest.mark.skipif(not os.path.isdir(os.path.join(REF, "i_whisper")),
                                reason="reference checkout not available")


def _reference_files():
    by_name = {}
    for root, dirs, files in os.walk(REF):
        dirs[:] = [d for d in dirs if d != ".git"]
        for f in files:
            by_name.setdefault(f, []).append(os.path.join(root, f))
    return by_name


def test_citations_point_inside_reference_files():
    by_name = _reference_files()
    tracked = subprocess.check_output(["git", "ls-files"], cwd=ROOT, text=True).split()
    lines = {}
    bad, checked = [], 0
    for rel in tracked:
        if not rel.endswith(SOURCES):
            continue
        text = open(os.path.join(ROOT, rel), errors="replace").read()
        for m in CITE.finditer(text):
            name, a = m.group(1), int(m.group(2))
            b = int(m.group(3) or a)
            cands = by_name.get(os.path.basename(name))
            if not cands:
                continue  # a file of this repository, not of the reference
            path = next((c for c in cands if c.endswith(name)), cands[0])
            if path not in lines:
                lines[path] = sum(1 for _ in open(path, errors="replace"))
            checked += 1
            if not (1 <= a <= b <= lines[path]):
                bad.append(f"{rel}: {m.group(0)} ({lines[path]} lines)")
    assert checked > 100
    assert not bad, bad
