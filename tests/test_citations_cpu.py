"""Citations of the reference (`file:line` or `file:first-last`) in this repository's code and
documents point inside the cited file. Runs where the reference checkout is present (the build
host); elsewhere it is skipped. A citation is checked when its file name is unique in the
reference tree (or its path suffix picks one file); names of this repository's own files are not
in the reference and are left alone. The planning inputs (SURVEY.md and the like) are not ours
and are not checked."""
from __future__ import annotations

import collections
import os
import re
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
REFERENCE = Path(os.environ.get("ATTNRANK_REFERENCE", "/root/reference"))
INPUTS = {"SURVEY.md", "VERDICT.md", "ADVICE.md"}
SUFFIXES = (".py", ".cu", ".cuh", ".h", ".cpp", ".md")
CITATION = re.compile(r"((?:[\w./-]+/)?([\w-]+\.(?:cu|cpp|hpp|h|py|md|tex))):(\d+)(?:-(\d+))?")


def _ours():
    for path in ROOT.rglob("*"):
        parts = set(path.relative_to(ROOT).parts)
        if (path.is_file() and path.suffix in SUFFIXES and path.name not in INPUTS
                and not parts & {"_work", "gpurun_out", ".git", "baseline", "_ref"}):
            yield path


def test_reference_citations_point_inside_the_cited_file():
    if not (REFERENCE / "attnrank" / "src" / "model.cu").is_file():
        pytest.skip("the reference checkout is not present")
    by_name = collections.defaultdict(list)
    for path in REFERENCE.rglob("*"):
        if path.is_file() and path.suffix in (".cu", ".cpp", ".hpp", ".h", ".py", ".md", ".tex"):
            by_name[path.name].append(path)
    lengths: dict[Path, int] = {}
    checked, wrong = 0, []
    for source in _ours():
        for match in CITATION.finditer(source.read_text(errors="ignore")):
            cited, name, first, last = match.group(1), match.group(2), int(match.group(3)), match.group(4)
            candidates = by_name.get(name, [])
            if "/" in cited:
                candidates = [c for c in candidates if str(c).endswith(cited)] or candidates
            if len(candidates) != 1:
                continue
            target = candidates[0]
            if target not in lengths:
                lengths[target] = len(target.read_text(errors="ignore").splitlines())
            last_line = int(last) if last else first
            checked += 1
            if not (1 <= first <= last_line <= lengths[target]):
                wrong.append(f"{source.relative_to(ROOT)}: {match.group(0)} ({target.name} has {lengths[target]} lines)")
    assert checked > 300
    assert not wrong, "\n".join(wrong)
