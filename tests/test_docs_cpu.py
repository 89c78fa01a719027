"""The documents stay true to the code: every `bench.py` flag quoted in the profiles and the
design / baseline / readme files is one bench.py accepts, and every file the design's file map
names exists. No GPU."""
from __future__ import annotations

import re
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]
DOCS = [ROOT / name for name in ("DESIGN.md", "BASELINE.md", "README.md", "INTEGRATION.md")] + \
    sorted((ROOT / "profiles").glob("*.md"))


def test_quoted_bench_flags_exist():
    help_text = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--help"], capture_output=True, text=True,
                               timeout=300, cwd=ROOT).stdout
    accepted = set(re.findall(r"--[a-z][a-z-]*", help_text))
    assert "--steps" in accepted
    for doc in DOCS:
        for command in re.findall(r"bench\.py[^`\n]*", doc.read_text()):
            for flag in re.findall(r"--[a-z][a-z-]*", command):
                assert flag in accepted, f"{doc.name}: `{command.strip()}` uses {flag}, which bench.py does not take"


def test_file_map_paths_exist():
    text = (ROOT / "DESIGN.md").read_text()
    section = text[text.index("## 10. File map"):]
    paths = set(re.findall(r"`([A-Za-z_./-]+\.(?:cu|h|cpp|py|md|json)|[a-z_]+/)`", section))
    assert len(paths) > 15
    missing = [p for p in sorted(paths)
               if not any((base / p).exists() for base in (ROOT, ROOT / "attention-rank_b200"))]
    assert not missing, missing
