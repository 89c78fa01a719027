"""Write the reference-side C++ adapters of INTEGRATION.md (B200AttentionProvider, B200LanguageModel)
as one source file, so that they can be compiled against the reference's headers exactly as the
document shows them. Test infrastructure only.

    python oracle/extract_adapter.py INTEGRATION.md oracle/_ref/b200_provider.cpp
"""
from __future__ import annotations

import re
import sys
from pathlib import Path


def adapter_source(document: str) -> str:
    blocks = re.findall(r"```cpp\n(.*?)```", document, re.S)
    if len(blocks) != 2:
        raise ValueError("INTEGRATION.md holds the provider and the language model blocks")
    # the second block continues the first one's namespace
    return blocks[0].replace("}  // namespace attnrank\n", "") + blocks[1] + "\n}  // namespace attnrank\n"


if __name__ == "__main__":
    Path(sys.argv[2]).write_text(adapter_source(Path(sys.argv[1]).read_text()))
