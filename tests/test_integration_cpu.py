"""The reference-side code of INTEGRATION.md is real code: the C++ adapters (IAttentionProvider /
ILanguageModel over the C ABI) compile against the reference's headers and link against the
reference's compiled sources plus libattnrank_b200.so, and the Python ctypes stub loads the
library with a prompt struct laid out like `ar_prompt`. No GPU: nothing is run on a device."""
from __future__ import annotations

import ctypes
import re
import shutil
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
DOC = (ROOT / "INTEGRATION.md").read_text()
from oracle import REFERENCE_ROOT as REFERENCE  # noqa: E402
REFERENCE_LIBRARY = ROOT / "oracle" / "_ref" / "libattnrank_ref.so"
LIBRARY_DIR = ROOT / "attention-rank_b200" / "attnrank"

LINK_MAIN = """
int main(int argc, char**) {
  if (argc < 0) {  // never taken: the link is what is checked
    attnrank::LlamaConfig config;
    attnrank::WeightRegistry weights;
    attnrank::LlamaRuntimeOptions options;
    attnrank::B200AttentionProvider provider(config, weights, options);
    attnrank::B200LanguageModel model(nullptr, config, options, nullptr);
    return provider.measure_attention_by_layer({}, {}).layer_begin + model.config().vocab_size;
  }
  return 0;
}
"""


def _adapter_source() -> str:
    from oracle.extract_adapter import adapter_source
    return adapter_source(DOC)


def test_cpp_adapters_compile_and_link_against_the_reference(tmp_path):
    if not (REFERENCE / "include" / "attnrank" / "model.hpp").is_file():
        pytest.skip("the reference checkout is not present")
    if not REFERENCE_LIBRARY.is_file() or shutil.which("g++") is None:
        pytest.skip("oracle/_ref is not built")
    source = tmp_path / "b200_provider.cpp"
    source.write_text(_adapter_source() + LINK_MAIN)
    command = ["g++", "-std=c++17", "-Wall", "-Werror", f"-I{REFERENCE / 'include'}", f"-I{ROOT / 'include'}",
               "-I/usr/local/cuda/include", str(source), "-o", str(tmp_path / "provider"),
               f"-L{REFERENCE_LIBRARY.parent}", "-lattnrank_ref", f"-L{LIBRARY_DIR}", "-lattnrank_b200",
               "-L/usr/local/cuda/lib64", "-lcudart"]
    result = subprocess.run(command, capture_output=True, text=True)
    assert result.returncode == 0, result.stderr[-4000:]


def test_python_stub_loads_the_library():
    from attnrank import _native
    block = re.findall(r"```python\n(.*?)```", DOC, re.S)[0]
    block = block.replace("/path/to/attention-rank_b200/attnrank/libattnrank_b200.so", str(_native.LIBRARY_PATH))
    scope: dict = {}
    exec(compile(block, "INTEGRATION.md", "exec"), scope)  # noqa: S102 - the document's own stub
    lib, prompt_type, check = scope["lib"], scope["ArPrompt"], scope["check"]
    assert ctypes.sizeof(prompt_type) == ctypes.sizeof(_native.PromptStruct)
    assert [name for name, _ in prompt_type._fields_] == [name for name, _ in _native.PromptStruct._fields_]
    order = (ctypes.c_int * 3)()
    check(lib.ar_resolve_position_order((ctypes.c_int * 2)(2, 0), 2, 3, order))
    assert list(order) == [2, 0, 1]
    with pytest.raises(RuntimeError):
        check(lib.ar_resolve_position_order(None, 0, -1, order))
