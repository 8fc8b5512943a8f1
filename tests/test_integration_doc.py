"""The ctypes bindings INTEGRATION.md shows a reference maintainer stay in
step with the library: the self-contained bridge class runs against the
built libb200bench.so (ABI handshake, no GPU needed), and the argtypes lists
of the other snippets match the library's own signature table."""
import ctypes
import re
from pathlib import Path

import pytest

from gb300_microbench_b200 import _native as nat

DOC = Path(__file__).resolve().parents[1] / "INTEGRATION.md"


def _blocks():
    return re.findall(r"```python\n(.*?)```", DOC.read_text(), re.S)


def test_gemm_bridge_snippet_binds_the_library():
    if not nat.BENCH_LIB_PATH.exists():
        pytest.skip("libb200bench.so not built")
    scope: dict = {}
    exec(_blocks()[0], scope)
    bridge = scope["B200GemmBridge"](str(nat.BENCH_LIB_PATH))  # runs the ABI handshake
    assert bridge.lib.bb_abi_version() == 1
    assert scope["VARIANT"]["tuned"] == nat.BB_VARIANT_TUNED
    assert (scope["BF16"], scope["F32"]) == (nat.BB_DTYPE_BF16, nat.BB_DTYPE_F32)
    assert ctypes.sizeof(scope["GemmInfo"]) == ctypes.sizeof(nat.GemmInfo)


@pytest.mark.parametrize("name", ["bb_lowp_plan_create", "bb_copy_run"])
def test_snippet_argtypes_match_the_library(name):
    for block in _blocks():
        m = re.search(rf"lib\.{name}\.argtypes = (\[.*?\])\n", block, re.S)
        if m:
            break
    else:
        pytest.fail(f"no argtypes for {name} in INTEGRATION.md")
    scope = {k: getattr(ctypes, k) for k in dir(ctypes) if k.startswith(("c_", "POINTER"))}
    scope["LowpInfo"] = nat.LowpInfo
    doc_types = eval(m.group(1), scope)
    _, lib_types = nat.BENCH_SIGNATURES[name]
    assert len(doc_types) == len(lib_types)
    for d, l in zip(doc_types, lib_types):
        assert ctypes.sizeof(d) == ctypes.sizeof(l), (name, d, l)
