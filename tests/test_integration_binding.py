"""The reference-side binding (gb300_microbench_b200/integration.py, the
code a maintainer of the reference copies) stays in step with the library:
the bridge runs its ABI handshake against the built libb200bench.so (no GPU
needed), its structures have the library's sizes, and every argument list
it declares matches the library's own signature table."""
import ctypes

import pytest

from gb300_microbench_b200 import _native as nat
from gb300_microbench_b200 import integration as integ


def test_gemm_bridge_binds_the_library():
    if not nat.BENCH_LIB_PATH.exists():
        pytest.skip("libb200bench.so not built")
    bridge = integ.B200GemmBridge(str(nat.BENCH_LIB_PATH))  # runs the ABI handshake
    assert bridge.lib.bb_abi_version() == 1
    assert integ.VARIANT["tuned"] == nat.BB_VARIANT_TUNED
    assert (integ.BF16, integ.F32) == (nat.BB_DTYPE_BF16, nat.BB_DTYPE_F32)
    assert ctypes.sizeof(integ.GemmInfo) == ctypes.sizeof(nat.GemmInfo)
    assert ctypes.sizeof(integ.LowpInfo) == ctypes.sizeof(nat.LowpInfo) == bridge.lib.bb_lowp_info_size()


@pytest.mark.parametrize("name", ["bb_gemm_plan_create", "bb_gemm_run_noalloc", "bb_lowp_plan_create",
                                  "bb_copy_run", "bb_umma_run_ex"])
def test_binding_argtypes_match_the_library(name):
    if not nat.BENCH_LIB_PATH.exists():
        pytest.skip("libb200bench.so not built")
    lib = ctypes.CDLL(str(nat.BENCH_LIB_PATH))
    lib.bb_abi_version.restype = ctypes.c_int
    lib.bb_gemm_info_size.restype = ctypes.c_size_t
    if name.startswith("bb_gemm"):
        lib = integ.B200GemmBridge(str(nat.BENCH_LIB_PATH)).lib
    else:
        integ.bind_other_entry_points(lib)
    doc_types = getattr(lib, name).argtypes
    _, lib_types = nat.BENCH_SIGNATURES[name]
    assert len(doc_types) == len(lib_types)
    for d, l in zip(doc_types, lib_types):
        assert ctypes.sizeof(d) == ctypes.sizeof(l), (name, d, l)
