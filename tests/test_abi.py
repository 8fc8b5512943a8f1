"""CPU-only checks of the C-ABI boundary: the library builds, loads without
a GPU, exports every symbol include/*.h declares, and its struct sizes and
ABI version match the ctypes shim. No compute call is made."""
import ctypes
import re
import subprocess
from pathlib import Path

import pytest

from gb300_microbench_b200 import _native as nat
from gb300_microbench_b200 import build as buildmod

ROOT = Path(__file__).resolve().parents[1]


def _declared(header: Path) -> set[str]:
    text = header.read_text()
    return set(re.findall(r"BB(?:_CMP)?_API\s+[\w\s\*]+?\b(bb_\w+)\s*\(", text))


@pytest.fixture(scope="module")
def libs():
    buildmod.build()
    return nat.bench_lib(), nat.cmp_lib()


def test_every_declared_symbol_is_exported(libs):
    for header, lib_path in ((ROOT / "include" / "b200bench.h", nat.BENCH_LIB_PATH),
                             (ROOT / "include" / "b200cmp.h", nat.CMP_LIB_PATH)):
        declared = _declared(header)
        assert declared, header
        out = subprocess.run(["nm", "-D", "--defined-only", str(lib_path)], capture_output=True, text=True,
                             check=True).stdout
        exported = set(re.findall(r"\sT\s(bb_\w+)", out))
        missing = declared - exported
        assert not missing, f"{lib_path.name} misses {sorted(missing)}"


def test_shim_binds_exactly_the_header(libs):
    assert _declared(ROOT / "include" / "b200bench.h") == set(nat.BENCH_SIGNATURES)
    assert _declared(ROOT / "include" / "b200cmp.h") == set(nat.CMP_SIGNATURES)


def test_abi_handshake(libs):
    bench, cmp = libs
    assert bench.bb_abi_version() == nat.ABI_VERSION
    assert bench.bb_gemm_info_size() == ctypes.sizeof(nat.GemmInfo) == 16 * 8
    assert bench.bb_copy_info_size() == ctypes.sizeof(nat.CopyInfo)
    assert cmp.bb_cmp_abi_version() == 2
    assert cmp.bb_cmp_info_size() == ctypes.sizeof(nat.CmpInfo)
    assert bench.bb_status_name(nat.BB_ERR_TIMEOUT) == b"TIMEOUT"


def test_host_only_geometry_matches_reference_table(libs):
    """bb_copy_plan with an explicit SM count needs no GPU. The nine
    reference specialisations (tma.cu:273-298 table) must come out exact."""
    from gb300_microbench_b200 import streaming

    expected = {(2, 16): (8192, 32), (2, 32): (16384, 64), (2, 64): (32768, 128), (4, 16): (4096, 16),
                (4, 32): (8192, 32), (4, 64): (16384, 64), (8, 16): (2048, 8), (8, 32): (4096, 16),
                (8, 64): (8192, 32)}
    for (stages, bif), (stage_bytes, tile_height) in expected.items():
        for method in ("ldgsts", "tma"):
            info = streaming.plan(method, stages, bif, 148 * 32 * 1024 * 8, row_bytes=256, sm_count=148)
            assert info["stage_bytes"] == stage_bytes
            assert info["tile_rows"] == tile_height
            assert info["bytes_in_flight"] == stages * stage_bytes
            assert info["grid_ctas"] == 148
    # Three stages: rounded down to the copy granularity.
    assert streaming.plan("ldgsts", 3, 16, 1 << 20, sm_count=148)["stage_bytes"] == 4096
    assert streaming.plan("tma", 3, 64, 1 << 20, row_bytes=128, sm_count=148)["tile_rows"] == 170


def test_bad_arguments_fail_cleanly_without_gpu(libs):
    bench, _ = libs
    info = nat.CopyInfo()
    rc = bench.bb_copy_plan(0, 5, 16, 256, 1 << 20, 148, ctypes.byref(info))
    assert rc == nat.BB_ERR_ARGUMENT
    assert b"stages" in bench.bb_last_error()
    plan = ctypes.c_void_p()
    rc = bench.bb_gemm_plan_create(0, 1, 1, 1, None, None, None, 1, 1, 1, 3, None, ctypes.byref(plan), None)
    assert rc == nat.BB_ERR_ARGUMENT
    assert bench.bb_umma_kernel_name(1, 256, 256) == b"umma_1sm_m128n256k16_d256"
    assert bench.bb_umma_kernel_name(2, 64, 4) == b"umma_2sm_m256n64k16_d4"
    assert bench.bb_umma_kernel_name(1, 96, 4) is None


def test_no_cluster_broadcast_loads_in_sources():
    """No TMA or bulk load with a cluster-broadcast qualifier anywhere in the
    kernel sources (the token is assembled here so this file names none)."""
    token = "multi" + "cast"
    for path in list((ROOT / "gb300_microbench_b200" / "csrc").glob("*")) + [ROOT / "bench.py"]:
        if path.is_file():
            assert token not in path.read_text(), path
