"""ctypes shim over ``libb200bench.so`` (``include/b200bench.h``) and
``libb200cmp.so`` (``include/b200cmp.h``).

The shim follows the loading discipline of the reference's cuBLASLt wrapper
(gemm_comparison/gemm_comparison.py:1292-1452): load the library from an
explicit path, check the ABI version and every struct size before the first
real call, declare every argument and return type, and turn a non-zero status
into an exception carrying ``bb_last_error()``.

There is no fallback: when the library is missing, every entry point raises
``NativeLibraryError``. The library is built in-tree by
``python -m gb300_microbench_b200.build``.
"""
from __future__ import annotations

import ctypes
import threading
from ctypes import POINTER, c_char_p, c_float, c_int, c_int64, c_size_t, c_uint64, c_void_p
from pathlib import Path

LIB_DIR = Path(__file__).resolve().parent / "lib"
BENCH_LIB_PATH = LIB_DIR / "libb200bench.so"
CMP_LIB_PATH = LIB_DIR / "libb200cmp.so"

ABI_VERSION = 1

BB_OK = 0
BB_ERR_ARGUMENT = 1
BB_ERR_CUDA = 2
BB_ERR_MISMATCH = 3
BB_ERR_TIMEOUT = 4
BB_ERR_UNSUPPORTED = 5
BB_ERR_INTERNAL = 6

BB_DTYPE_BF16 = 1
BB_DTYPE_F32 = 2

BB_VARIANT_NONPERSISTENT_1CTA = 0
BB_VARIANT_PERSISTENT_1CTA = 1
BB_VARIANT_PERSISTENT_2CTA = 2
BB_VARIANT_TUNED = 3

BB_COPY_LDGSTS = 0
BB_COPY_TMA = 1


class NativeLibraryError(RuntimeError):
    """The native library is missing, mismatched or failed to load."""


class NativeCallError(RuntimeError):
    """A C-ABI call returned a non-zero status."""

    def __init__(self, func: str, status: int, message: str):
        super().__init__(f"{func} failed with status {status} ({STATUS_NAMES.get(status, '?')}): {message}")
        self.func = func
        self.status = status
        self.message = message


STATUS_NAMES = {
    BB_OK: "OK",
    BB_ERR_ARGUMENT: "BAD_ARGUMENT",
    BB_ERR_CUDA: "CUDA_ERROR",
    BB_ERR_MISMATCH: "MISMATCH",
    BB_ERR_TIMEOUT: "TIMEOUT",
    BB_ERR_UNSUPPORTED: "UNSUPPORTED",
    BB_ERR_INTERNAL: "INTERNAL",
}


class GemmInfo(ctypes.Structure):
    _fields_ = [(name, c_int64) for name in (
        "mma_tiler_m", "mma_tiler_n", "cluster_m", "cluster_n", "use_2cta_instrs", "max_active_clusters",
        "stages", "grid_ctas", "num_tiles", "smem_bytes", "tmem_columns", "threads_per_cta", "persistent",
        "raster_group_m", "c_dtype", "variant")]

    def as_dict(self) -> dict:
        return {name: int(getattr(self, name)) for name, _ in self._fields_}


class CopyInfo(ctypes.Structure):
    _fields_ = [(name, c_int64) for name in (
        "method", "stages", "bytes_in_flight_kib", "stage_bytes", "bytes_in_flight", "copies_per_thread",
        "row_bytes", "tile_rows", "threads_per_cta", "grid_ctas", "smem_bytes", "total_tiles",
        "occupancy_ctas_per_sm")] + [("reserved", c_int64 * 3)]

    def as_dict(self) -> dict:
        return {name: int(getattr(self, name)) for name, _ in self._fields_ if name != "reserved"}


class LowpInfo(ctypes.Structure):
    """bb_lowp_info of include/b200bench.h."""
    _fields_ = [(name, c_int64) for name in (
        "kind", "tile_m", "tile_n", "tile_k", "stages", "grid_ctas", "num_tiles", "smem_bytes", "tmem_columns",
        "threads_per_cta", "cta_group")] + [("reserved", c_int64 * 5)]

    def as_dict(self) -> dict:
        return {name: int(getattr(self, name)) for name, _ in self._fields_ if name != "reserved"}


BB_LOWP_NVFP4 = 1
BB_LOWP_FP8_BLOCK128 = 2

# Every symbol include/b200bench.h declares, with (restype, argtypes).
BENCH_SIGNATURES: dict[str, tuple] = {
    "bb_abi_version": (c_int, []),
    "bb_last_error": (c_char_p, []),
    "bb_status_name": (c_char_p, [c_int]),
    "bb_gemm_info_size": (c_size_t, []),
    "bb_gemm_plan_create": (c_int, [c_int64, c_int64, c_int64, c_int64, c_void_p, c_void_p, c_void_p, c_int, c_int,
                                    c_int, c_int, c_void_p, POINTER(c_void_p), POINTER(GemmInfo)]),
    "bb_gemm_execute": (c_int, [c_void_p]),
    "bb_gemm_execute_n": (c_int, [c_void_p, c_int]),
    "bb_gemm_run_host": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p]),
    "bb_gemm_synchronize": (c_int, [c_void_p]),
    "bb_gemm_launches": (c_int64, [c_void_p]),
    "bb_gemm_plan_set_epilogue": (c_int, [c_void_p, c_float, c_float, c_void_p]),
    "bb_gemm_destroy": (c_int, [c_void_p]),
    "bb_gemm_run_noalloc": (c_int, [c_int64, c_int64, c_int64, c_int64, c_void_p, c_void_p, c_void_p, c_int,
                                    c_void_p, c_int]),
    "bb_copy_info_size": (c_size_t, []),
    "bb_copy_plan": (c_int, [c_int, c_int, c_int, c_int, c_int64, c_int, POINTER(CopyInfo)]),
    "bb_copy_run": (c_int, [c_int, c_int, c_int, c_int, c_void_p, c_int64, c_int64, c_int64, c_void_p, c_void_p,
                            c_void_p]),
    "bb_copy_validate": (c_int, [c_int, c_int, c_int, c_int, c_void_p, c_int64, c_void_p, c_void_p, c_void_p,
                                 c_void_p]),
    "bb_fill_pattern": (c_int, [c_void_p, c_int64, c_void_p]),
    "bb_fill_uniform_u32": (c_int, [c_void_p, c_int64, c_uint64, c_void_p]),
    "bb_umma_run": (c_int, [c_int, c_int, c_int, c_int64, c_int, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                            c_void_p, c_void_p]),
    "bb_umma_run_ex": (c_int, [c_int, c_int, c_int, c_int64, c_int, c_int, c_void_p, c_void_p, c_void_p, c_void_p,
                               c_void_p, c_void_p, c_void_p]),
    "bb_umma_kernel_name": (c_char_p, [c_int, c_int, c_int]),
    "bb_test_wait_timeout": (c_int, [c_int64, c_void_p, c_void_p]),
    "bb_kernel_launches": (c_int64, []),
    "bb_lowp_info_size": (c_size_t, []),
    "bb_lowp_scale_bytes": (c_int64, [c_int, c_int64, c_int64]),
    "bb_lowp_plan_create": (c_int, [c_int, c_int64, c_int64, c_int64, c_void_p, c_void_p, c_void_p, c_void_p,
                                    c_float, c_void_p, c_void_p, POINTER(c_void_p), POINTER(LowpInfo)]),
    "bb_lowp_execute_n": (c_int, [c_void_p, c_int]),
    "bb_lowp_synchronize": (c_int, [c_void_p]),
    "bb_lowp_launches": (c_int64, [c_void_p]),
    "bb_lowp_destroy": (c_int, [c_void_p]),
}

class CmpInfo(ctypes.Structure):
    """bb_cmp_info of include/b200cmp.h."""
    _fields_ = [(name, c_int64) for name in (
        "layout", "cublaslt_version", "lda", "ldb", "ldc", "ldd", "transa", "transb", "order_a", "order_b",
        "order_c", "order_d", "type_ab", "type_d", "compute_type", "scale_type", "pointer_mode", "epilogue",
        "search_mode", "workspace_limit_bytes", "workspace_bytes", "heuristic_requested", "heuristic_returned",
        "heuristic_index", "alignment_a_bytes", "alignment_b_bytes", "alignment_c_bytes", "alignment_d_bytes",
        "algo_id", "tile_id", "stages_id", "split_k", "reduction_scheme", "cta_swizzling", "custom_option",
        "inner_shape_id", "cluster_shape_id")] + [("waves_count", ctypes.c_double), ("alpha", ctypes.c_double),
                                                   ("beta", ctypes.c_double)]

    def as_dict(self) -> dict:
        return {name: getattr(self, name) for name, _ in self._fields_}


CMP_SIGNATURES: dict[str, tuple] = {
    "bb_cmp_abi_version": (c_int, []),
    "bb_cmp_info_size": (c_size_t, []),
    "bb_cmp_last_error": (c_char_p, []),
    "bb_cmp_plan_create": (c_int, [c_int64, c_int64, c_int64, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int,
                                   c_void_p, POINTER(c_void_p), POINTER(CmpInfo)]),
    "bb_cmp_lowp_plan_create": (c_int, [c_int, c_int64, c_int64, c_int64, c_void_p, c_void_p, c_void_p, c_void_p,
                                        c_float, c_void_p, c_int, c_void_p, POINTER(c_void_p), POINTER(CmpInfo)]),
    "bb_cmp_plan_set_epilogue": (c_int, [c_void_p, c_float, c_float, c_void_p]),
    "bb_cmp_execute_n": (c_int, [c_void_p, c_int]),
    "bb_cmp_destroy": (c_int, [c_void_p]),
}

_lock = threading.Lock()
_bench = None
_cmp = None


def _bind(lib: ctypes.CDLL, sigs: dict[str, tuple]) -> None:
    for name, (res, args) in sigs.items():
        fn = getattr(lib, name)  # AttributeError if the symbol is missing
        fn.restype = res
        fn.argtypes = args


def bench_lib() -> ctypes.CDLL:
    """Loads libb200bench.so once, checking the ABI handshake."""
    global _bench
    with _lock:
        if _bench is not None:
            return _bench
        if not BENCH_LIB_PATH.exists():
            raise NativeLibraryError(
                f"{BENCH_LIB_PATH} is missing; build it with `python -m gb300_microbench_b200.build`")
        try:
            lib = ctypes.CDLL(str(BENCH_LIB_PATH))
            _bind(lib, BENCH_SIGNATURES)
        except (OSError, AttributeError) as exc:
            raise NativeLibraryError(f"cannot load {BENCH_LIB_PATH}: {exc}") from exc
        if lib.bb_abi_version() != ABI_VERSION:
            raise NativeLibraryError(f"ABI version {lib.bb_abi_version()} != {ABI_VERSION}")
        if lib.bb_gemm_info_size() != ctypes.sizeof(GemmInfo):
            raise NativeLibraryError("bb_gemm_info size mismatch")
        if lib.bb_copy_info_size() != ctypes.sizeof(CopyInfo):
            raise NativeLibraryError("bb_copy_info size mismatch")
        if lib.bb_lowp_info_size() != ctypes.sizeof(LowpInfo):
            raise NativeLibraryError("bb_lowp_info size mismatch")
        _bench = lib
        return lib


def cmp_lib() -> ctypes.CDLL:
    """Loads the cuBLASLt comparator library once."""
    global _cmp
    with _lock:
        if _cmp is not None:
            return _cmp
        if not CMP_LIB_PATH.exists():
            raise NativeLibraryError(f"{CMP_LIB_PATH} is missing; build it first")
        try:
            lib = ctypes.CDLL(str(CMP_LIB_PATH))
            _bind(lib, CMP_SIGNATURES)
        except (OSError, AttributeError) as exc:
            raise NativeLibraryError(f"cannot load {CMP_LIB_PATH}: {exc}") from exc
        if lib.bb_cmp_abi_version() != 2 or lib.bb_cmp_info_size() != ctypes.sizeof(CmpInfo):
            raise NativeLibraryError("comparator ABI version or bb_cmp_info size mismatch")
        _cmp = lib
        return lib


def check(func: str, status: int) -> None:
    if status != BB_OK:
        msg = bench_lib().bb_last_error()
        raise NativeCallError(func, status, msg.decode() if msg else "")


def call(func: str, *args):
    """Calls a status-returning entry point, raising on failure."""
    status = getattr(bench_lib(), func)(*args)
    check(func, status)
    return status


def kernel_launches() -> int:
    return int(bench_lib().bb_kernel_launches())
