"""The ctypes binding a maintainer of the reference adds to reach this
library: the drop-in for the CuTe DSL candidates of gemm_comparison.py
(built and launched at gemm_comparison.py:2806-2867, wrapped like the
reference's own cuBLASLt bridge, ``CublasLtBridge`` at
gemm_comparison.py:1292-1452), plus the argument lists of the block-scaled,
streaming and UMMA entry points.

Self-contained on purpose (only ctypes): it is the code a reference-side
caller copies, and the tests import it to check it against the library.
"""
from __future__ import annotations

import ctypes
from ctypes import POINTER, c_char_p, c_float, c_int, c_int64, c_size_t, c_void_p

VARIANT = {"nonpersistent_1cta": 0, "persistent_1cta": 1, "persistent_2cta": 2, "tuned": 3}
BF16, F32 = 1, 2


class GemmInfo(ctypes.Structure):  # bb_gemm_info: 16 x int64
    _fields_ = [(n, c_int64) for n in (
        "mma_tiler_m", "mma_tiler_n", "cluster_m", "cluster_n", "use_2cta_instrs",
        "max_active_clusters", "stages", "grid_ctas", "num_tiles", "smem_bytes",
        "tmem_columns", "threads_per_cta", "persistent", "raster_group_m", "c_dtype", "variant")]


class B200GemmBridge:
    """Plan create / execute in place of ``cute.compile`` / ``compiled(a, b,
    c, stream)``; the reference's timing loop, NaN reset, oracle and
    ``validate_result`` stay as they are."""

    def __init__(self, path: str):
        lib = ctypes.CDLL(path)
        lib.bb_abi_version.restype = c_int
        lib.bb_gemm_info_size.restype = c_size_t
        lib.bb_last_error.restype = c_char_p
        lib.bb_gemm_plan_create.argtypes = [c_int64] * 4 + [c_void_p] * 3 + [c_int] * 4 + [
            c_void_p, POINTER(c_void_p), POINTER(GemmInfo)]
        lib.bb_gemm_execute.argtypes = [c_void_p]
        lib.bb_gemm_synchronize.argtypes = [c_void_p]
        lib.bb_gemm_destroy.argtypes = [c_void_p]
        lib.bb_gemm_run_noalloc.argtypes = [c_int64] * 4 + [c_void_p] * 3 + [c_int, c_void_p, c_int]
        # Handshake, as gemm_comparison.py:1355-1367 does for p35_*:
        if lib.bb_abi_version() != 1 or lib.bb_gemm_info_size() != ctypes.sizeof(GemmInfo):
            raise RuntimeError("libb200bench ABI mismatch")
        self.lib = lib

    def plan(self, a, b, c, variant: str, stream):
        """a: (M, K, L) K-major BF16 with strides (K, 1, MK); b: (N, K, L);
        c: (M, N, L) FP32 or BF16. Returns (handle, info); info fills the
        CSV's mma_tiler_m/n, cluster_m/n, use_2cta_instrs, max_active_clusters."""
        m, k, l = a.shape
        n = b.shape[0]
        h, info = c_void_p(), GemmInfo()
        c_dtype = F32 if c.element_size() == 4 else BF16
        rc = self.lib.bb_gemm_plan_create(m, n, k, l, a.data_ptr(), b.data_ptr(), c.data_ptr(), BF16, BF16, c_dtype,
                                          VARIANT[variant], stream.cuda_stream, ctypes.byref(h), ctypes.byref(info))
        if rc:
            raise RuntimeError(self.lib.bb_last_error().decode())
        return h, info

    def launch(self, h) -> None:
        """In place of ``compiled(a, b, c, stream)``."""
        if self.lib.bb_gemm_execute(h):
            raise RuntimeError(self.lib.bb_last_error().decode())

    def run_noalloc(self, a, b, c, stream, wait: bool = True) -> None:
        """The tuned GEMM without a plan and without device allocation."""
        m, k, l = a.shape
        n = b.shape[0]
        c_dtype = F32 if c.element_size() == 4 else BF16
        if self.lib.bb_gemm_run_noalloc(m, n, k, l, a.data_ptr(), b.data_ptr(), c.data_ptr(), c_dtype,
                                        stream.cuda_stream, 1 if wait else 0):
            raise RuntimeError(self.lib.bb_last_error().decode())

    def destroy(self, h) -> None:
        self.lib.bb_gemm_destroy(h)


class LowpInfo(ctypes.Structure):  # bb_lowp_info: 16 x int64
    _fields_ = [(n, c_int64) for n in (
        "kind", "tile_m", "tile_n", "tile_k", "stages", "grid_ctas", "num_tiles", "smem_bytes", "tmem_columns",
        "threads_per_cta", "cta_group")] + [("reserved", c_int64 * 5)]


def bind_other_entry_points(lib) -> None:
    """Argument lists of the block-scaled GEMM (kind 1 = NVFP4: packed E2M1
    rows x K/2 bytes with 512-byte UE4M3 scale atoms and alpha = the product
    of the tensor scales; kind 2 = FP8: E4M3 bytes with FP32 [ceil(rows/128)]
    [K/128] scales, alpha = 1), of the streaming pass (method 0 = LDGSTS,
    1 = TMA; row_bytes 256 for the reference grid, 128 for the baseline
    grid; one uint32 checksum per CTA into sink) and of the UMMA probe
    (handshake = 1: the reference's per-iteration CTA-pair handshake)."""
    lib.bb_lowp_plan_create.argtypes = [c_int, c_int64, c_int64, c_int64, c_void_p, c_void_p, c_void_p,
                                        c_void_p, c_float, c_void_p, c_void_p, POINTER(c_void_p),
                                        POINTER(LowpInfo)]
    lib.bb_copy_run.argtypes = [c_int, c_int, c_int, c_int, c_void_p, c_int64, c_int64, c_int64,
                                c_void_p, c_void_p, c_void_p]
    lib.bb_umma_run_ex.argtypes = [c_int, c_int, c_int, c_int64, c_int, c_int, c_void_p, c_void_p, c_void_p,
                                   c_void_p, c_void_p, c_void_p, c_void_p]
