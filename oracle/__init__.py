"""CPU oracle for the gb300-microbench hot path. TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline
leg use this package, and only as the checker (or the timed CPU baseline):
nothing in ``gb300_microbench_b200`` imports it, and the product path has no
CPU fallback.

* ``bb_oracle.c`` (built to ``liboracle.so`` by ``oracle/Makefile``): the
  SplitMix64 pattern (memory_paths/ldgsts.cu:220-232), the per-CTA XOR
  checksums of the streaming kernels, the UMMA known answer
  (umma_throughput/umma_1sm.cu:566-575) and a double-accumulated GEMM for
  small shapes, plus the elementwise check of
  gemm_comparison/gemm_comparison.py:2718-2755.
* :func:`gemm_reference_fp32`: the reference's FP32 oracle
  (gemm_comparison.py:2698-2715, einsum in IEEE FP32) run with torch on the
  CPU, also the timed CPU baseline.

Pinning: ``tests/test_oracle.py`` checks the mixer against SplitMix64's
published seed-0 output, the UMMA answer against the reference's own
``reference_d`` (``oracle/_ref/libref_umma.so``, built from the reference
sources by ``make -C oracle ref``) and the golden fixtures of
``tests/golden/``.
"""
from __future__ import annotations

import ctypes
import subprocess
from ctypes import POINTER, c_double, c_int, c_int64, c_uint32, c_uint64, c_void_p
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "liboracle.so"
REF_LIB_PATH = HERE / "_ref" / "libref_umma.so"

_lib = None


def build(reference: str | None = None) -> None:
    """Builds liboracle.so (and the reference harness when `reference` is a
    readable reference tree)."""
    subprocess.run(["make", "-s", "-C", str(HERE)], check=True)
    if reference and Path(reference, "umma_throughput", "umma_1sm.cu").exists():
        subprocess.run(["make", "-s", "-C", str(HERE), "ref", f"REFERENCE={reference}"], check=True)


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            build()
        L = ctypes.CDLL(str(LIB_PATH))
        L.bbo_mix64.restype = c_uint64
        L.bbo_mix64.argtypes = [c_uint64]
        L.bbo_pattern.argtypes = [c_void_p, c_int64, c_int64]
        L.bbo_uniform_u32.argtypes = [c_void_p, c_int64, c_int64, c_uint64]
        L.bbo_copy_checksums.argtypes = [c_void_p, c_int64, c_int64, c_int, c_int64, c_void_p]
        L.bbo_xor_all.restype = c_uint32
        L.bbo_xor_all.argtypes = [c_void_p, c_int64]
        L.bbo_umma_reference_d.restype = c_double
        L.bbo_umma_reference_d.argtypes = [c_int, c_int, c_int]
        L.bbo_umma_expected.argtypes = [c_void_p, c_void_p, c_int, c_int, c_int, c_void_p]
        L.bbo_gemm_ref.argtypes = [c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_int64]
        L.bbo_validate_elementwise.restype = c_int64
        L.bbo_validate_elementwise.argtypes = [c_void_p, c_void_p, c_int64, c_double, c_double, c_double,
                                               POINTER(c_double), POINTER(c_double)]
        _lib = L
    return _lib


def _ptr(a: np.ndarray) -> int:
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data


def mix64(x: int) -> int:
    return int(lib().bbo_mix64(x))


def pattern_words(vec0: int, nvec: int) -> np.ndarray:
    out = np.empty(4 * nvec, dtype=np.uint32)
    lib().bbo_pattern(_ptr(out), vec0, nvec)
    return out


def uniform_u32(n: int, seed: int = 0, word0: int = 0) -> np.ndarray:
    out = np.empty(n, dtype=np.uint32)
    lib().bbo_uniform_u32(_ptr(out), word0, n, seed)
    return out


def copy_checksums(words: np.ndarray, stage_bytes: int, grid: int, passes: int = 1) -> np.ndarray:
    words = np.ascontiguousarray(words, dtype=np.uint32)
    sink = np.empty(grid, dtype=np.uint32)
    lib().bbo_copy_checksums(_ptr(words), words.size * 4, stage_bytes, grid, passes, _ptr(sink))
    return sink


def xor_all(words: np.ndarray) -> int:
    words = np.ascontiguousarray(words, dtype=np.uint32)
    return int(lib().bbo_xor_all(_ptr(words), words.size))


def umma_reference_d(cta_group: int, n: int, depth: int) -> np.ndarray:
    m = 128 * cta_group
    out = np.empty((m, n), dtype=np.float64)
    f = lib().bbo_umma_reference_d
    for r in range(m):
        for c in range(n):
            out[r, c] = f(r, c, depth)
    return out


def umma_expected(a_bf16_bits: np.ndarray, b_bf16_bits: np.ndarray, depth: int) -> np.ndarray:
    """depth * A @ B^T in double from BF16 bit patterns (uint16 arrays)."""
    a = np.ascontiguousarray(a_bf16_bits, dtype=np.uint16)
    b = np.ascontiguousarray(b_bf16_bits, dtype=np.uint16)
    m, n = a.shape[0], b.shape[0]
    out = np.empty((m, n), dtype=np.float64)
    lib().bbo_umma_expected(_ptr(a), _ptr(b), m, n, depth, _ptr(out))
    return out


def gemm_ref_small(a_bf16_bits: np.ndarray, b_bf16_bits: np.ndarray) -> np.ndarray:
    """C = A @ B^T (double accumulation, FP32 result) for small shapes."""
    a = np.ascontiguousarray(a_bf16_bits, dtype=np.uint16)
    b = np.ascontiguousarray(b_bf16_bits, dtype=np.uint16)
    m, k = a.shape
    n = b.shape[0]
    out = np.empty((m, n), dtype=np.float32)
    lib().bbo_gemm_ref(_ptr(a), _ptr(b), _ptr(out), m, n, k)
    return out


def validate_elementwise(c: np.ndarray, ref: np.ndarray, atol: float = 0.1, rtol: float = 1e-5,
                         floor: float = 1.0) -> tuple[int, float, float]:
    """(mismatches or -1 if non-finite, max_abs_error, max_rel_error)."""
    c = np.ascontiguousarray(c, dtype=np.float32)
    ref = np.ascontiguousarray(ref, dtype=np.float32)
    ma, mr = c_double(), c_double()
    bad = lib().bbo_validate_elementwise(_ptr(c), _ptr(ref), c.size, atol, rtol, floor, ctypes.byref(ma),
                                         ctypes.byref(mr))
    return int(bad), float(ma.value), float(mr.value)


def gemm_reference_fp32(a, b):
    """The reference's FP32 oracle on the CPU: einsum("mk,nk->mn") of the
    upcast BF16 operands in IEEE FP32 (torch tensors in, torch tensor out)."""
    import torch

    return torch.matmul(a.to(torch.float32), b.to(torch.float32).t())


def rel_frobenius(c, ref) -> float:
    """||C - ref||_F / ||ref||_F in double."""
    import torch

    c64 = c.to(torch.float64)
    r64 = ref.to(torch.float64)
    return float(torch.linalg.vector_norm(c64 - r64) / torch.linalg.vector_norm(r64))


def ref_umma_lib():
    """The reference's own reference_d, when oracle/_ref was built."""
    if not REF_LIB_PATH.exists():
        return None
    L = ctypes.CDLL(str(REF_LIB_PATH))
    L.ref_umma_reference_d.restype = c_double
    L.ref_umma_reference_d.argtypes = [c_int, c_int, c_int]
    return L
