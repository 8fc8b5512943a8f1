"""Python face of the sm_100a GEMM: C = A @ B^T, BF16 in, FP32 accumulate.

Mirrors how the reference drives its GEMM candidates
(gemm_comparison/gemm_comparison.py:2806-2867: build, then call the compiled
kernel with (a, b, c, stream)): a :class:`GemmPlan` is built once per
problem and launched many times. Tensors stay owned by the caller.

Layouts (the reference's, gemm_comparison.py:2663-2684): A is (M, K) or
(L, M, K) row-major BF16, B is (N, K) or (L, N, K) row-major BF16 (K-major),
C is (M, N) or (L, M, N) row-major BF16 or FP32.
"""
from __future__ import annotations

import ctypes

import torch

from . import _native as nat

VARIANTS = {
    "nonpersistent_1cta": nat.BB_VARIANT_NONPERSISTENT_1CTA,
    "persistent_1cta": nat.BB_VARIANT_PERSISTENT_1CTA,
    "persistent_2cta": nat.BB_VARIANT_PERSISTENT_2CTA,
    "tuned": nat.BB_VARIANT_TUNED,
}

_DTYPES = {torch.bfloat16: nat.BB_DTYPE_BF16, torch.float32: nat.BB_DTYPE_F32}


def _dims(a: torch.Tensor, b: torch.Tensor, c: torch.Tensor) -> tuple[int, int, int, int]:
    if a.dim() == 2:
        a, b, c = a.unsqueeze(0), b.unsqueeze(0), c.unsqueeze(0)
    if not (a.dim() == b.dim() == c.dim() == 3):
        raise ValueError("A, B and C must all be 2-D or all be 3-D (batched)")
    l, m, k = a.shape
    lb, n, kb = b.shape
    lc, mc, nc = c.shape
    if (lb, kb) != (l, k) or (lc, mc, nc) != (l, m, n):
        raise ValueError(f"shape mismatch: A{tuple(a.shape)} B{tuple(b.shape)} C{tuple(c.shape)}")
    return m, n, k, l


def _check_tensor(name: str, t: torch.Tensor) -> None:
    if not t.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor")
    if not t.is_contiguous():
        raise ValueError(f"{name} must be contiguous")


class GemmPlan:
    """A compiled launch of the GEMM for fixed tensors (the plan owns nothing
    but its tensor maps and a 4-byte device status word)."""

    def __init__(self, a: torch.Tensor, b: torch.Tensor, c: torch.Tensor, variant: str = "tuned",
                 stream: torch.cuda.Stream | None = None):
        for name, t in (("A", a), ("B", b), ("C", c)):
            _check_tensor(name, t)
        if a.dtype != torch.bfloat16 or b.dtype != torch.bfloat16:
            raise ValueError("A and B must be bfloat16")
        if c.dtype not in _DTYPES:
            raise ValueError("C must be bfloat16 or float32")
        if variant not in VARIANTS:
            raise ValueError(f"unknown variant {variant!r}; expected one of {sorted(VARIANTS)}")
        if not (a.device == b.device == c.device):
            raise ValueError(f"A, B, C on {a.device}, {b.device}, {c.device}: all must be on one device")
        self.m, self.n, self.k, self.l = _dims(a, b, c)
        self.a, self.b, self.c = a, b, c
        self.variant = variant
        self.stream = stream if stream is not None else torch.cuda.current_stream(a.device)
        if self.stream.device != a.device:
            raise ValueError(f"stream on {self.stream.device}, tensors on {a.device}")
        self._lib = nat.bench_lib()
        handle = ctypes.c_void_p()
        info = nat.GemmInfo()
        with torch.cuda.device(a.device):
            nat.check("bb_gemm_plan_create", self._lib.bb_gemm_plan_create(
                self.m, self.n, self.k, self.l, a.data_ptr(), b.data_ptr(), c.data_ptr(), nat.BB_DTYPE_BF16,
                nat.BB_DTYPE_BF16, _DTYPES[c.dtype], VARIANTS[variant], self.stream.cuda_stream,
                ctypes.byref(handle), ctypes.byref(info)))
        self._handle = handle
        self.info = info.as_dict()

    @property
    def flops(self) -> int:
        return 2 * self.m * self.n * self.k * self.l

    def run(self, iterations: int = 1) -> None:
        """`iterations` back-to-back launches on the plan's stream (async)."""
        nat.check("bb_gemm_execute_n", self._lib.bb_gemm_execute_n(self._handle, int(iterations)))

    def synchronize(self) -> None:
        """Waits for the stream; raises on a device-side wait timeout."""
        nat.check("bb_gemm_synchronize", self._lib.bb_gemm_synchronize(self._handle))

    def run_host(self, a_host: torch.Tensor, b_host: torch.Tensor, c_host: torch.Tensor) -> None:
        """End-to-end call with host buffers (H2D A, B; GEMM; D2H C; sync)."""
        for name, t, dev in (("A", a_host, self.a), ("B", b_host, self.b), ("C", c_host, self.c)):
            if t.is_cuda or not t.is_contiguous() or t.numel() != dev.numel() or t.dtype != dev.dtype:
                raise ValueError(f"host {name} must be a contiguous CPU tensor matching the device tensor")
        nat.check("bb_gemm_run_host", self._lib.bb_gemm_run_host(
            self._handle, a_host.data_ptr(), b_host.data_ptr(), c_host.data_ptr()))

    def set_epilogue(self, alpha: float = 1.0, beta: float = 0.0, c_src: torch.Tensor | None = None) -> None:
        """Later launches compute C = alpha * A @ B^T + beta * c_src; c_src has
        C's shape and dtype (it may be C itself)."""
        ptr = None
        if beta != 0.0:
            if c_src is None:
                raise ValueError("beta != 0 needs c_src")
            if c_src.shape != self.c.shape or c_src.dtype != self.c.dtype or not c_src.is_contiguous() or c_src.device != self.c.device:
                raise ValueError("c_src must be a contiguous CUDA tensor with C's shape and dtype")
            self._c_src = c_src
            ptr = c_src.data_ptr()
        nat.check("bb_gemm_plan_set_epilogue", self._lib.bb_gemm_plan_set_epilogue(self._handle, float(alpha),
                                                                                   float(beta), ptr))

    @property
    def launches(self) -> int:
        return int(self._lib.bb_gemm_launches(self._handle))

    def close(self) -> None:
        if getattr(self, "_handle", None):
            self._lib.bb_gemm_destroy(self._handle)
            self._handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()


def gemm(a: torch.Tensor, b: torch.Tensor, out_dtype: torch.dtype = torch.bfloat16, variant: str = "tuned",
         out: torch.Tensor | None = None) -> torch.Tensor:
    """One-shot C = A @ B^T through the native kernel (synchronising)."""
    if out is None:
        shape = (*a.shape[:-1], b.shape[-2])
        out = torch.empty(shape, dtype=out_dtype, device=a.device)
    with GemmPlan(a, b, out, variant=variant) as plan:
        plan.run()
        plan.synchronize()
    return out


class CublasLtPlan:
    """The cuBLASLt comparator on the same tensors (a library call, the
    role of the reference's cublaslt_bridge.cu). ``layout="reference"`` uses
    the reference's row-major descriptor (cublaslt_bridge.cu:75-128),
    ``"column"`` the column-major view."""

    LAYOUTS = {"column": 0, "reference": 1}

    def __init__(self, a: torch.Tensor, b: torch.Tensor, c: torch.Tensor, autotune: bool = False,
                 stream: torch.cuda.Stream | None = None, layout: str = "column"):
        if not (a.dim() == b.dim() == c.dim() == 2):
            raise ValueError("the comparator takes 2-D operands")
        for name, t in (("A", a), ("B", b), ("C", c)):
            _check_tensor(name, t)
        if not (a.device == b.device == c.device):
            raise ValueError(f"A, B, C on {a.device}, {b.device}, {c.device}: all must be on one device")
        if a.dtype != torch.bfloat16 or b.dtype != torch.bfloat16 or c.dtype not in _DTYPES:
            raise ValueError("A and B must be bfloat16, C bfloat16 or float32")
        if layout not in self.LAYOUTS:
            raise ValueError(f"unknown layout {layout!r}; expected one of {sorted(self.LAYOUTS)}")
        m, k = a.shape
        n = b.shape[0]
        if tuple(b.shape) != (n, k) or tuple(c.shape) != (m, n) or b.shape[1] != k:
            raise ValueError(f"shape mismatch: A{tuple(a.shape)} B{tuple(b.shape)} C{tuple(c.shape)}")
        self._lib = nat.cmp_lib()
        self.stream = stream if stream is not None else torch.cuda.current_stream(a.device)
        self._c = c
        handle = ctypes.c_void_p()
        info = nat.CmpInfo()
        rc = self._lib.bb_cmp_plan_create(m, n, k, a.data_ptr(), b.data_ptr(), c.data_ptr(), _DTYPES[c.dtype],
                                          self.LAYOUTS[layout], 1 if autotune else 0, self.stream.cuda_stream,
                                          ctypes.byref(handle), ctypes.byref(info))
        if rc != 0:
            raise nat.NativeCallError("bb_cmp_plan_create", rc, self._lib.bb_cmp_last_error().decode())
        self._handle = handle
        self.info = info.as_dict()
        self.algo_index = int(info.heuristic_index)
        self.algo_count = int(info.heuristic_returned)
        self.workspace_bytes = int(info.workspace_bytes)

    def set_epilogue(self, alpha: float = 1.0, beta: float = 0.0, c_src: torch.Tensor | None = None) -> None:
        """Later executions compute D = alpha * A @ B^T + beta * c_src."""
        if beta != 0.0:
            if c_src is None:
                raise ValueError("beta != 0 needs c_src")
            if (c_src.shape != self._c.shape or c_src.dtype != self._c.dtype or not c_src.is_contiguous()
                    or c_src.device != self._c.device):
                raise ValueError("c_src must be a contiguous CUDA tensor with C's shape and dtype")
        self._c_src = c_src
        rc = self._lib.bb_cmp_plan_set_epilogue(self._handle, float(alpha), float(beta),
                                                c_src.data_ptr() if beta != 0.0 else None)
        if rc != 0:
            raise nat.NativeCallError("bb_cmp_plan_set_epilogue", rc, self._lib.bb_cmp_last_error().decode())

    def run(self, iterations: int = 1) -> None:
        rc = self._lib.bb_cmp_execute_n(self._handle, int(iterations))
        if rc != 0:
            raise nat.NativeCallError("bb_cmp_execute_n", rc, self._lib.bb_cmp_last_error().decode())

    def close(self) -> None:
        if getattr(self, "_handle", None):
            self._lib.bb_cmp_destroy(self._handle)
            self._handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
