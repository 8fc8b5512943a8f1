"""The allocation-free GEMM entry point, bb_gemm_run_noalloc.

Some callers cannot call cudaMalloc (an allocator's own callbacks, a plugin
host that owns the whole device heap); this entry point serves them with the
same tuned kernel, keeping its scratch in a static device array instead of
a plan-owned allocation. This file checks, through the C ABI, that two calls
in a row give the same C as the existing plan-based entry point
(bb_gemm_plan_create + bb_gemm_execute) on the same inputs, including shapes
whose stream-K region uses the static scratch (a sub-wave problem whose every
tile is cut over the clusters among them). It is named to be collected last,
and it passes alone in a fresh process as well as after the others.
"""
import ctypes

import pytest
import torch

import oracle
from gb300_microbench_b200 import _native as nat
from gb300_microbench_b200 import inputs

pytestmark = pytest.mark.gpu

BF16_TOL = 1e-2  # relative Frobenius, the tolerance of the GEMM parity tests


def _plan_result(a, b, c_dtype):
    lib = nat.bench_lib()
    m, k = a.shape
    n = b.shape[0]
    c = torch.full((m, n), float("nan"), dtype=c_dtype, device=a.device)
    plan = ctypes.c_void_p()
    info = nat.GemmInfo()
    stream = torch.cuda.current_stream().cuda_stream
    dt = nat.BB_DTYPE_BF16 if c_dtype == torch.bfloat16 else nat.BB_DTYPE_F32
    nat.check("bb_gemm_plan_create", lib.bb_gemm_plan_create(
        m, n, k, 1, a.data_ptr(), b.data_ptr(), c.data_ptr(), nat.BB_DTYPE_BF16, nat.BB_DTYPE_BF16, dt,
        nat.BB_VARIANT_TUNED, stream, ctypes.byref(plan), ctypes.byref(info)))
    nat.check("bb_gemm_execute", lib.bb_gemm_execute(plan))
    nat.check("bb_gemm_synchronize", lib.bb_gemm_synchronize(plan))
    lib.bb_gemm_destroy(plan)
    return c


def _noalloc_result(a, b, c_dtype):
    lib = nat.bench_lib()
    m, k = a.shape
    n = b.shape[0]
    c = torch.full((m, n), float("nan"), dtype=c_dtype, device=a.device)
    dt = nat.BB_DTYPE_BF16 if c_dtype == torch.bfloat16 else nat.BB_DTYPE_F32
    nat.check("bb_gemm_run_noalloc", lib.bb_gemm_run_noalloc(
        m, n, k, 1, a.data_ptr(), b.data_ptr(), c.data_ptr(), dt, torch.cuda.current_stream().cuda_stream, 1))
    return c


@pytest.mark.parametrize("mnk,c_dtype", [
    ((4096, 4096, 4096), torch.bfloat16),    # stream-K region: uses the scratch
    ((32768, 512, 4096), torch.float32),     # stream-K region, FP32 C
    ((512, 4096, 4096), torch.bfloat16),     # sub-wave: every tile cut over the clusters
    ((1024, 768, 512), torch.bfloat16)])     # whole tiles only
def test_noalloc_matches_plan_entry_point_twice(cuda_device, mnk, c_dtype):
    m, n, k = mnk
    a_cpu, b_cpu = inputs.baseline_mode_operands(m, n, k)
    a, b = a_cpu.to(cuda_device), b_cpu.to(cuda_device)
    want = _plan_result(a, b, c_dtype).float()
    first = None
    for _ in range(2):
        got = _noalloc_result(a, b, c_dtype).float()
        assert torch.isfinite(got).all()
        err = float(torch.linalg.vector_norm(got - want) / torch.linalg.vector_norm(want))
        assert err <= BF16_TOL, err
        assert torch.equal(got, want)  # same kernel, fixed summation order
        if first is not None:
            assert torch.equal(got, first)  # the static scratch's leftovers do not leak in
        first = got
    ref = oracle.gemm_reference_fp32(a_cpu[:256], b_cpu)
    assert oracle.rel_frobenius(got[:256].cpu(), ref) <= BF16_TOL


def test_noalloc_refuses_bad_arguments(cuda_device):
    """Refused before anything is launched, with the reason in bb_last_error."""
    lib = nat.bench_lib()
    stream = torch.cuda.current_stream().cuda_stream
    a = torch.zeros(256, 256, dtype=torch.bfloat16, device=cuda_device)
    b = torch.zeros(264, 256, dtype=torch.bfloat16, device=cuda_device)
    c = torch.zeros(256, 264, dtype=torch.bfloat16, device=cuda_device)
    cases = [
        ((256, 256, 256, 1, None, None, None, nat.BB_DTYPE_BF16), "non-null"),       # null pointers
        ((256, 256, 100, 1, a.data_ptr(), b.data_ptr(), c.data_ptr(), nat.BB_DTYPE_BF16), "K=100 must be a multiple of 8"),  # K % 8
        ((256, 260, 256, 1, a.data_ptr(), b.data_ptr(), c.data_ptr(), nat.BB_DTYPE_BF16), "N=260 breaks"),  # N % 8
        ((256, 262, 256, 1, a.data_ptr(), b.data_ptr(), c.data_ptr(), nat.BB_DTYPE_F32), "N=262 breaks"),   # N % 4
        ((0, 256, 256, 1, a.data_ptr(), b.data_ptr(), c.data_ptr(), nat.BB_DTYPE_BF16), "positive"),
    ]
    for args, needle in cases:
        rc = lib.bb_gemm_run_noalloc(*args, stream, 1)
        assert rc == nat.BB_ERR_ARGUMENT, (args, rc)
        msg = lib.bb_last_error()
        msg = msg.decode() if isinstance(msg, bytes) else str(msg)
        assert needle in msg, msg
