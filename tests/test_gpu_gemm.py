"""GEMM parity on the GPU through the C ABI, against the CPU oracle.

Reference mode (integer operands, FP32 C) must be exact; the reference's
elementwise check (|d| <= 0.1 + 1e-5 |ref|, gemm_comparison.py:2718-2755) is
applied as well. Baseline mode (N(0,1) operands, BF16 C) must be within a
relative Frobenius error of 1e-2 of the FP32 oracle.
"""
import pytest
import torch

import oracle
from gb300_microbench_b200 import inputs
from gb300_microbench_b200.gemm import VARIANTS, CublasLtPlan, GemmPlan

pytestmark = pytest.mark.gpu

BF16_TOL = 1e-2  # relative Frobenius bound of baseline mode (N(0,1) operands, BF16 C)


def _run(a, b, out_dtype, variant, dev):
    l = a.shape[0] if a.dim() == 3 else None
    ad, bd = a.to(dev).contiguous(), b.to(dev).contiguous()
    shape = (*a.shape[:-1], b.shape[-2])
    c = torch.full(shape, float("nan"), dtype=out_dtype, device=dev)
    plan = GemmPlan(ad, bd, c, variant=variant)
    plan.run()
    plan.synchronize()
    plan.close()
    return c.cpu()


@pytest.mark.parametrize("variant", list(VARIANTS))
@pytest.mark.parametrize("mnk", [(256, 256, 128), (512, 768, 320), (300, 264, 200), (128, 128, 64),
                                 (1024, 512, 1024)])
def test_reference_mode_exact(cuda_device, variant, mnk):
    m, n, k = mnk
    a, b = inputs.reference_mode_operands(m, n, k)
    a, b = a[0], b[0]
    c = _run(a, b, torch.float32, variant, cuda_device)
    ref = torch.from_numpy(oracle.gemm_ref_small(a.view(torch.int16).numpy().view("uint16"),
                                                 b.view(torch.int16).numpy().view("uint16")))
    assert torch.isfinite(c).all(), "unwritten (NaN) output elements"
    assert torch.equal(c, ref)
    bad, max_abs, _ = oracle.validate_elementwise(c.numpy(), ref.numpy())
    assert bad == 0 and max_abs == 0.0


@pytest.mark.parametrize("variant", list(VARIANTS))
@pytest.mark.parametrize("mnk", [(256, 256, 256), (384, 640, 448), (1000, 1000, 1000)])
def test_baseline_mode_bf16(cuda_device, variant, mnk):
    m, n, k = mnk
    a, b = inputs.baseline_mode_operands(m, n, k)
    c = _run(a, b, torch.bfloat16, variant, cuda_device)
    ref = oracle.gemm_reference_fp32(a, b)
    assert torch.isfinite(c.float()).all()
    err = oracle.rel_frobenius(c.float(), ref)
    assert err <= BF16_TOL, err
    # BF16 rounding of the output alone gives ~2e-3; a layout bug gives ~1.
    assert err < 5e-3


@pytest.mark.parametrize("variant", ["persistent_2cta", "tuned", "persistent_1cta"])
def test_batched_l2(cuda_device, variant):
    a, b = inputs.reference_mode_operands(384, 512, 256, l=2)
    c = _run(a, b, torch.float32, variant, cuda_device)
    for i in range(2):
        ref = oracle.gemm_reference_fp32(a[i], b[i])
        assert torch.equal(c[i], ref)


@pytest.mark.parametrize("variant", list(VARIANTS))
@pytest.mark.parametrize("mnkl", [(300, 264, 200, 3), (129, 8, 72, 2)])
def test_batched_ragged(cuda_device, variant, mnkl):
    """Batches whose every extent is ragged against the tiles: each batch
    entry must be exact and no entry may write into another's rows."""
    m, n, k, l = mnkl
    a, b = inputs.reference_mode_operands(m, n, k, l=l)
    c = _run(a, b, torch.float32, variant, cuda_device)
    assert torch.isfinite(c).all(), "unwritten (NaN) output elements"
    for i in range(l):
        assert torch.equal(c[i], oracle.gemm_reference_fp32(a[i], b[i]))


@pytest.mark.parametrize("variant", list(VARIANTS))
@pytest.mark.parametrize("mnk", [(1, 8, 8), (1, 16, 64), (7, 8, 72), (129, 264, 8), (2, 520, 136)])
def test_minimal_extents_exact(cuda_device, variant, mnk):
    """The smallest legal extents (M = 1, N = 8, K = 8) and shapes below one
    tile in every dimension: the tensor maps' zero fill and the clipped
    stores must give the exact product and write every element of C."""
    m, n, k = mnk
    a, b = inputs.reference_mode_operands(m, n, k)
    a, b = a[0], b[0]
    c = _run(a, b, torch.float32, variant, cuda_device)
    assert torch.isfinite(c).all(), "unwritten (NaN) output elements"
    assert torch.equal(c, oracle.gemm_reference_fp32(a, b))
    cb = _run(a, b, torch.bfloat16, variant, cuda_device)
    assert torch.equal(cb, oracle.gemm_reference_fp32(a, b).to(torch.bfloat16))


@pytest.mark.parametrize("variant", ["tuned", "persistent_1cta"])
@pytest.mark.parametrize("mnk", [(256, 256, 16384), (128, 64, 32768)])
def test_long_k_exact(cuda_device, variant, mnk):
    """Long reductions (256-512 k-blocks; the tuned variant cuts the single
    tile's k-blocks over the clusters and fixes up the partials): integer
    products stay exact in FP32, so any dropped or doubled k-block shows."""
    m, n, k = mnk
    a, b = inputs.reference_mode_operands(m, n, k)
    a, b = a[0], b[0]
    c = _run(a, b, torch.float32, variant, cuda_device)
    assert torch.equal(c, oracle.gemm_reference_fp32(a, b))


@pytest.mark.parametrize("variant", ["tuned", "persistent_2cta"])
def test_full_size_4096_baseline(cuda_device, variant):
    """Config 0 at full size: 4096^3, N(0,1) seed 0, BF16 C."""
    a, b = inputs.baseline_mode_operands(4096, 4096, 4096)
    c = _run(a, b, torch.bfloat16, variant, cuda_device)
    ref = oracle.gemm_reference_fp32(a, b)
    err = oracle.rel_frobenius(c.float(), ref)
    assert err <= BF16_TOL, err


def test_repeat_launches_idempotent(cuda_device):
    """Back-to-back launches of one plan rewrite the same C (persistent
    scheduler, TMEM double buffer and ring phases all restart per launch)."""
    a, b = inputs.baseline_mode_operands(2048, 1536, 1024)
    ad, bd = a.to(cuda_device), b.to(cuda_device)
    c = torch.empty(2048, 1536, dtype=torch.bfloat16, device=cuda_device)
    plan = GemmPlan(ad, bd, c, variant="tuned")
    plan.run()
    plan.synchronize()
    first = c.clone()
    plan.run(5)
    plan.synchronize()
    assert torch.equal(first, c)
    assert plan.launches == 6


def test_skinny_shapes_reference_mode(cuda_device):
    """The three skinny shapes of the sweep, scaled down in K (exact check)."""
    for m, n, k in [(16384, 512, 256), (512, 16384, 256), (4096, 512, 512)]:
        a, b = inputs.reference_mode_operands(m, n, k)
        c = _run(a[0], b[0], torch.float32, "tuned", cuda_device)
        ref = oracle.gemm_reference_fp32(a[0], b[0])
        assert torch.equal(c, ref), (m, n, k)


def test_run_host_matches_device_path(cuda_device):
    a, b = inputs.baseline_mode_operands(512, 512, 512)
    ad = torch.empty_like(a, device=cuda_device)
    bd = torch.empty_like(b, device=cuda_device)
    c = torch.empty(512, 512, dtype=torch.bfloat16, device=cuda_device)
    plan = GemmPlan(ad, bd, c)
    c_host = torch.empty(512, 512, dtype=torch.bfloat16).pin_memory()
    plan.run_host(a.pin_memory(), b.pin_memory(), c_host)
    ref = _run(a, b, torch.bfloat16, "tuned", cuda_device)
    assert torch.equal(c_host, ref)


@pytest.mark.parametrize("mnk,dtype", [((4096, 1024, 2048), torch.bfloat16), ((1280, 520, 264), torch.float32)])
def test_run_host_pipelined(cuda_device, mnk, dtype):
    """Host-buffer path with the row-chunk pipeline (B first, A chunks, each
    chunk's GEMM and C copy overlapping later transfers): integer operands,
    so every tiling gives the exact product."""
    m, n, k = mnk
    a, b = inputs.reference_mode_operands(m, n, k)
    a, b = a[0].contiguous(), b[0].contiguous()
    ad = torch.empty_like(a, device=cuda_device)
    bd = torch.empty_like(b, device=cuda_device)
    c = torch.empty(m, n, dtype=dtype, device=cuda_device)
    plan = GemmPlan(ad, bd, c)
    c_host = torch.full((m, n), float("nan"), dtype=dtype).pin_memory()
    for _ in range(2):  # the second call reuses the pipeline
        plan.run_host(a.pin_memory(), b.pin_memory(), c_host)
    ref = oracle.gemm_reference_fp32(a, b)
    if dtype == torch.float32:
        assert torch.equal(c_host, ref)
    else:
        assert oracle.rel_frobenius(c_host.float(), ref) < 4e-3
    plan.set_epilogue(2.0, 0.0)
    plan.run_host(a.pin_memory(), b.pin_memory(), c_host)
    if dtype == torch.float32:
        assert torch.equal(c_host, 2.0 * ref)
    plan.close()


def test_run_host_batched_serial_path(cuda_device):
    """Batched problems (L > 1) take the serial host path."""
    a, b = inputs.reference_mode_operands(512, 264, 128, l=2)
    ad = torch.empty_like(a, device=cuda_device)
    bd = torch.empty_like(b, device=cuda_device)
    c = torch.empty(2, 512, 264, dtype=torch.float32, device=cuda_device)
    plan = GemmPlan(ad, bd, c)
    c_host = torch.full((2, 512, 264), float("nan"), dtype=torch.float32).pin_memory()
    plan.run_host(a.contiguous().pin_memory(), b.contiguous().pin_memory(), c_host)
    for i in range(2):
        assert torch.equal(c_host[i], oracle.gemm_reference_fp32(a[i], b[i]))
    plan.close()


def test_cublaslt_comparator_agrees(cuda_device):
    a, b = inputs.baseline_mode_operands(1024, 1024, 1024)
    ad, bd = a.to(cuda_device), b.to(cuda_device)
    c = torch.empty(1024, 1024, dtype=torch.float32, device=cuda_device)
    cmp = CublasLtPlan(ad, bd, c)
    cmp.run()
    torch.cuda.synchronize()
    ref = oracle.gemm_reference_fp32(a, b)
    assert oracle.rel_frobenius(c.cpu(), ref) < 1e-5


def test_bad_arguments_rejected(cuda_device):
    from gb300_microbench_b200 import _native as nat

    a = torch.zeros(128, 100, dtype=torch.bfloat16, device=cuda_device)  # K not a multiple of 8
    b = torch.zeros(128, 100, dtype=torch.bfloat16, device=cuda_device)
    c = torch.zeros(128, 128, dtype=torch.bfloat16, device=cuda_device)
    with pytest.raises(nat.NativeCallError) as ei:
        GemmPlan(a, b, c)
    assert ei.value.status == nat.BB_ERR_ARGUMENT


def test_negative_iteration_count_rejected(cuda_device):
    from gb300_microbench_b200 import _native as nat

    a = torch.zeros(256, 128, dtype=torch.bfloat16, device=cuda_device)
    b = torch.zeros(256, 128, dtype=torch.bfloat16, device=cuda_device)
    c = torch.zeros(256, 256, dtype=torch.bfloat16, device=cuda_device)
    plan = GemmPlan(a, b, c)
    try:
        before = plan.launches
        plan.run(0)
        with pytest.raises(nat.NativeCallError) as ei:
            plan.run(-1)
        assert ei.value.status == nat.BB_ERR_ARGUMENT
        assert plan.launches == before
    finally:
        plan.close()


@pytest.mark.parametrize("snap", [None, "0"])
@pytest.mark.parametrize("mnk", [(4096, 4096, 1024), (16384, 512, 1024), (512, 16384, 1024), (2304, 2048, 4096),
                                 (640, 768, 2048), (32768, 512, 4096), (256, 2560, 3072), (512, 4096, 4096),
                                 (1024, 4096, 4096), (2048, 4096, 4096), (1536, 4096, 1000)])
def test_stream_k_exact(cuda_device, mnk, snap, monkeypatch):
    """Shapes whose last wave is partial run a stream-K region (the tail's
    (tile, k-block) iterations cut evenly over all clusters; partial pieces
    fixed up by whichever finishes last) in the tuned variant;
    BB_GEMM_STREAM_K=1 forces it even where the cost model declines, and
    BB_GEMM_SK_SNAP=0 keeps range ends off the tile edges, so pieces of one
    or two k-blocks occur. Integer operands make every split of K exact."""
    monkeypatch.setenv("BB_GEMM_STREAM_K", "1")
    if snap is not None:
        monkeypatch.setenv("BB_GEMM_SK_SNAP", snap)
    m, n, k = mnk
    a, b = inputs.reference_mode_operands(m, n, k)
    c = _run(a[0], b[0], torch.float32, "tuned", cuda_device)
    ref = oracle.gemm_reference_fp32(a[0], b[0])
    assert torch.equal(c, ref)


@pytest.mark.parametrize("mnk", [(4096, 4096, 1024), (512, 4096, 4096), (1280, 1040, 520), (300, 600, 200),
                                 (2304, 2056, 1024), (256, 264, 64)])
def test_narrow_tail_exact(cuda_device, mnk, monkeypatch):
    """The narrow tail: the partial last wave's 256-wide tiles computed as
    two half-width (256 x 128) items on twice as many clusters, in the same
    kernel as the whole tiles (BB_GEMM_NARROW=1 forces it where legal).
    Ragged N leaves a second half partly or wholly outside C. Integer
    operands: exact in FP32 and in BF16."""
    monkeypatch.setenv("BB_GEMM_NARROW", "1")
    monkeypatch.setenv("BB_GEMM_TILE_N", "256")
    m, n, k = mnk
    a, b = inputs.reference_mode_operands(m, n, k)
    ref = oracle.gemm_reference_fp32(a[0], b[0])
    for out in (torch.float32, torch.bfloat16):
        c = _run(a[0], b[0], out, "tuned", cuda_device)
        assert torch.isfinite(c.float()).all(), "unwritten (NaN) output elements"
        assert torch.equal(c, ref.to(out))


def test_narrow_tail_epilogue_and_repeat(cuda_device, monkeypatch):
    """alpha / beta on the half-width items, and repeated launches."""
    monkeypatch.setenv("BB_GEMM_NARROW", "1")
    monkeypatch.setenv("BB_GEMM_TILE_N", "256")
    m, n, k = 4096, 4096, 512
    a, b = inputs.reference_mode_operands(m, n, k)
    a, b = a[0], b[0]
    csrc = torch.randint(-4, 5, (m, n), generator=torch.Generator().manual_seed(9)).float()
    c = torch.full((m, n), float("nan"), dtype=torch.float32, device=cuda_device)
    plan = GemmPlan(a.to(cuda_device), b.to(cuda_device), c, variant="tuned")
    src = csrc.to(cuda_device)
    plan.set_epilogue(0.5, -1.5, src)
    plan.run(3)
    plan.synchronize()
    plan.close()
    assert torch.equal(c.cpu(), 0.5 * oracle.gemm_reference_fp32(a, b) - 1.5 * csrc)


def test_stream_k_deterministic_bf16(cuda_device):
    """The fix-up sums partials in k order whoever finishes last: repeated
    launches are bit-identical even though arrival order varies."""
    a, b = inputs.baseline_mode_operands(4096, 4096, 2048)
    ad, bd = a.to(cuda_device), b.to(cuda_device)
    c = torch.empty(4096, 4096, dtype=torch.bfloat16, device=cuda_device)
    plan = GemmPlan(ad, bd, c, variant="tuned")
    plan.run()
    plan.synchronize()
    first = c.clone()
    for _ in range(3):
        plan.run(3)
        plan.synchronize()
        assert torch.equal(first, c)
    ref = oracle.gemm_reference_fp32(a, b)
    assert oracle.rel_frobenius(c.cpu().float(), ref) <= BF16_TOL


def test_stream_k_concurrent_plans(cuda_device):
    """Two stream-K plans launched at the same time on two streams share the
    SMs, so some clusters of each launch only start when the other launch's
    clusters exit. No piece waits for another (the last to finish does the
    fix-up), so both complete without a timeout and stay exact."""
    shapes = [(512, 4096, 4096), (2048, 4096, 2048)]
    runs = []
    for m, n, k in shapes:
        a, b = inputs.reference_mode_operands(m, n, k)
        a, b = a[0], b[0]
        c = torch.full((m, n), float("nan"), dtype=torch.float32, device=cuda_device)
        s = torch.cuda.Stream(device=cuda_device)
        with torch.cuda.stream(s):
            plan = GemmPlan(a.to(cuda_device), b.to(cuda_device), c, variant="tuned")
        runs.append((plan, c, oracle.gemm_reference_fp32(a, b), s))
    torch.cuda.synchronize()
    for _ in range(5):
        for plan, _, _, _ in runs:
            plan.run(2)
    for plan, c, ref, _ in runs:
        plan.synchronize()
        assert torch.equal(c.cpu(), ref)
        plan.close()


@pytest.mark.parametrize("tile_n", ["256", "512"])
@pytest.mark.parametrize("mnk,force_split", [((512, 1024, 512), False), ((300, 600, 200), False),
                                             ((1024, 1536, 4096), True), ((4096, 4096, 3072), True),
                                             ((8192, 512, 1024), False)])
def test_tuned_tile_shapes_exact(cuda_device, monkeypatch, tile_n, mnk, force_split):
    """Both CTA-pair tile shapes of the tuned variant (256 x 256 with a
    double-buffered accumulator, 256 x 512 with two N = 256 MMAs per K step),
    including ragged N (half of the second MMA outside C) and the stream-K
    region, are exact on integer operands."""
    monkeypatch.setenv("BB_GEMM_TILE_N", tile_n)
    if force_split:
        monkeypatch.setenv("BB_GEMM_STREAM_K", "1")
    m, n, k = mnk
    a, b = inputs.reference_mode_operands(m, n, k)
    for out in (torch.float32, torch.bfloat16):
        c = _run(a[0], b[0], out, "tuned", cuda_device)
        ref = oracle.gemm_reference_fp32(a[0], b[0])
        if out == torch.float32:
            assert torch.equal(c, ref)
        else:
            assert torch.equal(c, ref.to(torch.bfloat16))


EPI_CASES = [(v, mnk, None) for v in ("tuned", "persistent_1cta", "persistent_2cta")
             for mnk in ((512, 768, 320), (300, 264, 200), (1024, 1024, 4096))]
EPI_CASES += [("tuned", (4096, 4096, 4096), None),   # stream-K region
              ("tuned", (1024, 1024, 4096), "512")]  # 512-wide tile, eight-warp epilogue


@pytest.mark.parametrize("out_dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("variant,mnk,tile_n", EPI_CASES)
@pytest.mark.parametrize("alpha,beta,inplace", [(0.5, 0.0, False), (1.5, -2.0, False), (1.0, 1.0, True)])
def test_alpha_beta_epilogue(cuda_device, out_dtype, variant, mnk, tile_n, alpha, beta, inplace, monkeypatch):
    """C = alpha A B^T + beta Csrc on every store path (whole tiles, the
    512-wide tile, the stream-K fix-up), Csrc separate or C itself. Integer
    operands, FP32 output: exact; BF16 output: within BF16 rounding."""
    if tile_n:
        monkeypatch.setenv("BB_GEMM_TILE_N", tile_n)
    m, n, k = mnk
    a, b = inputs.reference_mode_operands(m, n, k)
    a, b = a[0], b[0]
    g = torch.Generator().manual_seed(7)
    csrc = torch.randint(-4, 5, (m, n), generator=g).to(out_dtype)
    ad, bd = a.to(cuda_device), b.to(cuda_device)
    c = (csrc.clone() if inplace else torch.full((m, n), float("nan"), dtype=out_dtype)).to(cuda_device)
    src = c if inplace else csrc.to(cuda_device)
    plan = GemmPlan(ad, bd, c, variant=variant)
    if tile_n:
        assert plan.info["mma_tiler_n"] == int(tile_n)
    plan.set_epilogue(alpha, beta, src if beta != 0.0 else None)
    plan.run()
    plan.synchronize()
    plan.close()
    prod = oracle.gemm_reference_fp32(a, b)
    ref = alpha * prod + beta * csrc.float()
    got = c.float().cpu()
    if out_dtype == torch.float32:
        assert torch.equal(got, ref), (got - ref).abs().max()
    else:
        err = oracle.rel_frobenius(got, ref)
        assert err <= 4e-3, err


def test_alpha_beta_matches_cublaslt(cuda_device):
    """The comparator computes the same epilogue on the same operands."""
    m, n, k = 1024, 768, 512
    a, b = inputs.reference_mode_operands(m, n, k)
    ad, bd = a[0].to(cuda_device), b[0].to(cuda_device)
    csrc = torch.randint(-3, 4, (m, n), generator=torch.Generator().manual_seed(3)).float().to(cuda_device)
    ours = torch.empty(m, n, dtype=torch.float32, device=cuda_device)
    theirs = torch.empty_like(ours)
    plan = GemmPlan(ad, bd, ours, variant="tuned")
    plan.set_epilogue(0.25, 3.0, csrc)
    plan.run()
    plan.synchronize()
    cmp = CublasLtPlan(ad, bd, theirs, layout="reference")
    cmp.set_epilogue(0.25, 3.0, csrc)
    cmp.run()
    torch.cuda.synchronize()
    assert torch.equal(ours, theirs)
    plan.close()
    cmp.close()
