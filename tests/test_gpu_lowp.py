"""Block-scaled GEMM parity on the GPU (FP8 128 x 128-block, NVFP4) through the C ABI.

Two kinds of cases per format:
* exact: operands encoded directly with power-of-two block scales and small
  values, so every product and partial sum is exact in FP32; D must equal the
  oracle's FP32 result rounded to BF16 bit for bit. These pin the operand,
  scale-atom and TMEM scale layouts.
* quantised N(0, 1): relative Frobenius error of D against the FP32 matmul of
  the dequantised inputs <= 2e-2 (the configuration's check); observed errors
  are BF16 output rounding, about 2e-3.
"""
import numpy as np
import pytest
import torch

import oracle
from oracle import lowp as olp
from gb300_microbench_b200 import lowp

pytestmark = pytest.mark.gpu

LOWP_TOL = 2e-2  # relative Frobenius bound of the block-scaled GEMMs


def _e4m3_pow2(exps: torch.Tensor) -> torch.Tensor:
    """E4M3 bits of 2^e for -6 <= e <= 8."""
    return ((exps + 7) << 3).to(torch.uint8)


def _nvfp4_exact_operand(rows, k, gen):
    codes = torch.randint(0, 16, (rows, k), generator=gen, dtype=torch.uint8)
    packed = (codes[:, 0::2] | (codes[:, 1::2] << 4)).contiguous()
    exps = torch.randint(-1, 2, (rows, k // 16), generator=gen)
    return lowp.Nvfp4Operand.from_parts(packed, _e4m3_pow2(exps), 1.0)


def _fp8_exact_operand(rows, k, gen):
    # E4M3 integers 0..15 with random sign: exactly representable.
    ints = torch.randint(0, 16, (rows, k), generator=gen).float()
    sign = torch.where(torch.rand(rows, k, generator=gen) < 0.5, -1.0, 1.0)
    q = (ints * sign).to(torch.float8_e4m3fn).view(torch.uint8)
    exps = torch.randint(-1, 2, (-(-rows // 128), k // 128), generator=gen)
    return lowp.Fp8BlockOperand.from_parts(q, torch.exp2(exps.float()))


def _oracle_d(kind, a, b):
    if kind == "nvfp4":
        ad = olp.nvfp4_dequant(a.data.cpu().numpy(), a.atoms.cpu().numpy(), a.tensor_scale, a.rows, a.k)
        bd = olp.nvfp4_dequant(b.data.cpu().numpy(), b.atoms.cpu().numpy(), b.tensor_scale, b.rows, b.k)
    else:
        ad = olp.fp8_block_dequant(a.data.cpu().numpy(), a.scales.cpu().numpy())
        bd = olp.fp8_block_dequant(b.data.cpu().numpy(), b.scales.cpu().numpy())
    return olp.gemm_dequant_fp32(ad, bd)


def _run(kind, a, b, dev):
    ad, bd = a.to(dev), b.to(dev)
    d = torch.full((a.rows, b.rows), float("nan"), dtype=torch.bfloat16, device=dev)
    plan = lowp.LowpGemmPlan(kind, ad, bd, d)
    plan.run()
    plan.synchronize()
    assert plan.launches == 1
    plan.close()
    return d.cpu()


EXACT_SHAPES = [(128, 256, 256), (256, 512, 512), (384, 256, 1024), (200, 264, 512), (1024, 768, 768),
                (520, 136, 256), (1, 8, 256), (130, 24, 256)]  # the last two: minimal and sub-tile extents


@pytest.mark.parametrize("cta_group", ["1", "2"])
@pytest.mark.parametrize("kind", ["nvfp4", "fp8_block128"])
@pytest.mark.parametrize("mnk", EXACT_SHAPES)
def test_exact(cuda_device, kind, mnk, cta_group, monkeypatch):
    """Both tile shapes (BB_LOWP_CTA_GROUP forces 128 x 256 single-CTA or
    256 x 256 CTA-pair tiles)."""
    monkeypatch.setenv("BB_LOWP_CTA_GROUP", cta_group)
    m, n, k = mnk
    if kind == "nvfp4" and k % 256:
        pytest.skip("NVFP4 needs K % 256 == 0")
    gen = torch.Generator().manual_seed(m * 7 + n * 3 + k)
    make = _nvfp4_exact_operand if kind == "nvfp4" else _fp8_exact_operand
    a, b = make(m, k, gen), make(n, k, gen)
    ref = _oracle_d(kind, a, b)
    d = _run(kind, a, b, cuda_device)
    ref_bf16 = torch.from_numpy(ref).to(torch.bfloat16)
    mismatch = (d.view(torch.int16) != ref_bf16.view(torch.int16)).sum().item()
    assert mismatch == 0, f"{mismatch} of {m * n} elements differ from the exact result"


@pytest.mark.parametrize("kind", ["nvfp4", "fp8_block128"])
@pytest.mark.parametrize("mnk", [(256, 256, 512), (512, 1024, 2048), (1000, 776, 1536)])
def test_quantised_normal(cuda_device, kind, mnk):
    m, n, k = mnk
    x, y = lowp.config4_inputs(m, n, k, seed=0, device="cpu")
    op = lowp.Nvfp4Operand if kind == "nvfp4" else lowp.Fp8BlockOperand
    a, b = op(x), op(y)
    ref = _oracle_d(kind, a, b)
    d = _run(kind, a, b, cuda_device).float().numpy()
    err = oracle.rel_frobenius(torch.from_numpy(d), torch.from_numpy(ref))
    assert err <= LOWP_TOL, err
    assert err <= 5e-3, f"error {err} well above BF16 output rounding"


def test_argument_errors(cuda_device):
    gen = torch.Generator().manual_seed(0)
    a = _nvfp4_exact_operand(128, 256, gen).to(cuda_device)
    b = _nvfp4_exact_operand(256, 256, gen).to(cuda_device)
    with pytest.raises(ValueError):
        lowp.LowpGemmPlan("nvfp4", a, b, torch.empty(128, 255, dtype=torch.bfloat16, device=cuda_device))
    from gb300_microbench_b200 import _native as nat
    with pytest.raises(nat.NativeCallError):
        # K = 128 is not a multiple of the NVFP4 stage (256)
        a2 = _nvfp4_exact_operand(128, 128, gen).to(cuda_device)
        b2 = _nvfp4_exact_operand(256, 128, gen).to(cuda_device)
        lowp.LowpGemmPlan("nvfp4", a2, b2, torch.empty(128, 256, dtype=torch.bfloat16, device=cuda_device))
    # FP8 block scales smaller than the (R/128, K/128) grid the kernel reads
    q = torch.zeros(256, 256, dtype=torch.uint8, device=cuda_device)
    short = lowp.Fp8BlockOperand.from_parts(q, torch.ones(1, 1, device=cuda_device))
    full = lowp.Fp8BlockOperand.from_parts(q, torch.ones(2, 2, device=cuda_device))
    dd = torch.empty(256, 256, dtype=torch.bfloat16, device=cuda_device)
    for x, y in ((short, full), (full, short)):
        with pytest.raises(ValueError, match="scales hold"):
            lowp.LowpGemmPlan("fp8_block128", x, y, dd)
    plan = lowp.LowpGemmPlan("nvfp4", a, b, torch.empty(128, 256, dtype=torch.bfloat16, device=cuda_device))
    try:
        with pytest.raises(nat.NativeCallError) as ei:
            plan.run(-1)
        assert ei.value.status == nat.BB_ERR_ARGUMENT
        assert plan.launches == 0
    finally:
        plan.close()


def test_config4_size_checksums(cuda_device):
    """Full 8192^3 size: D of the quantised N(0, 1) inputs against the FP32
    product of the inputs as the oracle (oracle/lowp.py) decodes them, bit
    by bit from the stored codes and scales, on a sampled set of rows that
    spans every 128-row block (the full FP32 oracle at this size is minutes
    of CPU); B is decoded whole, in row chunks."""
    m = n = k = 8192
    x, y = lowp.config4_inputs(m, n, k, seed=0, device=cuda_device)
    rows = torch.arange(0, m, 61)
    for kind, op in (("nvfp4", lowp.Nvfp4Operand), ("fp8_block128", lowp.Fp8BlockOperand)):
        a, b = op(x), op(y)
        d = torch.empty(m, n, dtype=torch.bfloat16, device=cuda_device)
        plan = lowp.LowpGemmPlan(kind, a, b, d)
        plan.run()
        plan.synchronize()
        plan.close()
        got = d[rows.to(cuda_device)].float().cpu().numpy()
        del d
        if kind == "nvfp4":
            a_atoms, b_atoms = a.atoms.cpu().numpy(), b.atoms.cpu().numpy()
            a_rows = olp.nvfp4_dequant(a.data.cpu().numpy(), a_atoms, a.tensor_scale, m, k)[rows.numpy()]
            b_data = b.data.cpu().numpy()
            b_scales = olp.e4m3_decode(olp.unpack_scale_atoms(b_atoms, n, k)).astype(np.float32)
            b_deq = np.empty((n, k), dtype=np.float32)
            for r0 in range(0, n, 1024):
                vals = olp.e2m1_decode(olp.unpack_fp4(b_data[r0:r0 + 1024])).astype(np.float32)
                b_deq[r0:r0 + 1024] = vals * np.repeat(b_scales[r0:r0 + 1024], 16, axis=1) * np.float32(b.tensor_scale)
        else:
            a_scales, b_scales = a.scales.cpu().numpy(), b.scales.cpu().numpy()
            r = rows.numpy()
            a_rows = olp.e4m3_decode(a.data.cpu().numpy()[r]) * np.repeat(a_scales[r // 128], 128, axis=1)
            b_data = b.data.cpu().numpy()
            b_deq = np.empty((n, k), dtype=np.float32)
            for r0 in range(0, n, 1024):
                b_deq[r0:r0 + 1024] = olp.fp8_block_dequant(b_data[r0:r0 + 1024], b_scales[r0 // 128:(r0 + 1024) // 128])
        ref = olp.gemm_dequant_fp32(a_rows, b_deq).astype(np.float64)
        err = float(np.linalg.norm(got.astype(np.float64) - ref) / np.linalg.norm(ref))
        assert err <= LOWP_TOL, (kind, err)
        assert err < 5e-3, (kind, err)  # BF16 output rounding is about 2e-3
        del a, b, b_deq
