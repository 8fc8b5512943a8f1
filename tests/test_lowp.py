"""CPU tests of the block-scaled GEMM formats: the numpy oracle pinned to
published format values and to torch's own E4M3 conversion, and the product's
quantisers / scale-atom packing checked against the oracle."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from gb300_microbench_b200 import lowp
from oracle import lowp as olp


def test_e4m3_decode_known_values():
    # OCP FP8 E4M3FN: 0x38 = 1.0, 0x7E = 448 (max), 0x08 = 2^-6 (min normal),
    # 0x01 = 2^-9 (min subnormal), 0x7F = NaN, sign in bit 7.
    v = olp.e4m3_decode(np.array([0x38, 0x7E, 0x08, 0x01, 0x00, 0xB8, 0x40, 0x7F], dtype=np.uint8))
    assert v[0] == 1.0 and v[1] == 448.0 and v[2] == 2.0 ** -6 and v[3] == 2.0 ** -9
    assert v[4] == 0.0 and v[5] == -1.0 and v[6] == 2.0
    assert np.isnan(v[7])


def test_e4m3_decode_matches_torch_all_codes():
    codes = np.arange(256, dtype=np.uint8)
    ours = olp.e4m3_decode(codes)
    theirs = torch.from_numpy(codes).view(torch.float8_e4m3fn).float().double().numpy()
    np.testing.assert_array_equal(np.isnan(ours), np.isnan(theirs))
    ok = ~np.isnan(ours)
    np.testing.assert_array_equal(ours[ok], theirs[ok])


def test_e2m1_table():
    codes = np.arange(16, dtype=np.uint8)
    v = olp.e2m1_decode(codes)
    np.testing.assert_array_equal(v[:8], [0, 0.5, 1, 1.5, 2, 3, 4, 6])
    np.testing.assert_array_equal(v[8:], -np.array([0, 0.5, 1, 1.5, 2, 3, 4, 6]))
    np.testing.assert_array_equal(lowp.e2m1_decode(torch.arange(16, dtype=torch.uint8)).double().numpy(), v)


def test_e2m1_rounding_ties_to_even():
    y = torch.tensor([0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0, 7.0, 0.3, 2.6, -0.75, -5.0, -100.0])
    codes = lowp._e2m1_codes(y).tolist()
    assert codes == [0, 2, 2, 4, 4, 6, 6, 7, 1, 5, 10, 14, 15]


def test_scale_atom_layout_round_trip():
    torch.manual_seed(3)
    scales = torch.randint(0, 256, (300, 24), dtype=torch.uint8)  # 300 rows, K = 384
    atoms = lowp.pack_scale_atoms(scales)
    assert atoms.shape == (3, 6, 512)
    # the defining byte rule, for a few entries
    for r, j in [(0, 0), (31, 3), (32, 1), (127, 2), (128, 0), (299, 23)]:
        rb, rr = divmod(r, 128)
        kg, jj = divmod(j, 4)
        assert atoms[rb, kg, (rr % 32) * 16 + (rr // 32) * 4 + jj] == scales[r, j]
    back = olp.unpack_scale_atoms(atoms.numpy(), 300, 384)
    np.testing.assert_array_equal(back, scales.numpy())
    np.testing.assert_array_equal(olp.unpack_scale_atoms_bytewise(atoms.numpy(), 300, 384), scales.numpy())


def test_nvfp4_quantize_matches_oracle_dequant():
    g = torch.Generator().manual_seed(0)
    x = torch.randn(200, 512, generator=g)
    op = lowp.Nvfp4Operand(x)
    ours = op.dequantize().double().numpy()
    ref = olp.nvfp4_dequant(op.data.numpy(), op.atoms.numpy(), op.tensor_scale, 200, 512)
    np.testing.assert_allclose(ours, ref, rtol=1e-6, atol=0)
    # quantisation error of N(0, 1) data in NVFP4 is about 10 % (relative Frobenius)
    err = np.linalg.norm(ref - x.double().numpy()) / np.linalg.norm(x.double().numpy())
    assert 0.05 < err < 0.15
    # block scales: amax(block) / 6 / tensor_scale rounded to E4M3, never above 448
    s = olp.e4m3_decode(op.scales.numpy())
    assert np.all(s <= 448.0) and np.all(s > 0)


def test_fp8_block_quantize_matches_oracle_dequant():
    g = torch.Generator().manual_seed(1)
    x = torch.randn(256, 384, generator=g)
    q, s = lowp.fp8_block_quantize(x)
    assert s.shape == (2, 3)
    ref = olp.fp8_block_dequant(q.numpy(), s.numpy())
    np.testing.assert_allclose(lowp.fp8_block_dequantize(q, s).double().numpy(), ref, rtol=1e-6, atol=0)
    err = np.linalg.norm(ref - x.double().numpy()) / np.linalg.norm(x.double().numpy())
    assert err < 0.04
    # scale = amax / 448 per block, so every block holds a +-448 element
    blocks = np.abs(olp.e4m3_decode(q.numpy())).reshape(2, 128, 3, 128).max(axis=(1, 3))
    np.testing.assert_array_equal(blocks, 448.0)


def test_zero_block_and_zero_tensor():
    x = torch.zeros(128, 256)
    x[5, 17] = 3.0
    op = lowp.Nvfp4Operand(x)
    d = op.dequantize()
    assert d[5, 17].item() == pytest.approx(3.0, rel=0.1)
    assert torch.count_nonzero(d).item() == 1
    z = lowp.Nvfp4Operand(torch.zeros(128, 256))
    assert torch.count_nonzero(z.dequantize()).item() == 0
    q, s = lowp.fp8_block_quantize(torch.zeros(128, 128))
    assert torch.count_nonzero(q).item() == 0 and s.item() == 1.0


def test_scale_bytes_contract():
    from gb300_microbench_b200 import _native as nat
    try:
        lib = nat.bench_lib()
    except nat.NativeLibraryError as exc:
        pytest.skip(f"native library not built: {exc}")
    assert lib.bb_lowp_scale_bytes(nat.BB_LOWP_NVFP4, 300, 384) == 3 * 6 * 512
    assert lib.bb_lowp_scale_bytes(nat.BB_LOWP_FP8_BLOCK128, 300, 384) == 3 * 3 * 4
    assert lib.bb_lowp_scale_bytes(nat.BB_LOWP_NVFP4, 300, 100) == -1
    assert lib.bb_lowp_scale_bytes(9, 300, 384) == -1
