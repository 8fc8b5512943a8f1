"""CPU oracle for the block-scaled GEMMs. TEST INFRASTRUCTURE ONLY.

The reference has no low-precision GEMM (this path is new work), so
this module restates the operand formats from their published definitions
and the check the configuration names: an FP32 matmul of the dequantised
inputs, relative Frobenius error <= 2e-2.

* E2M1 (OCP Microscaling spec v1.0, FP4): 1 sign, 2 exponent (bias 1),
  1 mantissa bit; codes 0..7 are 0, 0.5, 1, 1.5, 2, 3, 4, 6.
* E4M3 (OCP FP8 spec, "FN" variant): 1 sign, 4 exponent (bias 7), 3
  mantissa bits, subnormals, no infinities, S.1111.111 is NaN; max 448.
* NVFP4 block scales: one unsigned E4M3 per 16 K elements; 512-byte atoms
  per (128-row block, 64-wide K group), scale j of row r at byte
  (r % 32) * 16 + (r // 32) * 4 + j.
* FP8 block scales: one FP32 per 128 x 128 block.

Everything is decoded bit by bit with numpy here, independently of the
torch dtypes the product's quantiser uses.
"""
from __future__ import annotations

import numpy as np

E2M1_VALUES = np.array([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0], dtype=np.float64)


def e2m1_decode(codes: np.ndarray) -> np.ndarray:
    codes = np.asarray(codes, dtype=np.uint8)
    mag = E2M1_VALUES[codes & 7]
    return np.where(codes & 8, -mag, mag)


def e4m3_decode(bits: np.ndarray) -> np.ndarray:
    bits = np.asarray(bits, dtype=np.uint8).astype(np.int64)
    sign = np.where(bits & 0x80, -1.0, 1.0)
    exp = (bits >> 3) & 0xF
    man = bits & 0x7
    normal = (1.0 + man / 8.0) * np.exp2(exp - 7.0)
    sub = (man / 8.0) * np.exp2(-6.0)
    val = np.where(exp == 0, sub, normal)
    val = np.where((exp == 0xF) & (man == 0x7), np.nan, val)
    return sign * val


def unpack_fp4(packed: np.ndarray) -> np.ndarray:
    """(R, K/2) bytes -> (R, K) codes, element 2i from the low nibble."""
    packed = np.asarray(packed, dtype=np.uint8)
    r, kh = packed.shape
    out = np.empty((r, 2 * kh), dtype=np.uint8)
    out[:, 0::2] = packed & 0xF
    out[:, 1::2] = packed >> 4
    return out


def unpack_scale_atoms(atoms: np.ndarray, rows: int, k: int) -> np.ndarray:
    """Atoms (flat bytes, [rb][K/64][512]) -> (rows, K/16) scale bytes.

    Byte (r % 32) * 16 + (r // 32) * 4 + j of atom (rb, g) is scale j of row
    rb * 128 + r in K group g: viewed as [rb][g][r % 32][r // 32][j]."""
    atoms = np.asarray(atoms, dtype=np.uint8).reshape(-1)
    rb = -(-rows // 128)
    kg = k // 64
    v = atoms[: rb * kg * 512].reshape(rb, kg, 32, 4, 4)
    out = v.transpose(0, 3, 2, 1, 4).reshape(rb * 128, kg * 4)
    return np.ascontiguousarray(out[:rows])


def unpack_scale_atoms_bytewise(atoms: np.ndarray, rows: int, k: int) -> np.ndarray:
    """The same unpacking one byte at a time (small cases: cross-checks the
    vectorised form)."""
    atoms = np.asarray(atoms, dtype=np.uint8).reshape(-1)
    kg = k // 64
    out = np.empty((rows, kg * 4), dtype=np.uint8)
    for r in range(rows):
        blk, rr = divmod(r, 128)
        for g in range(kg):
            for j in range(4):
                out[r, 4 * g + j] = atoms[(blk * kg + g) * 512 + (rr % 32) * 16 + (rr // 32) * 4 + j]
    return out


def nvfp4_dequant(packed: np.ndarray, atoms: np.ndarray, tensor_scale: float, rows: int, k: int) -> np.ndarray:
    vals = e2m1_decode(unpack_fp4(packed))
    scales = e4m3_decode(unpack_scale_atoms(atoms, rows, k))
    return vals * np.repeat(scales, 16, axis=1) * tensor_scale


def fp8_block_dequant(q: np.ndarray, scales: np.ndarray, block: int = 128) -> np.ndarray:
    v = e4m3_decode(q)
    s = np.repeat(np.repeat(np.asarray(scales, dtype=np.float64), block, 0), block, 1)
    return v * s[: v.shape[0], : v.shape[1]]


def gemm_dequant_fp32(a_deq: np.ndarray, b_deq: np.ndarray) -> np.ndarray:
    """The block-scaled GEMMs' check: FP32 matmul of the dequantised inputs."""
    return a_deq.astype(np.float32) @ b_deq.astype(np.float32).T
