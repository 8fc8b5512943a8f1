"""Low-precision operand formats of the block-scaled GEMMs (8192^3 FP8 128 x 128-block and NVFP4).

NVFP4: E2M1 values (two per byte, element 2i in the low nibble), one
UE4M3 scale per 16 consecutive K elements, and one FP32 scale per tensor:

    x ~= e2m1 * e4m3_block_scale * tensor_scale

with tensor_scale = amax(|x|) / (448 * 6) and block scale = amax(block) / 6 /
tensor_scale rounded to E4M3, values rounded to nearest (ties to even) on
the E2M1 grid {0, 0.5, 1, 1.5, 2, 3, 4, 6}.

FP8 block-scaled: E4M3 values with one FP32 scale per 128 x 128 block,
scale = amax(block) / 448.

The kernels read the NVFP4 block scales in "scale atoms": for each group of
128 rows and each 64 K elements (4 scales per row), 512 bytes in which the
scale j of row r sits at byte (r % 32) * 16 + (r // 32) * 4 + j. One atom is
what one ``tcgen05.cp.32x128b.warpx4`` moves into TMEM for one K = 64 MMA.
"""
from __future__ import annotations

import ctypes

import torch

from . import _native as nat

E2M1_GRID = torch.tensor([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0])
E4M3_MAX = 448.0
E2M1_MAX = 6.0


def _e2m1_codes(y: torch.Tensor) -> torch.Tensor:
    """Round |y| <= 6 to the E2M1 grid (nearest, ties to the even code) and
    return 4-bit codes (sign in bit 3)."""
    a = y.abs().clamp(max=E2M1_MAX)
    grid = E2M1_GRID.to(y.device)
    # Midpoints between grid points; ties go to the even code.
    mids = (grid[1:] + grid[:-1]) / 2
    idx = torch.bucketize(a, mids, right=False)  # a == mid -> lower index
    tie = (idx < 7) & (a == mids[idx.clamp(max=6)])
    idx = torch.where(tie & (idx % 2 == 1), idx + 1, idx)
    sign = (y < 0) & (idx > 0)
    return (idx | (sign.to(idx.dtype) << 3)).to(torch.uint8)


def e2m1_decode(codes: torch.Tensor) -> torch.Tensor:
    grid = E2M1_GRID.to(codes.device)
    mag = grid[(codes & 7).long()]
    return torch.where((codes & 8) != 0, -mag, mag)


def nvfp4_quantize(x: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor, float]:
    """x (R, K) float32, K % 16 == 0 -> (packed (R, K/2) uint8,
    block scales (R, K/16) uint8 E4M3 bits, tensor scale float)."""
    if x.dim() != 2 or x.shape[1] % 16:
        raise ValueError("x must be (R, K) with K a multiple of 16")
    x = x.float()
    r, k = x.shape
    amax = float(x.abs().max())
    gscale = amax / (E4M3_MAX * E2M1_MAX) if amax > 0 else 1.0
    blocks = x.view(r, k // 16, 16)
    bs = (blocks.abs().amax(dim=2) / E2M1_MAX / gscale).clamp(max=E4M3_MAX)
    bs8 = bs.to(torch.float8_e4m3fn)
    bsf = bs8.float()
    denom = (bsf * gscale).unsqueeze(2)
    y = torch.where(denom > 0, blocks / torch.where(denom > 0, denom, torch.ones_like(denom)),
                    torch.zeros_like(blocks))
    codes = _e2m1_codes(y).view(r, k)
    packed = (codes[:, 0::2] | (codes[:, 1::2] << 4)).contiguous()
    return packed, bs8.view(torch.uint8).contiguous(), gscale


def nvfp4_dequantize(packed: torch.Tensor, scales: torch.Tensor, gscale: float) -> torch.Tensor:
    r, kh = packed.shape
    codes = torch.empty(r, kh * 2, dtype=torch.uint8, device=packed.device)
    codes[:, 0::2] = packed & 0xF
    codes[:, 1::2] = packed >> 4
    vals = e2m1_decode(codes)
    s = scales.view(torch.float8_e4m3fn).float().repeat_interleave(16, dim=1)
    return vals * s * gscale


def pack_scale_atoms(scales: torch.Tensor) -> torch.Tensor:
    """(R, K/16) scale bytes -> (ceil(R/128), ceil(K/64), 512) atoms (rows and
    K padded with zero scales)."""
    r, ks = scales.shape
    rb = -(-r // 128)
    kg = -(-ks // 4)
    padded = torch.zeros(rb * 128, kg * 4, dtype=torch.uint8, device=scales.device)
    padded[:r, :ks] = scales
    # [rb][r32 = row // 32 within block][r % 32][kg][j]
    t = padded.view(rb, 4, 32, kg, 4)
    # atom byte = (r % 32) * 16 + (r // 32) * 4 + j  ->  order [rb][kg][r%32][r//32][j]
    return t.permute(0, 3, 2, 1, 4).contiguous().view(rb, kg, 512)


def fp8_block_quantize(x: torch.Tensor, block: int = 128) -> tuple[torch.Tensor, torch.Tensor]:
    """x (R, K) -> (E4M3 bits (R, K) uint8, FP32 scales (ceil(R/128), ceil(K/128)))
    with scale = amax(block) / 448."""
    x = x.float()
    r, k = x.shape
    rb, kb = -(-r // block), -(-k // block)
    pad = torch.zeros(rb * block, kb * block, device=x.device)
    pad[:r, :k] = x
    blocks = pad.view(rb, block, kb, block)
    amax = blocks.abs().amax(dim=(1, 3))
    scale = torch.where(amax > 0, amax / E4M3_MAX, torch.ones_like(amax))
    q = (blocks / scale[:, None, :, None]).clamp(-E4M3_MAX, E4M3_MAX).to(torch.float8_e4m3fn)
    return q.view(rb * block, kb * block)[:r, :k].contiguous().view(torch.uint8), scale.contiguous()


def fp8_block_dequantize(q: torch.Tensor, scale: torch.Tensor, block: int = 128) -> torch.Tensor:
    v = q.view(torch.float8_e4m3fn).float()
    s = scale.repeat_interleave(block, 0).repeat_interleave(block, 1)[: v.shape[0], : v.shape[1]]
    return v * s


# ------------------------------------------------------------------ operands
class Nvfp4Operand:
    """A quantised NVFP4 operand: packed E2M1 (R, K/2) bytes, scale atoms,
    per-tensor FP32 scale."""

    def __init__(self, x: torch.Tensor):
        self.rows, self.k = x.shape
        packed, scales, self.tensor_scale = nvfp4_quantize(x)
        self.data = packed
        self.scales = scales
        self.atoms = pack_scale_atoms(scales)

    @classmethod
    def from_parts(cls, data: torch.Tensor, scales: torch.Tensor, tensor_scale: float) -> "Nvfp4Operand":
        """An operand from already-encoded parts: packed E2M1 (R, K/2) bytes
        and E4M3 scale bytes (R, K/16)."""
        op = cls.__new__(cls)
        op.rows, op.k = data.shape[0], data.shape[1] * 2
        op.data, op.scales, op.tensor_scale = data.contiguous(), scales.contiguous(), float(tensor_scale)
        op.atoms = pack_scale_atoms(op.scales)
        return op

    def to(self, device) -> "Nvfp4Operand":
        op = Nvfp4Operand.from_parts(self.data.to(device), self.scales.to(device), self.tensor_scale)
        return op

    def dequantize(self) -> torch.Tensor:
        return nvfp4_dequantize(self.data, self.scales, self.tensor_scale)


class Fp8BlockOperand:
    """A quantised FP8 operand: E4M3 (R, K) bytes and FP32 128 x 128 block scales."""

    def __init__(self, x: torch.Tensor):
        self.rows, self.k = x.shape
        self.data, self.scales = fp8_block_quantize(x)

    @classmethod
    def from_parts(cls, data: torch.Tensor, scales: torch.Tensor) -> "Fp8BlockOperand":
        op = cls.__new__(cls)
        op.rows, op.k = data.shape
        op.data, op.scales = data.contiguous(), scales.contiguous().float()
        return op

    def to(self, device) -> "Fp8BlockOperand":
        return Fp8BlockOperand.from_parts(self.data.to(device), self.scales.to(device))

    def dequantize(self) -> torch.Tensor:
        return fp8_block_dequantize(self.data, self.scales)


def config4_inputs(m: int, n: int, k: int, seed: int = 0, device: str | torch.device = "cuda"):
    """The FP32 inputs of the block-scaled GEMMs: A (M, K) and B (N, K) ~ N(0, 1)
    from torch.Generator(seed) (the generator config 0 uses)."""
    g = torch.Generator(device="cpu").manual_seed(seed)
    a = torch.randn(m, k, generator=g)
    b = torch.randn(n, k, generator=g)
    return a.to(device), b.to(device)


# ------------------------------------------------------------------ GEMM plan
KINDS = {"nvfp4": nat.BB_LOWP_NVFP4, "fp8_block128": nat.BB_LOWP_FP8_BLOCK128}


def _check_buffers(kind: str, a, b, d: torch.Tensor, sfa: torch.Tensor, sfb: torch.Tensor, stream) -> None:
    """Every buffer on D's device, contiguous, and at least as large as the
    native side reads: its tensor maps and scale loads are sized from M, N
    and K, not from the buffers."""
    if b.k != a.k or tuple(d.shape) != (a.rows, b.rows):
        raise ValueError("shape mismatch between A, B and D")
    for t in (a.data, b.data, sfa, sfb):
        if not t.is_cuda or not t.is_contiguous():
            raise ValueError("operands must be contiguous CUDA tensors")
        if t.device != d.device:
            raise ValueError(f"operands on {t.device}, D on {d.device}: all must be on one device")
    if stream.device != d.device:
        raise ValueError(f"stream on {stream.device}, tensors on {d.device}")
    row_bytes = a.k // 2 if kind == "nvfp4" else a.k
    for name, op in (("A", a), ("B", b)):
        if op.data.numel() * op.data.element_size() < op.rows * row_bytes:
            raise ValueError(f"{name} data holds fewer than {op.rows} x {row_bytes} bytes")
    scale_kind = nat.BB_LOWP_NVFP4 if kind == "nvfp4" else nat.BB_LOWP_FP8_BLOCK128
    for name, rows, t in (("A", a.rows, sfa), ("B", b.rows, sfb)):
        need = int(nat.bench_lib().bb_lowp_scale_bytes(scale_kind, rows, a.k))
        have = t.numel() * t.element_size()
        if need > 0 and have < need:
            raise ValueError(f"{name} scales hold {have} bytes, the kernel reads {need}")


class LowpGemmPlan:
    """D (M, N) BF16 = dequant(A) @ dequant(B)^T through the sm_100a
    block-scaled kernel (bb_lowp_plan_create of include/b200bench.h)."""

    def __init__(self, kind: str, a, b, d: torch.Tensor, stream: torch.cuda.Stream | None = None):
        if kind not in KINDS:
            raise ValueError(f"unknown kind {kind!r}; expected one of {sorted(KINDS)}")
        if not d.is_cuda or d.dtype != torch.bfloat16 or not d.is_contiguous():
            raise ValueError("D must be a contiguous CUDA bfloat16 tensor")
        self.kind = kind
        self.m, self.n, self.k = a.rows, b.rows, a.k
        if b.k != a.k or tuple(d.shape) != (self.m, self.n):
            raise ValueError("shape mismatch between A, B and D")
        if kind == "nvfp4":
            sfa, sfb, gscale = a.atoms, b.atoms, a.tensor_scale * b.tensor_scale
        else:
            sfa, sfb, gscale = a.scales, b.scales, 1.0
        self.stream = stream if stream is not None else torch.cuda.current_stream(d.device)
        self._lib = nat.bench_lib()
        _check_buffers(kind, a, b, d, sfa, sfb, self.stream)
        self.a, self.b, self.d, self._keep = a, b, d, (sfa, sfb)
        handle = ctypes.c_void_p()
        info = nat.LowpInfo()
        with torch.cuda.device(d.device):
            nat.check("bb_lowp_plan_create", self._lib.bb_lowp_plan_create(
                KINDS[kind], self.m, self.n, self.k, a.data.data_ptr(), b.data.data_ptr(), sfa.data_ptr(),
                sfb.data_ptr(), float(gscale), d.data_ptr(), self.stream.cuda_stream, ctypes.byref(handle),
                ctypes.byref(info)))
        self._handle = handle
        self.info = info.as_dict()

    @property
    def flops(self) -> int:
        return 2 * self.m * self.n * self.k

    def run(self, iterations: int = 1) -> None:
        nat.check("bb_lowp_execute_n", self._lib.bb_lowp_execute_n(self._handle, int(iterations)))

    def synchronize(self) -> None:
        nat.check("bb_lowp_synchronize", self._lib.bb_lowp_synchronize(self._handle))

    @property
    def launches(self) -> int:
        return int(self._lib.bb_lowp_launches(self._handle))

    def close(self) -> None:
        if getattr(self, "_handle", None):
            self._lib.bb_lowp_destroy(self._handle)
            self._handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class CublasLtLowpPlan:
    """cuBLASLt's block-scaled GEMM on the same operands (the comparator, a
    library call; bb_cmp_lowp_plan_create of include/b200cmp.h).

    ``fp8_scales_kmajor`` chooses how the FP32 128 x 128 block scales are
    handed over: True passes them as stored ([row block][K block]), False
    passes the transpose ([K block][row block])."""

    CMP_KINDS = {**KINDS, "fp8_tensor_scaled": 3}

    def __init__(self, kind: str, a, b, d: torch.Tensor, autotune: bool = False,
                 stream: torch.cuda.Stream | None = None, fp8_scales_kmajor: bool = False):
        """kind "fp8_tensor_scaled" runs cuBLASLt's plain FP8 GEMM on the
        same E4M3 bytes without block scales: a throughput reference for the
        FP8 block-scaled kernel, not the same function."""
        if kind not in self.CMP_KINDS:
            raise ValueError(f"unknown kind {kind!r}")
        self._lib = nat.cmp_lib()
        self.stream = stream if stream is not None else torch.cuda.current_stream(d.device)
        m, n, k = a.rows, b.rows, a.k
        if kind == "nvfp4":
            sfa, sfb, gscale = a.atoms, b.atoms, a.tensor_scale * b.tensor_scale
        else:
            sfa, sfb, gscale = a.scales, b.scales, 1.0
            if kind != "fp8_tensor_scaled" and not fp8_scales_kmajor:
                sfa, sfb = sfa.t().contiguous(), sfb.t().contiguous()
        if not d.is_cuda or d.dtype != torch.bfloat16 or not d.is_contiguous():
            raise ValueError("D must be a contiguous CUDA bfloat16 tensor")
        _check_buffers(kind, a, b, d, sfa, sfb, self.stream)
        self._keep = (a, b, sfa, sfb, d)
        handle = ctypes.c_void_p()
        info = nat.CmpInfo()
        rc = self._lib.bb_cmp_lowp_plan_create(self.CMP_KINDS[kind], m, n, k, a.data.data_ptr(), b.data.data_ptr(),
                                               sfa.data_ptr(), sfb.data_ptr(), float(gscale), d.data_ptr(),
                                               1 if autotune else 0, self.stream.cuda_stream, ctypes.byref(handle),
                                               ctypes.byref(info))
        if rc != 0:
            raise nat.NativeCallError("bb_cmp_lowp_plan_create", rc, self._lib.bb_cmp_last_error().decode())
        self._handle = handle
        self.info = info.as_dict()

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
