"""Python face of the HBM->SMEM streaming kernels (LDGSTS and 2D TMA).

Replaces the per-specialisation drivers of the reference
(memory_paths/ldgsts.cu:774-941, memory_paths/tma.cu:1110-1290): geometry,
validation against the SplitMix64 pattern, and timed launches, here as
calls through the C ABI on caller-owned torch buffers.
"""
from __future__ import annotations

import ctypes

import torch

from . import _native as nat

METHODS = {"ldgsts": nat.BB_COPY_LDGSTS, "tma": nat.BB_COPY_TMA}

# Reference campaign grid (memory_paths/benchmark.py:13-16) and the
# streaming-benchmark grid of the B200 build (stages {2,3,4}).
REFERENCE_STAGES = (2, 4, 8)
BASELINE_STAGES = (2, 3, 4)
BIF_KIB = (16, 32, 64)


def plan(method: str, stages: int, bif_kib: int, nbytes: int, row_bytes: int = 256, sm_count: int = 0) -> dict:
    """Geometry of one configuration (host only when sm_count > 0)."""
    info = nat.CopyInfo()
    nat.check("bb_copy_plan", nat.bench_lib().bb_copy_plan(
        METHODS[method], stages, bif_kib, row_bytes, nbytes, sm_count, ctypes.byref(info)))
    return info.as_dict()


def _stream(stream):
    return (stream if stream is not None else torch.cuda.current_stream()).cuda_stream


def _check_buffer(buf: torch.Tensor) -> None:
    if not buf.is_cuda or not buf.is_contiguous():
        raise ValueError("the buffer must be a contiguous CUDA tensor")


def fill_pattern(buf: torch.Tensor, stream=None) -> None:
    _check_buffer(buf)
    nat.check("bb_fill_pattern", nat.bench_lib().bb_fill_pattern(buf.data_ptr(), buf.numel() * buf.element_size(),
                                                                  _stream(stream)))


def fill_uniform_u32(buf: torch.Tensor, seed: int = 0, stream=None) -> None:
    _check_buffer(buf)
    nat.check("bb_fill_uniform_u32", nat.bench_lib().bb_fill_uniform_u32(
        buf.data_ptr(), buf.numel() * buf.element_size(), seed, _stream(stream)))


class StreamingRun:
    """One (method, stages, bytes-in-flight) configuration over one buffer."""

    def __init__(self, method: str, stages: int, bif_kib: int, src: torch.Tensor, row_bytes: int = 256,
                 nbytes: int | None = None, stream=None):
        if method not in METHODS:
            raise ValueError(f"unknown method {method!r}")
        if not src.is_cuda or not src.is_contiguous():
            raise ValueError("src must be a contiguous CUDA tensor")
        self.method, self.stages, self.bif_kib, self.row_bytes = method, stages, bif_kib, row_bytes
        self.src = src
        have = src.numel() * src.element_size()
        self.nbytes = int(nbytes if nbytes is not None else have)
        if not 0 < self.nbytes <= have:
            raise ValueError(f"nbytes={self.nbytes} must be in (0, {have}], the size of src")
        self.stream = stream if stream is not None else torch.cuda.current_stream(src.device)
        self.info = plan(method, stages, bif_kib, self.nbytes, row_bytes)
        dev = src.device
        self.sink = torch.zeros(self.info["grid_ctas"], dtype=torch.int32, device=dev)
        self.status = torch.zeros(1, dtype=torch.int32, device=dev)
        self.mismatches = torch.zeros(1, dtype=torch.int64, device=dev)
        self._lib = nat.bench_lib()

    def run(self, passes: int = 1, rotation: int = 0) -> None:
        nat.check("bb_copy_run", self._lib.bb_copy_run(
            METHODS[self.method], self.stages, self.bif_kib, self.row_bytes, self.src.data_ptr(), self.nbytes,
            passes, rotation, self.sink.data_ptr(), self.status.data_ptr(), self.stream.cuda_stream))

    def validate(self) -> int:
        """Mismatching 16-byte vectors against the SplitMix64 pattern."""
        self.mismatches.zero_()
        nat.check("bb_copy_validate", self._lib.bb_copy_validate(
            METHODS[self.method], self.stages, self.bif_kib, self.row_bytes, self.src.data_ptr(), self.nbytes,
            self.sink.data_ptr(), self.mismatches.data_ptr(), self.status.data_ptr(), self.stream.cuda_stream))
        self.stream.synchronize()
        self.check_status()
        return int(self.mismatches.item())

    def check_status(self) -> None:
        st = int(self.status.item())
        if st != 0:
            raise nat.NativeCallError("copy kernel", nat.BB_ERR_TIMEOUT, f"device status 0x{st:x}")

    def checksums(self) -> list[int]:
        self.stream.synchronize()
        return [int(x) & 0xFFFFFFFF for x in self.sink.cpu().tolist()]
