"""Shared pieces of the command-line drivers: provenance, CSV formatting,
exit codes, argument helpers. Mirrors the host halves of the reference
binaries (memory_paths/ldgsts.cu:375-700, umma_throughput/umma_1sm.cu:
620-700) without any of their GPU checks that pin compute capability 10.3:
this build requires 10.0 (B200, sm_100a)."""
from __future__ import annotations

import datetime as _dt
import os
import subprocess
import sys
from dataclasses import dataclass
from pathlib import Path

EXIT_OK = 0
EXIT_FAILURE = 1
EXIT_USAGE = 2

REPO_ROOT = Path(__file__).resolve().parents[2]


class UsageError(Exception):
    pass


class RunFailure(Exception):
    pass


def eprint(*args):
    print(*args, file=sys.stderr, flush=True)


def now_utc_iso8601() -> str:
    return _dt.datetime.now(_dt.timezone.utc).strftime("%Y-%m-%dT%H:%M:%SZ")


def csv_quote(s: str) -> str:
    return '"' + s.replace('"', '""') + '"'


def fixed6(x: float) -> str:
    """std::fixed << std::setprecision(6), as the reference's CSV writers."""
    return f"{x:.6f}"


def git_commit_hash() -> str:
    """HEAD of this checkout; B200_GIT_COMMIT overrides it where the tree was
    copied without .git (a launcher passes the commit it copied)."""
    if os.environ.get("B200_GIT_COMMIT"):
        return os.environ["B200_GIT_COMMIT"]
    try:
        out = subprocess.run(["git", "rev-parse", "HEAD"], cwd=REPO_ROOT, capture_output=True, text=True)
        return out.stdout.strip() if out.returncode == 0 and out.stdout.strip() else "UNKNOWN"
    except OSError:
        return "UNKNOWN"


def git_dirty_flag() -> str:
    if os.environ.get("B200_GIT_DIRTY") in ("true", "false"):
        return os.environ["B200_GIT_DIRTY"]
    try:
        out = subprocess.run(["git", "status", "--porcelain"], cwd=REPO_ROOT, capture_output=True, text=True)
        if out.returncode != 0:
            return "unknown"
        return "true" if out.stdout.strip() else "false"
    except OSError:
        return "unknown"


@dataclass
class GpuInfo:
    name: str
    uuid: str
    major: int
    minor: int
    sm_count: int
    l2_bytes: int
    smem_per_sm_bytes: int
    driver_version: int
    runtime_version: int

    @property
    def compute_capability(self) -> str:
        return f"{self.major}.{self.minor}"


def query_gpu() -> GpuInfo:
    """Exactly one visible device, compute capability 10.0 (ldgsts.cu:390-440
    requires one device at 10.3; this build targets sm_100a)."""
    import ctypes

    import torch

    if not torch.cuda.is_available():
        raise RunFailure("no CUDA device is visible")
    n = torch.cuda.device_count()
    if n != 1:
        raise RunFailure(f"expected exactly 1 visible CUDA device, found {n}")
    torch.cuda.set_device(0)
    p = torch.cuda.get_device_properties(0)
    if (p.major, p.minor) != (10, 0):
        raise RunFailure(f"expected compute capability 10.0 (sm_100a), found {p.major}.{p.minor}")
    uuid = "GPU-" + str(p.uuid)
    rt = 0
    if torch.version.cuda:
        major, minor = (int(x) for x in torch.version.cuda.split(".")[:2])
        rt = major * 1000 + minor * 10
    drv = 0
    try:
        libcuda = ctypes.CDLL("libcuda.so.1")
        v = ctypes.c_int()
        if libcuda.cuDriverGetVersion(ctypes.byref(v)) == 0:
            drv = v.value
    except OSError:
        drv = 0
    return GpuInfo(name=p.name, uuid=uuid, major=p.major, minor=p.minor, sm_count=p.multi_processor_count,
                   l2_bytes=int(p.L2_cache_size), smem_per_sm_bytes=int(p.shared_memory_per_multiprocessor),
                   driver_version=drv, runtime_version=rt)


def expected_uuid(gpu: GpuInfo) -> str:
    """EXPECTED_GPU_UUID must be set and name the visible device (the
    reference's launcher sets it: scripts/run_gpu.sh:47-58)."""
    want = os.environ.get("EXPECTED_GPU_UUID", "")
    if not want:
        raise RunFailure("EXPECTED_GPU_UUID is not set; run through gb300_microbench_b200.cli.launch")
    if want != gpu.uuid:
        raise RunFailure(f"EXPECTED_GPU_UUID={want} does not match the visible device {gpu.uuid}")
    return want


def parse_int(text: str, lo: int, hi: int, flag: str) -> int:
    try:
        v = int(text, 10)
    except (TypeError, ValueError):
        raise UsageError(f"{flag} must be an integer in [{lo}, {hi}]")
    if v < lo or v > hi:
        raise UsageError(f"{flag} must be an integer in [{lo}, {hi}]")
    return v


def take_value(argv: list[str], i: int, flag: str) -> tuple[str, int]:
    if i + 1 >= len(argv):
        raise UsageError(f"{flag} needs a value")
    return argv[i + 1], i + 2
