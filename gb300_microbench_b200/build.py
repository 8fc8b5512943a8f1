"""Builds the native libraries of this package in-tree, for sm_100a only.

    python -m gb300_microbench_b200.build [--force] [--jobs N]

Produces ``gb300_microbench_b200/lib/libb200bench.so`` (the kernels and their
C ABI, ``include/b200bench.h``) and ``gb300_microbench_b200/lib/libb200cmp.so``
(the cuBLASLt comparator, ``include/b200cmp.h``). nvcc cross-compiles without
a GPU, so this runs on a CPU-only machine. Sources are recompiled only when
they (or a header) are newer than the library, unless ``--force``.
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
LIB = PKG / "lib"
OBJ = LIB / "obj"
INCLUDE = ROOT / "include"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC,-fvisibility=hidden",
                     "-I", str(INCLUDE), "--expt-relaxed-constexpr"]

BENCH_SOURCES = [
    "common.cu",
    "gemm_sm100.cu",
    "gemm_capi.cu",
    "gemm_noalloc.cu",
    "gemm_lowp.cu",
    "copy_kernels.cu",
    "umma_probe.cu",
]
CMP_SOURCES = ["cublaslt_cmp.cu"]

BENCH_LIB = LIB / "libb200bench.so"
CMP_LIB = LIB / "libb200cmp.so"


def nvcc() -> str:
    path = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(path).exists():
        raise RuntimeError("nvcc not found; the CUDA toolkit is required to build")
    return path


def _headers() -> list[Path]:
    return list(CSRC.glob("*.cuh")) + list(INCLUDE.glob("*.h"))


def _stale(target: Path, sources: list[Path]) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(s.stat().st_mtime > t for s in sources + _headers())


def _compile(src: Path, force: bool) -> Path:
    obj = OBJ / (src.stem + ".o")
    if force or _stale(obj, [src]):
        cmd = [nvcc(), *NVCC_FLAGS, "-c", str(src), "-o", str(obj)]
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"nvcc failed for {src.name}:\n{res.stdout}\n{res.stderr}")
    return obj


def _link(target: Path, objs: list[Path], extra: list[str]) -> None:
    cmd = [nvcc(), *ARCH, "-shared", "-o", str(target), *map(str, objs), *extra]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"link failed for {target.name}:\n{res.stdout}\n{res.stderr}")


def build(force: bool = False, jobs: int | None = None, verbose: bool = False) -> dict[str, Path]:
    OBJ.mkdir(parents=True, exist_ok=True)
    jobs = jobs or min(8, os.cpu_count() or 1)
    bench_src = [CSRC / s for s in BENCH_SOURCES]
    cmp_src = [CSRC / s for s in CMP_SOURCES]
    need_bench = force or _stale(BENCH_LIB, bench_src)
    need_cmp = force or _stale(CMP_LIB, cmp_src)
    todo = (bench_src if need_bench else []) + (cmp_src if need_cmp else [])
    with cf.ThreadPoolExecutor(max_workers=jobs) as ex:
        objs = dict(zip(todo, ex.map(lambda s: _compile(s, force), todo)))
    if need_bench:
        _link(BENCH_LIB, [objs[s] for s in bench_src], [])
        if verbose:
            print(f"built {BENCH_LIB}", file=sys.stderr)
    if need_cmp:
        _link(CMP_LIB, [objs[s] for s in cmp_src], ["-lcublasLt", "-Xlinker", "-rpath=/usr/local/cuda/lib64"])
        if verbose:
            print(f"built {CMP_LIB}", file=sys.stderr)
    return {"bench": BENCH_LIB, "cmp": CMP_LIB}


def main(argv: list[str] | None = None) -> int:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--jobs", type=int, default=None)
    args = ap.parse_args(argv)
    build(force=args.force, jobs=args.jobs, verbose=True)
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
