#!/usr/bin/env python3
"""The reference's own HBM->SMEM and UMMA microbenchmarks beside this
build's, on the same B200 (one GPU).

    make -C baseline REFERENCE=/path/to/the/reference kernels   # once, on any machine
    python baseline/run_reference_kernels.py [--repetitions N] [--warmup-ms N] [--out-dir results]

Runs the reference binaries built by baseline/Makefile (memory_paths/ldgsts,
tma; umma_throughput/umma_1sm, umma_2sm) over the reference's own grids
(memory_paths/benchmark.py: stages {2,4,8} x bytes in flight {16,32,64} KiB,
512 MiB working set x 32 passes; umma_throughput/benchmark.py: N {64,128,256}
x depth {4,16,64,256}, 1000 iterations, 10 warm-up launches), then this
build's CLIs with the same flags, and writes one side-by-side CSV per
experiment. Every row of either side must report PASS; the comparison is
the median over the repetitions of effective GB/s (memory) and of FLOP per
cycle per SM pair / SM (UMMA, the CSVs' flops_per_cycle).

The binaries are the reference's, built for sm_100a; they refuse any GPU but
compute capability 10.3 in their host code, which ref_b200_shim.h answers
(their rows carry compute_capability 10.3; the true value is recorded in
the "device_cc" column here). Only for one-GPU runs: the binaries require
exactly one visible device.
"""
from __future__ import annotations

import argparse
import contextlib
import csv
import io
import os
import statistics
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]
BIN = ROOT / "baseline" / "_ref" / "bin"
sys.path.insert(0, str(ROOT))

MEM_STAGES = (2, 4, 8)
MEM_BIF = (16, 32, 64)
UMMA_N = (64, 128, 256)
UMMA_DEPTH = (4, 16, 64, 256)


def gpu_uuid() -> str:
    import torch

    return "GPU-" + str(torch.cuda.get_device_properties(0).uuid)


def run_reference(binary: str, args: list[str], env: dict) -> list[dict]:
    res = subprocess.run([str(BIN / binary), *args], capture_output=True, text=True, env=env, check=False)
    if res.returncode != 0:
        raise RuntimeError(f"reference {binary} {' '.join(args)} exited {res.returncode}: {res.stderr[-2000:]}")
    return list(csv.DictReader(io.StringIO(res.stdout)))


def run_ours(module, method: str, args: list[str]) -> list[dict]:
    buf = io.StringIO()
    with contextlib.redirect_stdout(buf):
        rc = module.main([method, *args])
    if rc != 0:
        raise RuntimeError(f"ours {method} {' '.join(args)} exited {rc}")
    return list(csv.DictReader(io.StringIO(buf.getvalue())))


def median(rows: list[dict], key: str) -> float:
    return statistics.median(float(r[key]) for r in rows)


def passed(rows: list[dict]) -> bool:
    return bool(rows) and all(r["correctness"] in ("OK", "PASS") for r in rows)


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--repetitions", type=int, default=10)
    ap.add_argument("--warmup-ms", type=int, default=500)
    ap.add_argument("--out-dir", default=str(ROOT / "results"))
    ap.add_argument("--only", choices=("memory", "umma"), default=None)
    args = ap.parse_args(argv)

    import torch

    from gb300_microbench_b200.cli import memory_paths, umma

    if not BIN.is_dir():
        print(f"{BIN} is missing: make -C baseline REFERENCE=... kernels", file=sys.stderr)
        return 2
    env = dict(os.environ, EXPECTED_GPU_UUID=gpu_uuid())
    os.environ["EXPECTED_GPU_UUID"] = env["EXPECTED_GPU_UUID"]  # this build's CLIs check it too
    props = torch.cuda.get_device_properties(0)
    device = {"gpu_name": props.name, "device_cc": f"{props.major}.{props.minor}"}
    out_dir = Path(args.out_dir)
    out_dir.mkdir(parents=True, exist_ok=True)

    for binary in ("ldgsts", "tma", "umma_1sm", "umma_2sm"):
        if args.only and not binary.startswith({"memory": ("ldgsts", "tma"), "umma": ("umma",)}[args.only]):
            continue
        res = subprocess.run([str(BIN / binary), "--self-test"], capture_output=True, text=True, env=env, check=False)
        print(f"reference {binary} --self-test: exit {res.returncode}", file=sys.stderr)
        if res.returncode != 0:
            print(res.stderr[-2000:], file=sys.stderr)
            return 1

    if args.only in (None, "memory"):
        rows = []
        for method in ("ldgsts", "tma"):
            for stages in MEM_STAGES:
                for bif in MEM_BIF:
                    flags = ["--stages", str(stages), "--bytes-in-flight-kib", str(bif), "--run-kind", "benchmark",
                             "--working-set-mib", "512", "--passes", "32", "--warmup-ms", str(args.warmup_ms),
                             "--repetitions", str(args.repetitions)]
                    ref = run_reference(method, flags, env)
                    ours = run_ours(memory_paths, method, flags)
                    r_gbps, o_gbps = median(ref, "effective_gbps"), median(ours, "effective_gbps")
                    rows.append({"method": method, "stages": stages, "bytes_in_flight_kib": bif,
                                 "reference_gbps_median": f"{r_gbps:.1f}", "ours_gbps_median": f"{o_gbps:.1f}",
                                 "ours_over_reference": f"{o_gbps / r_gbps:.3f}",
                                 "reference_correctness": "PASS" if passed(ref) else "FAIL",
                                 "ours_correctness": "PASS" if passed(ours) else "FAIL",
                                 "repetitions": args.repetitions, "working_set_mib": 512, "passes": 32, **device})
                    print(f"{method} s={stages} bif={bif}: reference {r_gbps:.0f} GB/s, ours {o_gbps:.0f} GB/s",
                          file=sys.stderr)
        write(out_dir / "reference_on_b200_memory.csv", rows)

    if args.only in (None, "umma"):
        rows = []
        for method in ("umma_1sm", "umma_2sm"):
            for n in UMMA_N:
                for depth in UMMA_DEPTH:
                    flags = ["--run-kind", "benchmark", "--n", str(n), "--depth", str(depth), "--iterations", "1000",
                             "--warmup-iterations", "10", "--repetitions", str(args.repetitions)]
                    ref = run_reference(method, flags, env)
                    ours = run_ours(umma, method, flags)
                    r_f, o_f = median(ref, "flops_per_cycle"), median(ours, "flops_per_cycle")
                    rows.append({"method": method, "n": n, "depth": depth,
                                 "reference_flops_per_cycle_median": f"{r_f:.1f}",
                                 "ours_flops_per_cycle_median": f"{o_f:.1f}", "ours_over_reference": f"{o_f / r_f:.3f}",
                                 "reference_correctness": "PASS" if passed(ref) else "FAIL",
                                 "ours_correctness": "PASS" if passed(ours) else "FAIL",
                                 "iterations": 1000, "repetitions": args.repetitions, **device})
                    print(f"{method} n={n} d={depth}: reference {r_f:.0f}, ours {o_f:.0f} FLOP/cycle", file=sys.stderr)
        write(out_dir / "reference_on_b200_umma.csv", rows)
    return 0


def write(path: Path, rows: list[dict]) -> None:
    with path.open("w", newline="") as fh:
        w = csv.DictWriter(fh, fieldnames=list(rows[0]), lineterminator="\n")
        w.writeheader()
        w.writerows(rows)
    print(f"wrote {path}", file=sys.stderr)


if __name__ == "__main__":
    raise SystemExit(main())
