"""Configuration-grid sweeps writing one raw CSV each: the reference's
``memory_paths/benchmark.py`` and ``umma_throughput/benchmark.py``, run in
process instead of one subprocess per configuration.

    python -m gb300_microbench_b200.cli.sweeps memory --run-kind {smoke,benchmark} --output FILE
        [--grid {reference,baseline}] [--working-set-mib N] [--passes N] [--warmup-ms N] [--repetitions N]
    python -m gb300_microbench_b200.cli.sweeps umma --run-kind {smoke,benchmark} --output FILE
        [--grid {reference,baseline}] [--iterations N] [--warmup-iterations N] [--repetitions N]

``--grid reference`` is the reference's grid and defaults (memory:
stages {2,4,8} x bytes in flight {16,32,64} KiB x {ldgsts,tma}, 512 MiB x
32 passes; UMMA: N {64,128,256} x depth {4,16,64,256} x {1sm,2sm}), so the
output passes the reference's campaign validators unchanged.
``--grid baseline`` is the B200 build's streaming/UMMA grid: stages {2,3,4},
a 4 GiB seeded uniform buffer read once, 128-byte TMA rows; depths
{16,32,64,128,256} with N(0,1) operands. Each configuration is flushed to the
file as soon as it completes (memory_paths/benchmark.py:99-100).
"""
from __future__ import annotations

import argparse
import os
import sys
from pathlib import Path

from . import common as cm
from . import memory_paths as mp
from . import umma as um

MEMORY_DEFAULTS = {"smoke": (64, 2, 200, 5), "benchmark": (512, 32, 2000, 30)}  # memory_paths/benchmark.py:58-62
UMMA_DEFAULTS = {"smoke": (20, 5, 3), "benchmark": (1000, 10, 30)}  # umma_throughput/benchmark.py:58-61


def _pos(minimum):
    def parse(text):
        v = int(text)
        if v < minimum:
            raise argparse.ArgumentTypeError(f"must be >= {minimum}")
        return v
    return parse


def parse_args(argv):
    ap = argparse.ArgumentParser(prog="sweeps", description="Run a configuration grid and write one raw CSV.")
    ap.add_argument("experiment", choices=("memory", "umma"))
    ap.add_argument("--run-kind", required=True, choices=("smoke", "benchmark"))
    ap.add_argument("--output", required=True, type=Path)
    ap.add_argument("--grid", choices=("reference", "baseline"), default="reference")
    ap.add_argument("--working-set-mib", type=_pos(1))
    ap.add_argument("--passes", type=_pos(1))
    ap.add_argument("--warmup-ms", type=_pos(0))
    ap.add_argument("--iterations", type=_pos(1))
    ap.add_argument("--warmup-iterations", type=_pos(0))
    ap.add_argument("--repetitions", type=_pos(1))
    return ap.parse_args(argv)


def memory(args, gpu) -> int:
    ws, passes, warmup, reps = MEMORY_DEFAULTS[args.run_kind]
    if args.grid == "baseline":
        ws, passes, stages_set, fill, row_bytes = 4096, 1, (2, 3, 4), "uniform", 128
    else:
        stages_set, fill, row_bytes = mp.REFERENCE_STAGES, "pattern", 256
    ws = args.working_set_mib or ws
    passes = args.passes or passes
    warmup = warmup if args.warmup_ms is None else args.warmup_ms
    reps = args.repetitions or reps
    written = 0
    args.output.parent.mkdir(parents=True, exist_ok=True)
    with args.output.open("w", encoding="utf-8") as out:
        header = True
        for stages in stages_set:
            for bif in mp.BIF_KIB:
                for method in mp.METHODS:
                    cm.eprint(f"memory_paths: {method} stages={stages} bytes_in_flight_kib={bif}")
                    cfg = {"stages": stages, "bif_kib": bif, "run_kind": args.run_kind, "working_set_mib": ws,
                           "passes": passes, "warmup_ms": warmup, "repetitions": reps, "fill": fill, "seed": 0,
                           "row_bytes": row_bytes}
                    mp.run_config(method, cfg, gpu, gpu.uuid, print_header=header, out=out)
                    header = False
                    out.flush()
                    written += reps
    cm.eprint(f"memory_paths: wrote {written} rows to {args.output}")
    return cm.EXIT_OK


def umma(args, gpu) -> int:
    iters, warmup, reps = UMMA_DEFAULTS[args.run_kind]
    iters = args.iterations or iters
    warmup = warmup if args.warmup_iterations is None else args.warmup_iterations
    reps = args.repetitions or reps
    depths, operands = (um.REFERENCE_DEPTHS, "pattern") if args.grid == "reference" else ((16, 32, 64, 128, 256),
                                                                                            "random")
    written = 0
    args.output.parent.mkdir(parents=True, exist_ok=True)
    with args.output.open("w", encoding="utf-8") as out:
        header = True
        for n in um.N_VALUES:
            for depth in depths:
                for method in um.METHODS:
                    cm.eprint(f"umma_throughput: {method} n={n} depth={depth}")
                    cfg = {"run_kind": args.run_kind, "n": n, "depth": depth, "iterations": iters,
                           "warmup_iterations": warmup, "repetitions": reps, "operands": operands, "seed": 0}
                    um.run_config(method, cfg, gpu, print_header=header, out=out)
                    header = False
                    out.flush()
                    written += reps
    cm.eprint(f"umma_throughput: wrote {written} rows to {args.output}")
    return cm.EXIT_OK


def main(argv=None) -> int:
    args = parse_args(sys.argv[1:] if argv is None else argv)
    try:
        gpu = cm.query_gpu()
        os.environ.setdefault("EXPECTED_GPU_UUID", gpu.uuid)
        cm.expected_uuid(gpu)
        return memory(args, gpu) if args.experiment == "memory" else umma(args, gpu)
    except cm.RunFailure as exc:
        cm.eprint(f"sweeps: ERROR: {exc}")
        return cm.EXIT_FAILURE


if __name__ == "__main__":
    raise SystemExit(main())
