"""Multi-GPU GEMM sweep: the five frozen shapes (gemm_comparison.py:116-122, or --shapes)
row-sharded over the ranks of one node, B replicated, in baseline mode
(N(0,1) seed-0 BF16 operands, BF16 C). One process per GPU:

    python -m torch.distributed.run --nproc-per-node P --master-addr 127.0.0.1 \\
        -m gb300_microbench_b200.cli.multigpu [--iterations N] [--warmup-iterations N] [--output FILE]
        [--shapes MxNxK,...]

Each rank times its own block with CUDA events (N back-to-back launches
after warm-up); the shape's time is the max over ranks and the aggregate
TFLOP/s is 2MNK / that time (strong scaling: the global problem is fixed).
C is then all-gathered over NCCL (off the timed path) and checked on rank 0
against an FP32 matmul of the operands (relative Frobenius <= 1e-2). Rank 0
writes one CSV row per shape.
"""
from __future__ import annotations

import argparse
import csv
import os
import sys

from . import common as cm

SHAPES = ((4096, 4096, 4096), (8192, 8192, 8192), (16384, 512, 4096), (32768, 512, 4096), (512, 16384, 4096))
FIELDS = ("shape_id", "n_gpus", "rows_per_rank_max", "variant", "tile_n", "kernel_time_ms_max", "tflops_aggregate",
          "tflops_per_gpu", "rel_frobenius", "correctness", "gpu_name", "git_commit")


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="multigpu")
    ap.add_argument("--iterations", type=int, default=20)
    ap.add_argument("--warmup-iterations", type=int, default=5)
    ap.add_argument("--variant", default="tuned")
    ap.add_argument("--output", default="-")
    ap.add_argument("--shapes", default=None,
                    help="comma-separated MxNxK list instead of the five frozen shapes")
    args = ap.parse_args(sys.argv[1:] if argv is None else argv)
    shapes = SHAPES
    if args.shapes:
        try:
            shapes = tuple(tuple(int(v) for v in item.split("x")) for item in args.shapes.split(","))
            if any(len(t) != 3 or min(t) < 1 for t in shapes):
                raise ValueError
        except ValueError:
            cm.eprint(f"multigpu: --shapes wants MxNxK[,MxNxK...] with positive extents, got {args.shapes!r}")
            return cm.EXIT_USAGE

    import torch
    import torch.distributed as dist

    from ..gemm import GemmPlan
    from ..inputs import baseline_mode_operands
    from ..sharding import gather_rows, row_shard

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", device_id=dev)
    rows_out = []
    try:
        for (m, n, k) in shapes:
            a_cpu, b_cpu = baseline_mode_operands(m, n, k)
            shards = [row_shard(m, world, r, granule=128) for r in range(world)]
            me = shards[rank]
            a = a_cpu[me.row0: me.row0 + me.rows].to(dev)
            b = b_cpu.to(dev)
            c = torch.empty(me.rows, n, dtype=torch.bfloat16, device=dev)
            stream = torch.cuda.Stream(device=dev)
            # A rank whose block is empty (fewer 128-row granules than ranks)
            # launches nothing but still joins every collective.
            plan = GemmPlan(a, b, c, variant=args.variant, stream=stream) if me.rows > 0 else None
            if plan:
                plan.run(args.warmup_iterations)
                plan.synchronize()
            if world > 1:
                dist.barrier()
            local_ms = 0.0
            if plan:
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record(stream)
                plan.run(args.iterations)
                e1.record(stream)
                e1.synchronize()
                local_ms = e0.elapsed_time(e1) / args.iterations
            ms = torch.tensor([local_ms], dtype=torch.float64, device=dev)
            if world > 1:
                dist.all_reduce(ms, op=dist.ReduceOp.MAX)
            ms = float(ms.item())
            full = gather_rows(c, shards) if world > 1 else c
            info = plan.info if plan else None
            if plan:
                plan.close()
            if rank == 0:
                torch.backends.cuda.matmul.allow_tf32 = False
                ref = torch.matmul(a_cpu.to(dev).float(), b.float().t())
                rel = float(torch.linalg.vector_norm(full.float() - ref) / torch.linalg.vector_norm(ref))
                tfl = 2.0 * m * n * k / (ms * 1e9)
                rows_out.append({
                    "shape_id": f"{m}x{n}x{k}x1", "n_gpus": world, "rows_per_rank_max": max(s.rows for s in shards),
                    "variant": args.variant, "tile_n": info["mma_tiler_n"], "kernel_time_ms_max": f"{ms:.6f}",
                    "tflops_aggregate": f"{tfl:.3f}", "tflops_per_gpu": f"{tfl / world:.3f}",
                    "rel_frobenius": f"{rel:.3e}", "correctness": "PASS" if rel <= 1e-2 else "FAIL",
                    "gpu_name": torch.cuda.get_device_name(dev), "git_commit": cm.git_commit_hash()})
                cm.eprint(f"multigpu: {m}x{n}x{k} P={world} {tfl:.1f} TFLOP/s aggregate rel={rel:.2e}")
            del a, b, c, full
    finally:
        if world > 1:
            dist.destroy_process_group()
    if rank == 0:
        out = sys.stdout if args.output == "-" else open(args.output, "w", newline="")
        w = csv.DictWriter(out, fieldnames=FIELDS, lineterminator="\n")
        w.writeheader()
        w.writerows(rows_out)
        if out is not sys.stdout:
            out.close()
        if any(r["correctness"] != "PASS" for r in rows_out):
            return cm.EXIT_FAILURE
    return cm.EXIT_OK


if __name__ == "__main__":
    raise SystemExit(main())
