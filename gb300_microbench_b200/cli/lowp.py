"""Block-scaled GEMM sweep (8192^3 and three more shapes): FP8 E4M3 with 128 x 128 FP32
block scales and NVFP4 (E2M1, UE4M3 per 16 K, FP32 per tensor), BF16 D, on
one GPU, with cuBLASLt's block-scaled GEMM on the same operands beside it.

    python -m gb300_microbench_b200.cli.lowp [--iterations N] [--warmup-iterations N] [--output FILE]

Operands are N(0,1) FP32 from torch.Generator seed 0, quantised on the GPU.
Each shape is timed two ways with CUDA events: L2 flushed (256 MiB write
outside the events) before every launch, and hot (N back-to-back launches).
D is checked against the FP32 product of the dequantised inputs on every
61st row (relative Frobenius <= 2e-2). One CSV row per (shape, kind).
"""
from __future__ import annotations

import argparse
import csv
import statistics
import sys

from . import common as cm

SHAPES = ((8192, 8192, 8192), (4096, 4096, 4096), (16384, 512, 4096), (512, 16384, 4096))
KINDS = ("nvfp4", "fp8_block128")
TOL = 2e-2
FIELDS = ("m", "n", "k", "kind", "cta_group", "tile_m", "tile_n", "grid_ctas", "ours_ms_flushed", "ours_tflops_flushed",
          "ours_tflops_hot", "cublaslt_tflops_flushed", "cublaslt_tflops_hot", "ratio_ours_vs_cublaslt",
          "cublaslt_note", "cublaslt_fp8_tensor_scaled_tflops_flushed", "rel_frobenius_sampled", "correctness",
          "gpu_name", "git_commit")


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="lowp")
    ap.add_argument("--iterations", type=int, default=20)
    ap.add_argument("--warmup-iterations", type=int, default=5)
    ap.add_argument("--output", default="-")
    args = ap.parse_args(sys.argv[1:] if argv is None else argv)
    if args.iterations < 1 or args.warmup_iterations < 0:
        cm.eprint("lowp: --iterations must be >= 1 and --warmup-iterations >= 0")
        return 2

    import torch

    from .. import lowp

    dev = torch.device("cuda", 0)
    stream = torch.cuda.Stream(device=dev)
    flush = torch.empty(64 << 20, dtype=torch.float32, device=dev)
    gpu = cm.query_gpu()
    commit = cm.git_commit_hash()

    def timed(fn):
        evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
               for _ in range(args.iterations)]
        for e0, e1 in evs:
            with torch.cuda.stream(stream):
                flush.zero_()
            e0.record(stream)
            fn()
            e1.record(stream)
        stream.synchronize()
        flushed = statistics.mean(e0.elapsed_time(e1) for e0, e1 in evs)
        e0, e1 = evs[0]
        e0.record(stream)
        for _ in range(args.iterations):
            fn()
        e1.record(stream)
        stream.synchronize()
        return flushed, e0.elapsed_time(e1) / args.iterations

    rows = []
    failed = False
    for m, n, k in SHAPES:
        x, y = lowp.config4_inputs(m, n, k, seed=0, device=dev)
        flops = 2.0 * m * n * k
        for kind in KINDS:
            op = lowp.Nvfp4Operand if kind == "nvfp4" else lowp.Fp8BlockOperand
            with torch.cuda.stream(stream):
                a, b = op(x), op(y)
            stream.synchronize()
            d = torch.empty(m, n, dtype=torch.bfloat16, device=dev)
            plan = lowp.LowpGemmPlan(kind, a, b, d, stream=stream)
            plan.run()
            plan.synchronize()
            rows_idx = torch.arange(0, m, 61, device=dev)
            with torch.cuda.stream(stream):
                ref = a.dequantize()[rows_idx].double() @ b.dequantize().double().T
                err = ((d[rows_idx].double() - ref).norm() / ref.norm()).item()
            del ref
            plan.run(args.warmup_iterations)
            ms, hot_ms = timed(plan.run)
            plan.synchronize()
            info = plan.info
            plan.close()
            cl_fl = cl_hot = ratio = ""
            note = "ok"
            d2 = torch.empty_like(d)
            try:
                cmp = lowp.CublasLtLowpPlan(kind, a, b, d2, stream=stream)
                cmp.run(args.warmup_iterations)
                cms, chot = timed(cmp.run)
                cmp.close()
                cl_fl, cl_hot = cm.fixed6(flops / cms / 1e9), cm.fixed6(flops / chot / 1e9)
                ratio = cm.fixed6(cms / ms)
            except Exception as exc:  # no cuBLASLt algorithm for this scaling mode
                note = str(exc).splitlines()[0][:160].replace(",", ";")
            fp8_ref = ""
            if kind == "fp8_block128":
                # cuBLASLt's plain FP8 GEMM on the same bytes (per-tensor scale,
                # no block scales): a throughput reference, not the same function.
                try:
                    cmp = lowp.CublasLtLowpPlan("fp8_tensor_scaled", a, b, d2, stream=stream)
                    cmp.run(args.warmup_iterations)
                    tms, _ = timed(cmp.run)
                    cmp.close()
                    fp8_ref = cm.fixed6(flops / tms / 1e9)
                except Exception:
                    fp8_ref = ""
            ok = err <= TOL
            failed |= not ok
            rows.append({
                "m": m, "n": n, "k": k, "kind": kind, "cta_group": info["cta_group"], "tile_m": info["tile_m"],
                "tile_n": info["tile_n"], "grid_ctas": info["grid_ctas"], "ours_ms_flushed": cm.fixed6(ms),
                "ours_tflops_flushed": cm.fixed6(flops / ms / 1e9), "ours_tflops_hot": cm.fixed6(flops / hot_ms / 1e9),
                "cublaslt_tflops_flushed": cl_fl, "cublaslt_tflops_hot": cl_hot, "ratio_ours_vs_cublaslt": ratio,
                "cublaslt_note": note, "cublaslt_fp8_tensor_scaled_tflops_flushed": fp8_ref,
                "rel_frobenius_sampled": f"{err:.6e}", "correctness": "pass" if ok else "fail",
                "gpu_name": gpu.name, "git_commit": commit})
            del a, b, d, d2
        del x, y

    out = sys.stdout if args.output == "-" else open(args.output, "w", newline="")
    w = csv.DictWriter(out, fieldnames=FIELDS, lineterminator="\n")
    w.writeheader()
    for r in rows:
        w.writerow(r)
    if out is not sys.stdout:
        out.close()
    return 1 if failed else 0


if __name__ == "__main__":
    raise SystemExit(main())
