"""GEMM comparison driver: the reference's ``gemm_comparison/gemm_comparison.py``
with the sm_100a GEMM of libb200bench.so in the three CuTe DSL candidate
slots and the cuBLASLt comparator (libb200cmp.so, the reference's frozen
row-major descriptor) in the fourth.

    python -m gb300_microbench_b200.cli.gemm_comparison [--warmup-iterations N] [--iterations N]
    python -m gb300_microbench_b200.cli.gemm_comparison --mode baseline [...]
    python -m gb300_microbench_b200.cli.gemm_comparison --self-test

Reference mode (default) keeps the reference's contract: the five frozen
shapes (gemm_comparison.py:116-122) x four frozen candidates (:209-260), one
operand set per shape drawn as the pinned factory draws it (seed 1111,
integer values), FP32 C, a NaN reset before every candidate, the
elementwise check |d| <= 0.1 + 1e-5 |ref| against an IEEE-FP32 matmul of the
upcast operands on the GPU (:2698-2755), warm-up then CUDA events around N
back-to-back launches (:3048-3067), and exactly 21 lines of the 100-column
CSV (:319-429) or nothing. The "cutedsl" method string names the candidate
slot; in this build the slot holds the sm_100a kernel configured like the
reference's candidate (tile, cluster, 2-CTA instructions, scheduler), and the
provenance columns carry this build's identities in the same formats.

Baseline mode (``--mode baseline``) measures the same shapes in the
baseline contract: N(0,1) operands from ``torch.Generator`` seed 0,
BF16 C, relative Frobenius error <= 1e-2, and adds the ``tuned`` candidate;
its CSV carries ``schema_version=b200.baseline.v1`` and five candidates per
shape.

Exit codes: 0 success, 1 contract / correctness / execution failure, 2 usage.
"""
from __future__ import annotations

import argparse
import csv
import hashlib
import io
import math
import subprocess
import sys
import time
from pathlib import Path

from . import common as cm

SCHEMA_VERSION = "p35.v1"
BASELINE_SCHEMA_VERSION = "b200.baseline.v1"
EXPERIMENT = "exp03_cutedsl_vs_cublaslt"
UNIT = "P3.5"
RUN_KIND = "smoke"
REFERENCE = "torch_cuda_fp32_ieee"
CACHE_MODE = "hot"
NOT_APPLICABLE = "not_applicable"

FROZEN_SHAPES = ((4096, 4096, 4096, 1), (8192, 8192, 8192, 1), (16384, 512, 4096, 1), (32768, 512, 4096, 1),
                 (512, 16384, 4096, 1))
FROZEN_SEED = 1111
FROZEN_ATOL = 1e-1
FROZEN_RTOL = 1e-5
BASELINE_TOL = 1e-2
REL_ERROR_DENOMINATOR_FLOOR = 1.0
WORKSPACE_LIMIT = 67108864
HEURISTIC_REQUESTED = 32

# (method, variant, scheduler, tile, cluster, 2-CTA, persistent); the slot
# configuration of gemm_comparison.py:209-260.
CANDIDATES = (
    ("cutedsl", "nonpersistent_1cta", "nonpersistent", (128, 128), (1, 1), False, False),
    ("cutedsl", "persistent_1cta", "static_persistent", (128, 128), (1, 1), False, True),
    ("cutedsl", "persistent_2cta", "static_persistent", (256, 128), (2, 1), True, True),
    ("cublaslt", "heuristic_first_supported", None, None, None, None, False),
)
TUNED = ("cutedsl", "tuned", "static_persistent", (256, 256), (2, 1), True, True)
CUBLASLT_INDEX = 3

CSV_FIELDS = (
    "schema_version", "experiment", "unit", "run_kind", "shape_index", "shape_id", "candidate_index", "method",
    "variant", "m", "n", "k", "l", "ab_dtype", "acc_dtype", "c_dtype", "a_major", "b_major", "c_major",
    "scheduler", "mma_tiler_m", "mma_tiler_n", "cluster_m", "cluster_n", "use_2cta_instrs", "use_tma_store",
    "max_active_clusters", "order_a", "order_b", "order_c", "order_d", "transa", "transb", "lda", "ldb", "ldc",
    "ldd", "compute_type", "scale_type", "pointer_mode", "epilogue", "alpha", "beta", "search_mode",
    "workspace_limit_bytes", "workspace_bytes", "alignment_a_bytes", "alignment_b_bytes", "alignment_c_bytes",
    "alignment_d_bytes", "heuristic_requested", "heuristic_returned", "heuristic_index", "algo_id", "tile_id",
    "stages_id", "split_k", "reduction_scheme", "cta_swizzling", "custom_option", "inner_shape_id",
    "cluster_shape_id", "waves_count", "cublaslt_version", "seed", "reference", "atol", "rtol", "correctness",
    "max_abs_error", "max_rel_error", "compile_time_ms", "setup_time_ms", "first_launch_ms", "kernel_time_ms",
    "warmup_iterations", "iterations", "cache_mode", "flop_count", "tflops", "throughput_ratio_vs_cublaslt",
    "gap_to_cublaslt_pct", "rank_within_shape", "best_cutedsl_variant", "is_best_cutedsl", "gpu_name",
    "gpu_uuid", "compute_capability", "driver_version", "cuda_toolkit_version", "torch_cuda_version",
    "cutedsl_version", "cutlass_commit", "operand_factory_sha256", "upstream_kernel_file",
    "upstream_kernel_git_blob", "upstream_kernel_sha256", "git_commit", "git_dirty", "publishable")
assert len(CSV_FIELDS) == 100

CUTEDSL_ONLY = ("scheduler", "mma_tiler_m", "mma_tiler_n", "cluster_m", "cluster_n", "use_2cta_instrs",
                "use_tma_store", "max_active_clusters", "compile_time_ms", "upstream_kernel_file",
                "upstream_kernel_git_blob", "upstream_kernel_sha256")
CUBLASLT_ONLY = ("order_a", "order_b", "order_c", "order_d", "transa", "transb", "lda", "ldb", "ldc", "ldd",
                 "compute_type", "scale_type", "pointer_mode", "epilogue", "alpha", "beta", "search_mode",
                 "workspace_limit_bytes", "workspace_bytes", "alignment_a_bytes", "alignment_b_bytes",
                 "alignment_c_bytes", "alignment_d_bytes", "heuristic_requested", "heuristic_returned",
                 "heuristic_index", "algo_id", "tile_id", "stages_id", "split_k", "reduction_scheme",
                 "cta_swizzling", "custom_option", "inner_shape_id", "cluster_shape_id", "waves_count",
                 "cublaslt_version", "setup_time_ms")

# cuBLASLt enum names of the reference descriptor (cublaslt_bridge.cu:75-128).
ENUM_NAMES = {
    "order": {1: "CUBLASLT_ORDER_ROW", 0: "CUBLASLT_ORDER_COL"},
    "trans": {0: "CUBLAS_OP_N", 1: "CUBLAS_OP_T"},
    "compute_type": {68: "CUBLAS_COMPUTE_32F"},
    "scale_type": {0: "CUDA_R_32F"},
    "pointer_mode": {0: "CUBLASLT_POINTER_MODE_HOST"},
    "epilogue": {1: "CUBLASLT_EPILOGUE_DEFAULT"},
    "search_mode": {0: "CUBLASLT_SEARCH_BEST_FIT"},
}

KERNEL_SOURCE = Path(__file__).resolve().parents[1] / "gemm.py"
FACTORY_SOURCE = Path(__file__).resolve().parents[1] / "inputs.py"


class ContractError(Exception):
    pass


def shape_id(mnkl) -> str:
    return "x".join(str(v) for v in mnkl)


def fixed(v: float, d: int) -> str:
    if not math.isfinite(v) or v < 0:
        raise ContractError(f"{v!r} is not a finite non-negative number")
    return f"{v:.{d}f}"


def signed_fixed(v: float, d: int) -> str:
    if not math.isfinite(v):
        raise ContractError(f"{v!r} is not finite")
    text = f"{v:.{d}f}"
    if text.startswith("-") and float(text) == 0.0:
        text = text[1:]
    return text


def compute_flop_count(mnkl) -> int:
    """2*M*N*K (gemm_comparison.py:1619-1634)."""
    m, n, k, l = mnkl
    return 2 * m * n * k * l


def compute_tflops(flops: int, ms: float) -> float:
    """flop / (ms * 1e9) (gemm_comparison.py:1637-1655)."""
    if not (math.isfinite(ms) and ms > 0):
        raise ContractError(f"kernel_time_ms={ms!r} must be finite and positive")
    return flops / (ms * 1e9)


def compute_shape_comparison(mnkl, times_ms: list[float], cublaslt_index: int, cutedsl_indices, order):
    """Ratio, gap, rank and best variant (gemm_comparison.py:1658-1756):
    ratio = tflops / cublaslt_tflops, gap = 100 (1 - ratio), ranks by time
    with ties broken by candidate order, the best CuTe-slot variant by the
    same rule; the cuBLASLt row carries exactly 1 and 0."""
    flops = compute_flop_count(mnkl)
    tflops = [compute_tflops(flops, t) for t in times_ms]
    base = tflops[cublaslt_index]
    ranked = sorted(range(len(times_ms)), key=lambda i: (times_ms[i], i))
    rank = {i: pos + 1 for pos, i in enumerate(ranked)}
    best = min(cutedsl_indices, key=lambda i: (times_ms[i], i))
    out = []
    for i, t in enumerate(tflops):
        ratio = 1.0 if i == cublaslt_index else t / base
        gap = 0.0 if i == cublaslt_index else 100.0 * (1.0 - ratio)
        out.append({"flop_count": flops, "tflops": t, "throughput_ratio_vs_cublaslt": ratio,
                    "gap_to_cublaslt_pct": gap, "rank_within_shape": rank[i], "best_cutedsl_variant": order[best],
                    "is_best_cutedsl": i == best})
    return out


def git_blob(path: Path) -> str:
    data = path.read_bytes()
    return hashlib.sha1(b"blob %d\0" % len(data) + data).hexdigest()


def sha256(path: Path) -> str:
    return hashlib.sha256(path.read_bytes()).hexdigest()


def provenance(gpu: cm.GpuInfo) -> dict:
    import torch

    from .. import __version__

    commit = cm.git_commit_hash()
    if len(commit) != 40:
        commit = "0" * 40
    drv = "0"
    try:
        out = subprocess.run(["nvidia-smi", "--query-gpu=driver_version", "--format=csv,noheader", "-i", "0"],
                             capture_output=True, text=True, timeout=30)
        if out.returncode == 0 and out.stdout.strip():
            drv = out.stdout.strip().splitlines()[0]
    except (OSError, subprocess.TimeoutExpired):
        pass
    toolkit = "12.9"
    try:
        out = subprocess.run(["nvcc", "--version"], capture_output=True, text=True, timeout=30)
        for tok in out.stdout.replace(",", " ").split():
            if tok.startswith("V") and tok[1:2].isdigit():
                toolkit = ".".join(tok[1:].split(".")[:2])
    except (OSError, subprocess.TimeoutExpired):
        pass
    return {
        "gpu_name": gpu.name, "gpu_uuid": gpu.uuid, "compute_capability": gpu.compute_capability,
        "driver_version": drv, "cuda_toolkit_version": toolkit, "torch_cuda_version": torch.version.cuda or "0",
        "cutedsl_version": __version__, "cutlass_commit": commit,
        "operand_factory_sha256": sha256(FACTORY_SOURCE),
        "git_commit": commit, "git_dirty": cm.git_dirty_flag(),
    }


def make_operands(mode: str, mnkl):
    import torch

    from .. import inputs

    m, n, k, l = mnkl
    if mode == "reference":
        a, b = inputs.reference_mode_operands(m, n, k, l)
        return a[0].cuda(), b[0].cuda()
    a, b = inputs.baseline_mode_operands(m, n, k)
    return a.cuda(), b.cuda()


def reference_result(a, b):
    """IEEE FP32 matmul of the upcast operands on the GPU (the reference's
    oracle, gemm_comparison.py:2698-2715; TF32 off)."""
    import torch

    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        ref = torch.matmul(a.float(), b.float().t())
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev
    torch.cuda.synchronize()
    if not bool(torch.isfinite(ref).all()):
        raise ContractError("the FP32 reference contains non-finite values")
    return ref


def validate(mode: str, label: str, ref, c) -> tuple[float, float]:
    import torch

    res = c.float()
    if not bool(torch.isfinite(res).all()):
        raise ContractError(f"{label}: non-finite values (the output was reset to NaN before this candidate)")
    diff = (res - ref).abs()
    max_abs = float(diff.max())
    max_rel = float((diff / ref.abs().clamp_min(REL_ERROR_DENOMINATOR_FLOOR)).max())
    if mode == "reference":
        bad = int((diff > FROZEN_ATOL + FROZEN_RTOL * ref.abs()).sum())
        if bad:
            raise ContractError(f"{label}: {bad} element(s) exceed atol={FROZEN_ATOL} rtol={FROZEN_RTOL}")
    else:
        rel = float(torch.linalg.vector_norm(res - ref) / torch.linalg.vector_norm(ref))
        if rel > BASELINE_TOL:
            raise ContractError(f"{label}: relative Frobenius error {rel:.3e} > {BASELINE_TOL}")
    return max_abs, max_rel


def steady_state(run, stream, warmup: int, iterations: int) -> float:
    """Warm-up, then CUDA events around `iterations` back-to-back launches on
    one stream (gemm_comparison.py:3048-3067)."""
    import torch

    for _ in range(warmup):
        run()
    stream.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(iterations):
        run()
    e1.record(stream)
    e1.synchronize()
    return e0.elapsed_time(e1) / iterations


def first_launch(run, stream) -> float:
    import torch

    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    run()
    e1.record(stream)
    e1.synchronize()
    return e0.elapsed_time(e1)


def measure_shape(mode: str, mnkl, candidates, warmup: int, iterations: int) -> list[dict]:
    import torch

    from ..gemm import CublasLtPlan, GemmPlan

    m, n, k, l = mnkl
    a, b = make_operands(mode, mnkl)
    ref = reference_result(a, b)
    c_dtype = torch.float32 if mode == "reference" else torch.bfloat16
    c = torch.empty(m, n, dtype=c_dtype, device="cuda")
    stream = torch.cuda.Stream()
    results = []
    for spec in candidates:
        method, variant = spec[0], spec[1]
        c.fill_(float("nan"))
        torch.cuda.synchronize()
        label = f"{shape_id(mnkl)}/{variant}"
        if method == "cutedsl":
            t0 = time.perf_counter()
            plan = GemmPlan(a, b, c, variant=variant, stream=stream)
            setup_ms = (time.perf_counter() - t0) * 1000.0
            first_ms = first_launch(plan.run, stream)
            plan.synchronize()
            max_abs, max_rel = validate(mode, label, ref, c)
            ms = steady_state(plan.run, stream, warmup, iterations)
            plan.synchronize()
            info = plan.info
            plan.close()
            results.append({"spec": spec, "compile_ms": setup_ms, "setup_ms": None, "first_ms": first_ms, "ms": ms,
                            "max_abs": max_abs, "max_rel": max_rel, "info": info, "cmp": None})
        else:
            t0 = time.perf_counter()
            cmp = CublasLtPlan(a, b, c, stream=stream, layout="reference")
            setup_ms = (time.perf_counter() - t0) * 1000.0
            first_ms = first_launch(cmp.run, stream)
            max_abs, max_rel = validate(mode, label, ref, c)
            ms = steady_state(cmp.run, stream, warmup, iterations)
            results.append({"spec": spec, "compile_ms": None, "setup_ms": setup_ms, "first_ms": first_ms, "ms": ms,
                            "max_abs": max_abs, "max_rel": max_rel, "info": None, "cmp": cmp.info})
            cmp.close()
        cm.eprint(f"gemm_comparison: {label} {compute_tflops(compute_flop_count(mnkl), results[-1]['ms']):.1f} "
                  f"TFLOP/s max_abs_error={results[-1]['max_abs']:.3g}")
    return results


def cublaslt_fields(info: dict) -> dict:
    def name(kind, v):
        return ENUM_NAMES[kind].get(int(v), str(int(v)))

    return {
        "order_a": name("order", info["order_a"]), "order_b": name("order", info["order_b"]),
        "order_c": name("order", info["order_c"]), "order_d": name("order", info["order_d"]),
        "transa": name("trans", info["transa"]), "transb": name("trans", info["transb"]),
        "lda": str(info["lda"]), "ldb": str(info["ldb"]), "ldc": str(info["ldc"]), "ldd": str(info["ldd"]),
        "compute_type": name("compute_type", info["compute_type"]),
        "scale_type": name("scale_type", info["scale_type"]),
        "pointer_mode": name("pointer_mode", info["pointer_mode"]), "epilogue": name("epilogue", info["epilogue"]),
        "alpha": fixed(info["alpha"], 9), "beta": fixed(info["beta"], 9),
        "search_mode": name("search_mode", info["search_mode"]),
        "workspace_limit_bytes": str(info["workspace_limit_bytes"]), "workspace_bytes": str(info["workspace_bytes"]),
        "alignment_a_bytes": str(info["alignment_a_bytes"]), "alignment_b_bytes": str(info["alignment_b_bytes"]),
        "alignment_c_bytes": str(info["alignment_c_bytes"]), "alignment_d_bytes": str(info["alignment_d_bytes"]),
        "heuristic_requested": str(info["heuristic_requested"]), "heuristic_returned": str(info["heuristic_returned"]),
        "heuristic_index": str(info["heuristic_index"]), "algo_id": str(max(0, info["algo_id"])),
        "tile_id": str(max(0, info["tile_id"])), "stages_id": str(max(0, info["stages_id"])),
        "split_k": str(max(0, info["split_k"])), "reduction_scheme": str(max(0, info["reduction_scheme"])),
        "cta_swizzling": str(max(0, info["cta_swizzling"])), "custom_option": str(max(0, info["custom_option"])),
        "inner_shape_id": str(max(0, info["inner_shape_id"])),
        "cluster_shape_id": str(max(0, info["cluster_shape_id"])), "waves_count": fixed(info["waves_count"], 6),
        "cublaslt_version": str(info["cublaslt_version"]),
    }


def build_rows(mode: str, shape_index: int, mnkl, results, comparison, prov, warmup, iterations) -> list[dict]:
    rows = []
    m, n, k, l = mnkl
    for ci, (res, cmpf) in enumerate(zip(results, comparison)):
        method, variant, scheduler, tile, cluster, two_cta, persistent = res["spec"]
        if variant == "tuned" and "info" in res:
            # The tuned slot's tile is chosen per shape by the plan (256 x 256
            # or 256 x 512 CTA-pair tiles); record the one it chose.
            tile = (int(res["info"]["mma_tiler_m"]), int(res["info"]["mma_tiler_n"]))
        row = {f: NOT_APPLICABLE for f in (CUBLASLT_ONLY if method == "cutedsl" else CUTEDSL_ONLY)}
        row.update({
            "schema_version": SCHEMA_VERSION if mode == "reference" else BASELINE_SCHEMA_VERSION,
            "experiment": EXPERIMENT, "unit": UNIT, "run_kind": RUN_KIND, "shape_index": str(shape_index + 1),
            "shape_id": shape_id(mnkl), "candidate_index": str(ci + 1), "method": method, "variant": variant,
            "m": str(m), "n": str(n), "k": str(k), "l": str(l), "ab_dtype": "BFloat16", "acc_dtype": "Float32",
            "c_dtype": "Float32" if mode == "reference" else "BFloat16", "a_major": "k", "b_major": "k",
            "c_major": "n", "seed": str(FROZEN_SEED if mode == "reference" else 0), "reference": REFERENCE,
            # Baseline mode: both columns carry the relative Frobenius bound.
            "atol": fixed(FROZEN_ATOL if mode == "reference" else BASELINE_TOL, 9),
            "rtol": fixed(FROZEN_RTOL if mode == "reference" else BASELINE_TOL, 9),
            "correctness": "PASS", "max_abs_error": fixed(res["max_abs"], 9), "max_rel_error": fixed(res["max_rel"], 9),
            "first_launch_ms": fixed(res["first_ms"], 6), "kernel_time_ms": fixed(res["ms"], 6),
            "warmup_iterations": str(warmup), "iterations": str(iterations), "cache_mode": CACHE_MODE,
            "flop_count": str(cmpf["flop_count"]), "tflops": fixed(cmpf["tflops"], 6),
            "throughput_ratio_vs_cublaslt": fixed(cmpf["throughput_ratio_vs_cublaslt"], 9),
            "gap_to_cublaslt_pct": signed_fixed(cmpf["gap_to_cublaslt_pct"], 6),
            "rank_within_shape": str(cmpf["rank_within_shape"]), "best_cutedsl_variant": cmpf["best_cutedsl_variant"],
            "is_best_cutedsl": "true" if cmpf["is_best_cutedsl"] else "false", "publishable": "false",
        })
        row.update(prov)
        if method == "cutedsl":
            row.update({
                "scheduler": scheduler, "mma_tiler_m": str(tile[0]), "mma_tiler_n": str(tile[1]),
                "cluster_m": str(cluster[0]), "cluster_n": str(cluster[1]),
                "use_2cta_instrs": "true" if two_cta else "false", "use_tma_store": "true",
                "max_active_clusters": str(res["info"]["max_active_clusters"]) if persistent else NOT_APPLICABLE,
                "compile_time_ms": fixed(res["compile_ms"], 6),
                "upstream_kernel_file": "gb300_microbench_b200/gemm.py",
                "upstream_kernel_git_blob": git_blob(KERNEL_SOURCE), "upstream_kernel_sha256": sha256(KERNEL_SOURCE),
            })
            info = res["info"]
            if (info["mma_tiler_m"], info["mma_tiler_n"], info["cluster_m"]) != (tile[0], tile[1], cluster[0]):
                raise ContractError(f"{variant}: the plan ({info['mma_tiler_m']}x{info['mma_tiler_n']}, cluster "
                                    f"{info['cluster_m']}) does not match the slot's configuration")
        else:
            row.update(cublaslt_fields(res["cmp"]))
            row["setup_time_ms"] = fixed(res["setup_ms"], 6)
        if set(row) != set(CSV_FIELDS):
            raise ContractError(f"row fields differ from the schema: {sorted(set(row) ^ set(CSV_FIELDS))}")
        rows.append(row)
    return rows


def serialize(rows) -> str:
    buf = io.StringIO()
    w = csv.DictWriter(buf, fieldnames=list(CSV_FIELDS), extrasaction="raise", lineterminator="\n",
                       quoting=csv.QUOTE_MINIMAL)
    w.writeheader()
    for r in rows:
        w.writerow(r)
    return buf.getvalue()


def self_test() -> int:
    """GPU-free checks of the comparison arithmetic and the serializer."""
    checks = 0
    times = [2.0, 1.0, 1.0, 0.5]
    order = [c[1] for c in CANDIDATES]
    comp = compute_shape_comparison((4096, 4096, 4096, 1), times, CUBLASLT_INDEX, (0, 1, 2), order)
    assert comp[3]["throughput_ratio_vs_cublaslt"] == 1.0 and comp[3]["gap_to_cublaslt_pct"] == 0.0
    checks += 1
    assert [c["rank_within_shape"] for c in comp] == [4, 2, 3, 1]  # tie broken by candidate order
    checks += 1
    assert comp[1]["is_best_cutedsl"] and comp[0]["best_cutedsl_variant"] == "persistent_1cta"
    checks += 1
    assert abs(comp[0]["gap_to_cublaslt_pct"] - 75.0) < 1e-9
    checks += 1
    assert compute_flop_count((4096, 4096, 4096, 1)) == 2 * 4096 ** 3
    checks += 1
    assert signed_fixed(-0.0000001, 6) == "0.000000" and signed_fixed(-12.5, 6) == "-12.500000"
    checks += 1
    try:
        compute_tflops(1, 0.0)
        raise AssertionError("zero time accepted")
    except ContractError:
        checks += 1
    print(f"SELF_TEST: PASS ({checks} checks)")
    return cm.EXIT_OK


def parse_args(argv):
    ap = argparse.ArgumentParser(prog="gemm_comparison", description="sm_100a GEMM candidates vs cuBLASLt")
    ap.add_argument("--warmup-iterations", type=int, default=5)
    ap.add_argument("--iterations", type=int, default=20)
    ap.add_argument("--mode", choices=("reference", "baseline"), default="reference")
    ap.add_argument("--self-test", action="store_true")
    args = ap.parse_args(argv)
    if not 1 <= args.warmup_iterations <= 100 or not 1 <= args.iterations <= 100:
        ap.error("--warmup-iterations and --iterations must be in [1, 100]")
    return args


def main(argv=None) -> int:
    try:
        args = parse_args(sys.argv[1:] if argv is None else argv)
    except SystemExit as exc:
        return cm.EXIT_USAGE if exc.code else cm.EXIT_OK
    if args.self_test:
        return self_test()
    try:
        gpu = cm.query_gpu()
        prov = provenance(gpu)
        candidates = CANDIDATES if args.mode == "reference" else CANDIDATES + (TUNED,)
        cutedsl_idx = tuple(i for i, c in enumerate(candidates) if c[0] == "cutedsl")
        order = [c[1] for c in candidates]
        rows = []
        for si, mnkl in enumerate(FROZEN_SHAPES):
            results = measure_shape(args.mode, mnkl, candidates, args.warmup_iterations, args.iterations)
            comp = compute_shape_comparison(mnkl, [r["ms"] for r in results], CUBLASLT_INDEX, cutedsl_idx, order)
            rows += build_rows(args.mode, si, mnkl, results, comp, prov, args.warmup_iterations, args.iterations)
        expected = len(FROZEN_SHAPES) * len(candidates)
        if len(rows) != expected:
            raise ContractError(f"expected {expected} rows, got {len(rows)}")
        sys.stdout.write(serialize(rows))
        sys.stdout.flush()
        return cm.EXIT_OK
    except (ContractError, cm.RunFailure) as exc:
        cm.eprint(f"gemm_comparison: ERROR: {exc}; no CSV was emitted")
        return cm.EXIT_FAILURE
    except Exception as exc:
        cm.eprint(f"gemm_comparison: ERROR: {type(exc).__name__}: {exc}; no CSV was emitted")
        return cm.EXIT_FAILURE


if __name__ == "__main__":
    raise SystemExit(main())
