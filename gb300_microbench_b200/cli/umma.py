"""tcgen05 UMMA throughput CLI: the reference's ``umma_throughput/umma_1sm``
and ``umma_2sm`` binaries (umma_1sm.cu:700-1189, umma_2sm.cu), running the
sm_100a probes of libb200bench.so.

    python -m gb300_microbench_b200.cli.umma {umma_1sm,umma_2sm} --self-test
    python -m gb300_microbench_b200.cli.umma {umma_1sm,umma_2sm} --run-kind {smoke,benchmark}
        --n {64,128,256} --depth {4,16,32,64,128,256} --iterations N --warmup-iterations N
        --repetitions N [--operands {pattern,random}] [--seed N] [--handshake {cluster,none}]

Flags, exit codes and the 37-column CSV are the reference's
(umma_1sm.cu:965-995); depths 32 and 128 (the baseline-mode grid) and N(0,1)
operands (``--operands random``, checked against an FP32 host
restatement of depth * A * B^T within 1e-5 relative Frobenius error) are
additions. Pattern operands are checked for exact equality, every
repetition, as the reference does. ``umma_2sm`` runs the reference's loop:
a per-iteration handshake of both CTAs (each waits on its own mbarrier,
then a cluster barrier) inside the timed region (umma_2sm.cu:617-659);
``--handshake none`` (an addition) times only the issuing CTA's waits.
"""
from __future__ import annotations

import sys

from . import common as cm

METHODS = {"umma_1sm": 1, "umma_2sm": 2}
N_VALUES = (64, 128, 256)
DEPTHS = (4, 16, 32, 64, 128, 256)
REFERENCE_DEPTHS = (4, 16, 64, 256)
K = 16

CSV_HEADER = (
    "schema_version,timestamp_utc,run_kind,publishable,method,sample_index,cta_group,m,n,k,"
    "depth,iterations,warmup_iterations,repetitions,umma_per_iteration,total_umma,"
    "flops_per_umma,total_flops,elapsed_cycles,cycles_per_umma,flops_per_cycle,threads_per_cta,"
    "grid_blocks,tmem_columns,operand_path,input_type,accumulator_type,correctness,mismatches,"
    "max_abs_error,gpu_name,gpu_uuid,compute_capability,cuda_driver_version,"
    "cuda_runtime_version,git_commit,git_dirty")

SELF_TEST_ITERATIONS = 2  # umma_1sm.cu:1085


def usage(method: str) -> str:
    return f"""{method} - BF16 UMMA (tcgen05.mma kind::f16, cta_group::{METHODS[method]}) issue microbenchmark on B200

Usage:
  {method} --help
  {method} --self-test
  {method} --run-kind {{smoke,benchmark}} --n {{64,128,256}} --depth {{4,16,32,64,128,256}} \\
           --iterations N --warmup-iterations N --repetitions N [--operands {{pattern,random}}] [--seed N]
           [--handshake {{cluster,none}}]   (umma_2sm: per-iteration CTA-pair handshake, default cluster)
"""


def parse(argv: list[str]) -> dict:
    cfg = {"help": False, "self_test": False, "operands": "pattern", "seed": 0, "handshake": "cluster"}
    seen = set()
    i = 0
    while i < len(argv):
        a = argv[i]
        if a in ("--help", "--self-test"):
            key = "help" if a == "--help" else "self_test"
            if cfg[key]:
                raise cm.UsageError(f"{a} specified more than once")
            cfg[key] = True
            i += 1
            continue
        if a in seen:
            raise cm.UsageError(f"{a} specified more than once")
        seen.add(a)
        if a == "--run-kind":
            v, i = cm.take_value(argv, i, a)
            if v not in ("smoke", "benchmark"):
                raise cm.UsageError("--run-kind must be 'smoke' or 'benchmark'")
            cfg["run_kind"] = v
        elif a == "--n":
            v, i = cm.take_value(argv, i, a)
            if v not in ("64", "128", "256"):
                raise cm.UsageError("--n must be one of 64, 128, 256")
            cfg["n"] = int(v)
        elif a == "--depth":
            v, i = cm.take_value(argv, i, a)
            if v not in tuple(str(d) for d in DEPTHS):
                raise cm.UsageError("--depth must be one of 4, 16, 32, 64, 128, 256")
            cfg["depth"] = int(v)
        elif a == "--iterations":
            v, i = cm.take_value(argv, i, a)
            cfg["iterations"] = cm.parse_int(v, 1, 1 << 40, a)
        elif a == "--warmup-iterations":
            v, i = cm.take_value(argv, i, a)
            cfg["warmup_iterations"] = cm.parse_int(v, 0, 1 << 40, a)
        elif a == "--repetitions":
            v, i = cm.take_value(argv, i, a)
            cfg["repetitions"] = cm.parse_int(v, 1, 1 << 40, a)
        elif a == "--operands":
            v, i = cm.take_value(argv, i, a)
            if v not in ("pattern", "random"):
                raise cm.UsageError("--operands must be 'pattern' or 'random'")
            cfg["operands"] = v
        elif a == "--seed":
            v, i = cm.take_value(argv, i, a)
            cfg["seed"] = cm.parse_int(v, 0, (1 << 63) - 1, a)
        elif a == "--handshake":
            v, i = cm.take_value(argv, i, a)
            if v not in ("cluster", "none"):
                raise cm.UsageError("--handshake must be 'cluster' or 'none'")
            cfg["handshake"] = v
        else:
            raise cm.UsageError(f"unknown argument: {a}")
    if cfg["help"]:
        return cfg
    if cfg["self_test"]:
        if seen:
            raise cm.UsageError("--self-test cannot be combined with other options")
        return cfg
    for key in ("run_kind", "n", "depth", "iterations", "warmup_iterations", "repetitions"):
        if key not in cfg:
            raise cm.UsageError(f"--{key.replace('_', '-')} is required")
    return cfg


def expected_d(a, b, depth: int):
    """depth * A @ B^T in float64 on the host (A: M x 16, B: N x 16 BF16)."""
    import torch

    return depth * (a.to(torch.float64) @ b.to(torch.float64).t())


def check_d(d, want, operands: str) -> tuple[bool, int, float]:
    import torch

    d64 = d.to(torch.float64)
    diff = (d64 - want).abs()
    max_abs = float(diff.max())
    if operands == "pattern":
        mism = int((d64 != want).sum())
        return mism == 0, mism, max_abs
    rel = float(torch.linalg.vector_norm(d64 - want) / torch.linalg.vector_norm(want))
    return rel <= 1e-5, 0 if rel <= 1e-5 else int((diff > 1e-3 * want.abs().max()).sum()), max_abs


def operands_for(cg: int, n: int, operands: str, seed: int):
    from .. import inputs

    if operands == "pattern":
        return inputs.umma_pattern_operands(cg, n)
    return inputs.umma_random_operands(cg, n, seed=seed)


def format_row(method, cfg, sample, cycles, max_abs, gpu, commit, dirty) -> str:
    cg = METHODS[method]
    m = 128 * cg
    flops_per_umma = 2 * m * cfg["n"] * K
    total_umma = cfg["depth"] * cfg["iterations"]
    total_flops = flops_per_umma * total_umma
    fields = [
        "1", cm.now_utc_iso8601(), cfg["run_kind"], "false", method, str(sample), str(cg), str(m), str(cfg["n"]),
        str(K), str(cfg["depth"]), str(cfg["iterations"]), str(cfg["warmup_iterations"]), str(cfg["repetitions"]),
        str(cfg["depth"]), str(total_umma), str(flops_per_umma), str(total_flops), str(cycles),
        cm.fixed6(cycles / total_umma if total_umma else 0.0), cm.fixed6(total_flops / cycles if cycles else 0.0),
        "128", str(cg), str(cfg["n"]), "smem_smem", "bf16", "fp32", "OK", "0", cm.fixed6(max_abs) if max_abs else "0",
        cm.csv_quote(gpu.name), gpu.uuid, gpu.compute_capability, str(gpu.driver_version), str(gpu.runtime_version),
        commit, dirty,
    ]
    return ",".join(fields)


def run_config(method: str, cfg: dict, gpu: cm.GpuInfo, print_header: bool = True, out=None) -> int:
    import torch

    out = out if out is not None else sys.stdout  # resolved per call (callers may redirect stdout)

    from .. import umma

    cg = METHODS[method]
    a, b = operands_for(cg, cfg["n"], cfg["operands"], cfg["seed"])
    want = expected_d(a, b, cfg["depth"])
    probe = umma.UmmaProbe(cg, cfg["n"], cfg["depth"], a.cuda(), b.cuda(),
                           handshake=cg == 2 and cfg.get("handshake", "cluster") == "cluster")

    def once(timed: bool):
        probe.launch(cfg["iterations"], timed=timed)
        d, cycles = probe.result()
        ok, mism, max_abs = check_d(d, want, cfg["operands"])
        if not ok:
            raise cm.RunFailure(f"correctness validation FAILED for {probe.name}: mismatches={mism} "
                                f"max_abs_error={max_abs:.6g}; no timing or CSV output was produced")
        return cycles, max_abs

    once(False)
    cm.eprint(f"{method}: correctness=OK (pre-timing check)")
    for _ in range(cfg["warmup_iterations"]):
        once(False)
    commit, dirty = cm.git_commit_hash(), cm.git_dirty_flag()
    if print_header:
        print(CSV_HEADER, file=out)
    for rep in range(cfg["repetitions"]):
        cycles, max_abs = once(True)
        if cycles <= 0:
            raise cm.RunFailure(f"elapsed_cycles was not greater than zero for {probe.name}")
        print(format_row(method, cfg, rep, cycles, max_abs, gpu, commit, dirty), file=out, flush=True)
    del torch
    return cm.EXIT_OK


def self_test(method: str) -> int:
    from .. import umma

    cg = METHODS[method]
    passed = total = 0
    for n in N_VALUES:
        for depth in DEPTHS:
            a, b = operands_for(cg, n, "pattern", 0)
            probe = umma.UmmaProbe(cg, n, depth, a.cuda(), b.cuda(), handshake=cg == 2)
            probe.launch(SELF_TEST_ITERATIONS, timed=False)
            d, _ = probe.result()
            ok, mism, max_abs = check_d(d, expected_d(a, b, depth), "pattern")
            total += 1
            passed += 1 if ok else 0
            cm.eprint(f"{method}: SELF_TEST {probe.name} n={n} depth={depth} result={'PASS' if ok else 'FAIL'} "
                      f"mismatches={mism} max_abs_error={max_abs:.6g}")
    cm.eprint(f"{method}: SELF_TEST_RESULT {passed}/{total}")
    if passed == total:
        print(f"SELF_TEST: PASS ({passed}/{total})")
        return cm.EXIT_OK
    return cm.EXIT_FAILURE


def main(argv: list[str] | None = None) -> int:
    argv = list(sys.argv[1:] if argv is None else argv)
    if not argv or argv[0] not in METHODS:
        cm.eprint("usage: python -m gb300_microbench_b200.cli.umma {umma_1sm,umma_2sm} ...")
        return cm.EXIT_USAGE
    method, rest = argv[0], argv[1:]
    try:
        cfg = parse(rest)
    except cm.UsageError as exc:
        cm.eprint(f"{method}: ERROR: {exc}")
        cm.eprint(usage(method))
        return cm.EXIT_USAGE
    if cfg["help"]:
        print(usage(method))
        return cm.EXIT_OK
    try:
        gpu = cm.query_gpu()
        cm.expected_uuid(gpu)
        if cfg["self_test"]:
            return self_test(method)
        return run_config(method, cfg, gpu)
    except cm.RunFailure as exc:
        cm.eprint(f"{method}: ERROR: {exc}")
        return cm.EXIT_FAILURE
    except Exception as exc:
        cm.eprint(f"{method}: ERROR: {type(exc).__name__}: {exc}")
        return cm.EXIT_FAILURE


if __name__ == "__main__":
    raise SystemExit(main())
