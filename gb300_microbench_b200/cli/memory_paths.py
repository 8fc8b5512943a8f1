"""HBM->SMEM streaming benchmark CLI: the reference's ``memory_paths/ldgsts``
and ``memory_paths/tma`` binaries (ldgsts.cu:540-1088, tma.cu:1000-1427),
running the sm_100a kernels of libb200bench.so.

    python -m gb300_microbench_b200.cli.memory_paths {ldgsts,tma} --self-test
    python -m gb300_microbench_b200.cli.memory_paths {ldgsts,tma} \\
        --stages {2,3,4,8} --bytes-in-flight-kib {16,32,64} --run-kind {smoke,benchmark}
        [--working-set-mib N] [--passes N] [--warmup-ms N] [--repetitions N]
        [--fill {pattern,uniform}] [--seed N] [--row-bytes {128,256}]

The reference's flags keep their meaning, ranges, defaults and the
37-column CSV (ldgsts.cu:734-768). Additions for the streaming grid of the
B200 build: stage count 3 (stage bytes rounded down to the copy
granularity), ``--fill uniform`` (seeded uniform 32-bit words instead of the
SplitMix64 pattern; validated by comparing the checksum of checksums of the
LDGSTS and TMA data paths) and ``--row-bytes`` (the TMA box row width).
"""
from __future__ import annotations

import sys
import time

from . import common as cm

METHODS = ("ldgsts", "tma")
STAGES = (2, 3, 4, 8)
BIF_KIB = (16, 32, 64)
REFERENCE_STAGES = (2, 4, 8)

CSV_HEADER = (
    "schema_version,timestamp_utc,run_kind,method,sample_index,stages,"
    "tile_width_elements,tile_width_bytes,tile_height,stage_bytes,"
    "bytes_in_flight_per_sm,vector_bytes,copies_per_thread_per_stage,"
    "threads_per_cta,target_ctas_per_sm,occupancy_ctas_per_sm,grid_blocks,"
    "sm_count,smem_reservation_bytes,l2_bytes,requested_working_set_bytes,"
    "working_set_bytes,working_set_l2_ratio,passes,useful_bytes,warmup_ms,"
    "kernel_time_ms,effective_gbps,correctness,mismatches,gpu_name,gpu_uuid,"
    "compute_capability,cuda_driver_version,cuda_runtime_version,git_commit,"
    "git_dirty")

SELF_TEST_COMMON_MULTIPLES = 8  # ldgsts.cu:69


def usage(method: str) -> str:
    return f"""{method} - HBM->SMEM streaming read microbenchmark on B200 (sm_100a)

Usage:
  {method} --self-test
  {method} --stages {{2,3,4,8}} --bytes-in-flight-kib {{16,32,64}} --run-kind {{smoke,benchmark}}
         [--working-set-mib N] [--passes N] [--warmup-ms N] [--repetitions N]
         [--fill {{pattern,uniform}}] [--seed N] [--row-bytes {{128,256}}]

Options:
  --stages {{2,3,4,8}}               Ring depth. Required.
  --bytes-in-flight-kib {{16,32,64}} Bytes in flight per SM. Required.
  --working-set-mib N              Requested working set in MiB, in [1, 1048576], rounded up
                                   to a multiple of sm_count*32KiB. Default: 4x L2.
  --passes N                       Traversals per timed launch, in [1, 1000000]. Default 1.
  --warmup-ms N                    Warm-up time before the timed launches. Default 0.
  --repetitions N                  Timed launches (one CSV row each). Default 1.
  --run-kind {{smoke,benchmark}}     'benchmark' requires working_set_bytes > 2xL2. Required.
  --fill {{pattern,uniform}}         SplitMix64 pattern (default) or seeded uniform words.
  --seed N                         Seed of --fill uniform. Default 0.
  --row-bytes {{128,256}}            TMA box row width in bytes. Default 256.
  --self-test                      Validate every specialisation on a small working set.
  --help                           Show this help and exit.
"""


def parse(argv: list[str]) -> dict:
    cfg = {"help": False, "self_test": False, "passes": 1, "warmup_ms": 0, "repetitions": 1, "fill": "pattern",
           "seed": 0, "row_bytes": 256}
    seen = set()
    i = 0
    while i < len(argv):
        a = argv[i]
        if a in ("--help", "-h"):
            cfg["help"] = True
            i += 1
            continue
        if a == "--self-test":
            cfg["self_test"] = True
            i += 1
            continue
        if a in seen:
            raise cm.UsageError(f"{a} specified more than once")
        seen.add(a)
        if a == "--stages":
            v, i = cm.take_value(argv, i, a)
            if v not in ("2", "3", "4", "8"):
                raise cm.UsageError("--stages must be one of 2, 3, 4, 8")
            cfg["stages"] = int(v)
        elif a == "--bytes-in-flight-kib":
            v, i = cm.take_value(argv, i, a)
            if v not in ("16", "32", "64"):
                raise cm.UsageError("--bytes-in-flight-kib must be one of 16, 32, 64")
            cfg["bif_kib"] = int(v)
        elif a == "--working-set-mib":
            v, i = cm.take_value(argv, i, a)
            cfg["working_set_mib"] = cm.parse_int(v, 1, 1 << 20, a)
        elif a == "--passes":
            v, i = cm.take_value(argv, i, a)
            cfg["passes"] = cm.parse_int(v, 1, 1000000, a)
        elif a == "--warmup-ms":
            v, i = cm.take_value(argv, i, a)
            cfg["warmup_ms"] = cm.parse_int(v, 0, 3600000, a)
        elif a == "--repetitions":
            v, i = cm.take_value(argv, i, a)
            cfg["repetitions"] = cm.parse_int(v, 1, 1000000, a)
        elif a == "--run-kind":
            v, i = cm.take_value(argv, i, a)
            if v not in ("smoke", "benchmark"):
                raise cm.UsageError("--run-kind must be 'smoke' or 'benchmark'")
            cfg["run_kind"] = v
        elif a == "--fill":
            v, i = cm.take_value(argv, i, a)
            if v not in ("pattern", "uniform"):
                raise cm.UsageError("--fill must be 'pattern' or 'uniform'")
            cfg["fill"] = v
        elif a == "--seed":
            v, i = cm.take_value(argv, i, a)
            cfg["seed"] = cm.parse_int(v, 0, (1 << 63) - 1, a)
        elif a == "--row-bytes":
            v, i = cm.take_value(argv, i, a)
            if v not in ("128", "256"):
                raise cm.UsageError("--row-bytes must be 128 or 256")
            cfg["row_bytes"] = int(v)
        else:
            raise cm.UsageError(f"unknown argument: {a}")
    if cfg["help"]:
        return cfg
    if cfg["self_test"]:
        if seen:
            raise cm.UsageError("--self-test cannot be combined with benchmark options")
        return cfg
    for flag, key in (("--stages", "stages"), ("--bytes-in-flight-kib", "bif_kib"), ("--run-kind", "run_kind")):
        if key not in cfg:
            raise cm.UsageError(f"{flag} is required (unless --self-test)")
    return cfg


def round_up(v: int, m: int) -> int:
    return m if v <= 0 else (v + m - 1) // m * m


def plan_working_set(gpu: cm.GpuInfo, requested_mib) -> tuple[int, int]:
    """(requested_bytes, working_set_bytes): ldgsts.cu:452-465."""
    common = gpu.sm_count * 32 * 1024
    requested = requested_mib * 1024 * 1024 if requested_mib is not None else 4 * gpu.l2_bytes
    return requested, round_up(requested, common)


def format_row(method, run_kind, sample, info, gpu, requested, ws, passes, warmup_ms, ms, correctness, mismatches,
               commit, dirty) -> str:
    useful = ws * passes
    gbps = useful / (ms / 1000.0) / 1e9 if ms > 0 else 0.0
    row_bytes = info["row_bytes"]
    fields = [
        "1", cm.now_utc_iso8601(), run_kind, method, str(sample), str(info["stages"]), str(row_bytes // 2),
        str(row_bytes), str(info["tile_rows"]), str(info["stage_bytes"]), str(info["bytes_in_flight"]), "16",
        str(info["stage_bytes"] // (128 * 16)), str(info["threads_per_cta"]), "1", str(info["occupancy_ctas_per_sm"]),
        str(info["grid_ctas"]), str(gpu.sm_count), str(info["smem_bytes"]), str(gpu.l2_bytes), str(requested),
        str(ws), cm.fixed6(ws / gpu.l2_bytes), str(passes), str(useful), str(warmup_ms), cm.fixed6(ms),
        cm.fixed6(gbps), correctness, str(mismatches), cm.csv_quote(gpu.name), gpu.uuid, gpu.compute_capability,
        str(gpu.driver_version), str(gpu.runtime_version), commit, dirty,
    ]
    return ",".join(fields)


def _xor_of(sink_list) -> int:
    x = 0
    for v in sink_list:
        x ^= v
    return x


def run_config(method: str, cfg: dict, gpu: cm.GpuInfo, uuid: str, print_header: bool = True,
               out=None) -> int:
    import torch

    out = out if out is not None else sys.stdout  # resolved per call (callers may redirect stdout)

    from .. import streaming

    requested, ws = plan_working_set(gpu, cfg.get("working_set_mib"))
    if cfg["run_kind"] == "benchmark" and ws <= 2 * gpu.l2_bytes:
        raise cm.RunFailure(f"working_set_bytes={ws} is not strictly greater than 2xL2 ({2 * gpu.l2_bytes}); "
                            "increase --working-set-mib for a benchmark run")
    row_bytes = cfg["row_bytes"] if method == "tma" else 256
    buf = torch.empty(ws // 4, dtype=torch.int32, device="cuda")
    run = streaming.StreamingRun(method, cfg["stages"], cfg["bif_kib"], buf, row_bytes=row_bytes)
    info = run.info
    if info["occupancy_ctas_per_sm"] != 1:
        raise cm.RunFailure(f"occupancy check failed: {info['occupancy_ctas_per_sm']} CTAs/SM, need exactly 1")
    mismatches = 0
    if cfg["fill"] == "pattern":
        streaming.fill_pattern(buf)
        mismatches = run.validate()
        if mismatches:
            raise cm.RunFailure(f"correctness validation FAILED: mismatches={mismatches}; no benchmark was run")
    else:
        streaming.fill_uniform_u32(buf, seed=cfg["seed"])
        run.run(passes=1)
        mine = _xor_of(run.checksums())
        other_method = "tma" if method == "ldgsts" else "ldgsts"
        other = streaming.StreamingRun(other_method, cfg["stages"], cfg["bif_kib"], buf, row_bytes=128)
        other.run(passes=1)
        if mine != _xor_of(other.checksums()):
            raise cm.RunFailure("checksum of checksums differs between the LDGSTS and TMA data paths")
    torch.cuda.synchronize()

    stream = run.stream
    t0 = time.monotonic()
    while (time.monotonic() - t0) * 1000.0 < cfg["warmup_ms"]:
        run.run(passes=cfg["passes"])
        stream.synchronize()
    run.check_status()

    commit, dirty = cm.git_commit_hash(), cm.git_dirty_flag()
    if print_header:
        print(CSV_HEADER, file=out)
    tiles_per_cta = max(1, info["total_tiles"] // info["grid_ctas"])
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    for rep in range(cfg["repetitions"]):
        # Keep the GPU busy while the host prepares the launch, so the start
        # event is not followed by host-side idle time.
        with torch.cuda.stream(stream):
            torch.cuda._sleep(200000)
        e0.record(stream)
        run.run(passes=cfg["passes"], rotation=rep % tiles_per_cta)
        e1.record(stream)
        e1.synchronize()
        ms = e0.elapsed_time(e1)
        run.check_status()
        print(format_row(method, cfg["run_kind"], rep, info, gpu, requested, ws, cfg["passes"], cfg["warmup_ms"], ms,
                         "OK", mismatches, commit, dirty), file=out, flush=True)
    del buf
    return cm.EXIT_OK


def self_test(method: str, gpu: cm.GpuInfo) -> int:
    import torch

    from .. import streaming

    ws = gpu.sm_count * 32 * 1024 * SELF_TEST_COMMON_MULTIPLES
    buf = torch.empty(ws // 4, dtype=torch.int32, device="cuda")
    streaming.fill_pattern(buf)
    overall = "PASS"
    for stages in STAGES:
        for bif in BIF_KIB:
            run = streaming.StreamingRun(method, stages, bif, buf)
            mism = run.validate()
            status = "PASS" if mism == 0 else "MISMATCH"
            if mism:
                overall = "MISMATCH"
            cm.eprint(f"{method}: SELF_TEST stages={stages} bytes_in_flight_kib={bif} "
                      f"stage_bytes={run.info['stage_bytes']} result={status} mismatches={mism}")
    cm.eprint(f"{method}: SELF_TEST_RESULT={overall}")
    return cm.EXIT_OK if overall == "PASS" else cm.EXIT_FAILURE


def main(argv: list[str] | None = None) -> int:
    argv = list(sys.argv[1:] if argv is None else argv)
    if not argv or argv[0] not in METHODS:
        cm.eprint(f"usage: python -m gb300_microbench_b200.cli.memory_paths {{ldgsts,tma}} ...")
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
        uuid = cm.expected_uuid(gpu)
        if cfg["self_test"]:
            return self_test(method, gpu)
        return run_config(method, cfg, gpu, uuid)
    except cm.RunFailure as exc:
        cm.eprint(f"{method}: ERROR: {exc}")
        return cm.EXIT_FAILURE
    except Exception as exc:  # CUDA or native failure: no partial success
        cm.eprint(f"{method}: ERROR: {type(exc).__name__}: {exc}; discard any partial CSV output")
        return cm.EXIT_FAILURE


if __name__ == "__main__":
    raise SystemExit(main())
