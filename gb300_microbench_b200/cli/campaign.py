"""One measurement campaign on one GPU, frozen as the directory the
reference's analysis reads (scripts/run_campaign.py:407-511, without its
container launcher), optionally with the Nsight Compute stage of
scripts/ncu_capture.py.

    python -m gb300_microbench_b200.cli.campaign --kind {pilot,final} --output-root DIR
        [--campaign-id YYYYMMDDTHHMMSSZ] [--with-ncu]

Stages, in the reference's order: the memory sweep (the reference grid:
{ldgsts,tma} x stages {2,4,8} x {16,32,64} KiB in flight, 512 MiB x 32
passes, 2000 ms warm-up, 30 repetitions), the UMMA sweep (N {64,128,256} x
depth {4,16,64,256} x {umma_1sm,umma_2sm}, 1000 iterations, 10 warm-up
launches, 30 repetitions), the GEMM comparison (five frozen shapes x four
candidates, 2 warm-up and 10 timed launches, hot cache), then, with
--with-ncu, one Nsight Compute capture of each of the reference's planned
kernels (ncu_capture.py:42-79: six memory and 24 UMMA configurations, its
metric lists and collection flags, the campaign's own parameters with no
warm-up and one repetition). Each profiled command first runs once without
the profiler and must exit 0. A capture that fails is recorded with its
reason and never stops the campaign.

The manifest (schema gb300.campaign.v1) records: the commit (B200_GIT_COMMIT
where the tree was copied without .git), the GPU (uuid, name, driver), a
software-stack identity in place of a container image (there is none: the
sha256 of the Python, torch, CUDA runtime and driver versions), the hashes
of this build's sources, of the raw CSVs and of the profile files.
"""
from __future__ import annotations

import argparse
import datetime as dt
import hashlib
import json
import os
import platform
import re
import subprocess
import sys
import tempfile
from pathlib import Path

from . import common as cm

CAMPAIGN_RE = re.compile(r"^[0-9]{8}T[0-9]{6}Z$")
RAW_FILES = ("raw/memory_paths.csv", "raw/umma_throughput.csv", "raw/gemm_comparison.csv")
NCU_DIR = "ncu"
NCU_INDEX_SCHEMA = "gb300.ncu.v1"

# The reference's profile plan and metric lists (scripts/ncu_capture.py:42-95),
# kept so the analysis finds the cases and counters it expects.
MEMORY_CASES = (("ldgsts", 2, 16), ("tma", 2, 16), ("tma", 4, 32), ("ldgsts", 4, 32), ("ldgsts", 8, 64),
                ("tma", 8, 64))
UMMA_CASES = tuple((method, n, depth) for n in (64, 128, 256) for depth in (4, 16, 64, 256)
                   for method in ("umma_1sm", "umma_2sm"))
MEMORY_METRICS = ("dram__bytes_read.sum", "dram__bytes_write.sum",
                  "dram__throughput.avg.pct_of_peak_sustained_elapsed", "lts__t_bytes.sum", "gpu__time_duration.sum")
UMMA_METRICS = ("sm__cycles_elapsed.avg.per_second", "gpu__time_duration.sum",
                "sm__pipe_tensor_op_hmma_cycles_active.avg.pct_of_peak_sustained_elapsed",
                "sm__pipe_tensor_cycles_active.avg.pct_of_peak_sustained_elapsed",
                "sm__inst_executed_pipe_tensor.sum", "smsp__inst_executed_pipe_tensor.sum")
NCU_COLLECT = ("--clock-control", "none", "--pipeline-boost-state", "dynamic", "--cache-control", "none",
               "--kernel-name-base", "function", "--launch-count", "1", "--devices", "0", "--replay-mode", "kernel",
               "--print-summary", "none")
NCU_EXPORT = ("--csv", "--page", "raw", "--print-units", "base", "--print-fp", "--print-kernel-base", "function")
CAPTURE_TIMEOUT_S = 600

SOURCES = ("gb300_microbench_b200/csrc/copy_kernels.cu", "gb300_microbench_b200/csrc/umma_probe.cu",
           "gb300_microbench_b200/csrc/gemm_sm100.cu", "gb300_microbench_b200/csrc/gemm_capi.cu",
           "gb300_microbench_b200/csrc/cublaslt_cmp.cu", "gb300_microbench_b200/csrc/ptx.cuh",
           "gb300_microbench_b200/cli/memory_paths.py", "gb300_microbench_b200/cli/umma.py",
           "gb300_microbench_b200/cli/gemm_comparison.py", "gb300_microbench_b200/cli/sweeps.py",
           "gb300_microbench_b200/cli/campaign.py", "include/b200bench.h")


def sha256_file(path: Path) -> str:
    h = hashlib.sha256()
    with path.open("rb") as fh:
        for chunk in iter(lambda: fh.read(1 << 20), b""):
            h.update(chunk)
    return h.hexdigest()


def utc_now() -> dt.datetime:
    return dt.datetime.now(dt.timezone.utc).replace(microsecond=0)


def iso(t: dt.datetime) -> str:
    return t.isoformat().replace("+00:00", "Z")


def driver_version() -> str:
    """The display driver version as nvidia-smi prints it (e.g. 580.159)."""
    try:
        import pynvml

        pynvml.nvmlInit()
        v = pynvml.nvmlSystemGetDriverVersion()
        return v.decode() if isinstance(v, bytes) else str(v)
    except Exception:
        return "unknown"


def stack_identity() -> dict:
    import torch

    desc = {"python": platform.python_version(), "torch": torch.__version__, "cuda_runtime": torch.version.cuda,
            "driver": driver_version(), "platform": platform.platform()}
    digest = hashlib.sha256(json.dumps(desc, sort_keys=True).encode()).hexdigest()
    return {"tag": "software-stack", "id": f"sha256:{digest}", "components": desc}


def app_argv(section: str, case: tuple) -> list[str]:
    """One profiled launch with the campaign's own parameters
    (ncu_capture.py:299-323)."""
    if section == "memory_paths":
        method, stages, bif = case
        return [sys.executable, "-m", "gb300_microbench_b200.cli.memory_paths", method, "--stages", str(stages),
                "--bytes-in-flight-kib", str(bif), "--run-kind", "benchmark", "--working-set-mib", "512",
                "--passes", "32", "--warmup-ms", "0", "--repetitions", "1"]
    method, n, depth = case
    return [sys.executable, "-m", "gb300_microbench_b200.cli.umma", method, "--run-kind", "benchmark", "--n", str(n),
            "--depth", str(depth), "--iterations", "1000", "--warmup-iterations", "0", "--repetitions", "1"]


def useful_bytes_of(app_stdout: str):
    lines = [ln for ln in app_stdout.splitlines() if ln.strip()]
    if len(lines) < 2 or "useful_bytes" not in lines[0].split(","):
        return None
    header, cells = lines[0].split(","), lines[1].split(",")
    try:
        return float(cells[header.index("useful_bytes")]) if len(cells) == len(header) else None
    except ValueError:
        return None


def case_record(section: str, index: int, case: tuple) -> tuple[dict, tuple]:
    if section == "memory_paths":
        method, stages, bif = case
        return ({"section": section, "case": f"{index:02d}_{method}_s{stages}_bif{bif}", "method": method,
                 "stages": stages, "bytes_in_flight_kib": bif, "kernel_name": f"{method}_benchmark_kernel"},
                MEMORY_METRICS)
    method, n, depth = case
    kernel = f"umma_1sm_m128n{n}k16_d{depth}" if method == "umma_1sm" else f"umma_2sm_m256n{n}k16_d{depth}"
    return ({"section": section, "case": f"{index:02d}_{method}_n{n}_d{depth}", "method": method, "n": n,
             "depth": depth, "kernel_name": kernel}, UMMA_METRICS)


def capture(section: str, index: int, case: tuple, out_dir: Path, env: dict, ncu: str) -> dict:
    record, metrics = case_record(section, index, case)
    record.update({"status": "unavailable", "reason": "", "csv": "", "useful_bytes": None})
    app = app_argv(section, case)
    plain = subprocess.run(app, cwd=cm.REPO_ROOT, env=env, text=True, capture_output=True, check=False,
                           timeout=CAPTURE_TIMEOUT_S)
    if plain.returncode != 0:
        record["reason"] = f"plain_run_exit_{plain.returncode}"
        return record
    with tempfile.TemporaryDirectory(prefix="ncu_case.") as work:
        rep = Path(work) / "report"
        collect = [ncu, *NCU_COLLECT, "--kernel-name", record["kernel_name"], "--metrics", ",".join(metrics),
                   "--log-file", str(Path(work) / "tool.log"), "-o", str(rep), "--", *app]
        try:
            res = subprocess.run(collect, cwd=cm.REPO_ROOT, env=env, text=True, capture_output=True, check=False,
                                 timeout=CAPTURE_TIMEOUT_S)
        except subprocess.TimeoutExpired:
            record["reason"] = "capture_timeout"
            return record
        if res.returncode != 0 or not Path(f"{rep}.ncu-rep").exists():
            record["reason"] = f"profiler_exit_{res.returncode}"
            return record
        exp = subprocess.run([ncu, *NCU_EXPORT, "--import", f"{rep}.ncu-rep"], text=True, capture_output=True,
                             check=False)
        if exp.returncode != 0 or not exp.stdout.strip():
            record["reason"] = f"export_exit_{exp.returncode}"
            return record
    (out_dir / f"{record['case']}.csv").write_text(exp.stdout, encoding="utf-8")
    record.update({"status": "captured", "csv": f"{record['case']}.csv"})
    if section == "memory_paths":
        record["useful_bytes"] = useful_bytes_of(res.stdout) or useful_bytes_of(plain.stdout)
    return record


def ncu_stage(partial: Path, env: dict, ncu: str) -> dict:
    out = partial / NCU_DIR
    out.mkdir()
    started = iso(utc_now())
    cases = []
    for section, plan in (("memory_paths", MEMORY_CASES), ("umma_throughput", UMMA_CASES)):
        for i, case in enumerate(plan):
            cases.append(capture(section, i, case, out, env, ncu))
            cm.eprint(f"campaign: ncu {cases[-1]['case']}: {cases[-1]['status']} {cases[-1]['reason']}")
    captured = sum(1 for c in cases if c["status"] == "captured")
    state = "COMPLETE" if captured == len(cases) else ("PARTIAL" if captured else "UNAVAILABLE")
    index = {"schema_version": NCU_INDEX_SCHEMA, "state": state, "started_utc": started, "finished_utc": iso(utc_now()),
             "case_count": len(cases), "captured_count": captured,
             "metrics": {"memory_paths": list(MEMORY_METRICS), "umma_throughput": list(UMMA_METRICS)},
             "cases": cases}
    (out / "index.json").write_text(json.dumps(index, indent=2, sort_keys=True) + "\n", encoding="utf-8")
    files = sorted(p for p in out.iterdir() if p.is_file())
    return {"requested": True, "state": state, "case_count": len(cases), "captured_count": captured,
            "artifact_sha256": {f"{NCU_DIR}/{p.name}": sha256_file(p) for p in files}}


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="campaign", description=__doc__.splitlines()[0])
    ap.add_argument("--kind", choices=("pilot", "final"), required=True)
    ap.add_argument("--campaign-id")
    ap.add_argument("--output-root", type=Path, required=True)
    ap.add_argument("--with-ncu", action="store_true")
    ap.add_argument("--ncu-binary", default=os.environ.get("NCU_BINARY", "ncu"))
    args = ap.parse_args(sys.argv[1:] if argv is None else argv)
    campaign_id = args.campaign_id or utc_now().strftime("%Y%m%dT%H%M%SZ")
    if not CAMPAIGN_RE.fullmatch(campaign_id):
        cm.eprint("campaign: the campaign ID must match YYYYMMDDTHHMMSSZ")
        return cm.EXIT_USAGE
    commit = cm.git_commit_hash()
    if not re.fullmatch(r"[0-9a-f]{40}", commit):
        cm.eprint(f"campaign: no usable git commit ({commit!r}); set B200_GIT_COMMIT")
        return cm.EXIT_USAGE
    final = args.output_root / campaign_id
    partial = args.output_root / f"{campaign_id}.partial"
    if final.exists() or partial.exists():
        cm.eprint(f"campaign: {final} already exists")
        return cm.EXIT_USAGE
    gpu_info = cm.query_gpu()
    gpu = {"index": "0", "uuid": gpu_info.uuid, "name": gpu_info.name, "driver_version": driver_version()}
    env = dict(os.environ, EXPECTED_GPU_UUID=gpu_info.uuid, B200_GIT_COMMIT=commit,
               B200_GIT_DIRTY=os.environ.get("B200_GIT_DIRTY", cm.git_dirty_flag()))
    started = utc_now()
    (partial / "raw").mkdir(parents=True)
    steps = (
        (["gb300_microbench_b200.cli.sweeps", "memory", "--run-kind", "benchmark", "--output",
          str(partial / RAW_FILES[0])], None),
        (["gb300_microbench_b200.cli.sweeps", "umma", "--run-kind", "benchmark", "--output",
          str(partial / RAW_FILES[1])], None),
        # The GEMM comparison writes its CSV to stdout.
        (["gb300_microbench_b200.cli.gemm_comparison", "--warmup-iterations", "2", "--iterations", "10"],
         partial / RAW_FILES[2]),
    )
    for argv_, stdout_file in steps:
        res = subprocess.run([sys.executable, "-m", *argv_], cwd=cm.REPO_ROOT, env=env, text=True,
                             capture_output=True, check=False)
        if res.returncode != 0:
            cm.eprint(f"campaign: {' '.join(argv_)} exited {res.returncode}:\n{res.stderr[-3000:]}")
            return cm.EXIT_FAILURE
        if stdout_file is not None:
            stdout_file.write_text(res.stdout, encoding="utf-8")
        cm.eprint(f"campaign: {argv_[0]} {argv_[1]} done")
    ncu = (ncu_stage(partial, env, args.ncu_binary) if args.with_ncu
           else {"requested": False, "state": "NOT_REQUESTED", "case_count": 0, "captured_count": 0,
                 "artifact_sha256": {}})
    artifacts = {rel: sha256_file(partial / rel) for rel in RAW_FILES}
    manifest = {
        "schema_version": "gb300.campaign.v1", "campaign_id": campaign_id, "campaign_kind": args.kind,
        "state": "COMPLETE", "started_utc": iso(started), "finished_utc": iso(utc_now()), "git_commit": commit,
        "git_dirty": env["B200_GIT_DIRTY"] == "true", "gpu": gpu, "container_image": stack_identity(),
        "stage_order": ["memory_paths", "umma_throughput", "gemm_comparison"]
                       + (["ncu_capture"] if args.with_ncu else []),
        "parameters": {
            "memory_paths": {"working_set_mib": 512, "passes": 32, "warmup_ms": 2000, "repetitions": 30,
                             "configuration_count": 18},
            "umma_throughput": {"iterations": 1000, "warmup_iterations": 10, "repetitions": 30,
                                "configuration_count": 24},
            "gemm_comparison": {"warmup_iterations": 2, "iterations": 10, "shape_count": 5, "candidate_count": 4,
                                "cache_mode": "hot"},
        },
        "artifact_sha256": artifacts, "ncu": ncu,
        "source_sha256": {rel: sha256_file(cm.REPO_ROOT / rel) for rel in SOURCES},
    }
    (partial / "manifest.json").write_text(json.dumps(manifest, indent=2, sort_keys=True) + "\n", encoding="utf-8")
    (partial / "SHA256SUMS").write_text("".join(f"{d}  {r}\n" for r, d in sorted(artifacts.items())),
                                        encoding="utf-8")
    partial.rename(final)
    cm.eprint(f"campaign: COMPLETE {final}")
    return cm.EXIT_OK


if __name__ == "__main__":
    raise SystemExit(main())
