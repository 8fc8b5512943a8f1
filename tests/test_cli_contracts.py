"""CPU checks of the command-line drivers against the reference's contracts:
CSV schemas equal the reference's (golden headers read from its sources),
the GEMM comparison arithmetic equals the reference's own functions, rows
built by our GEMM driver pass the reference's row and table validators, and
the committed B200 result CSVs pass the reference's campaign validators.
Checks that need the reference tree skip where it is absent."""
import csv
import importlib.util
import json
import os
import random
import sys
from pathlib import Path

import pytest

from gb300_microbench_b200.cli import gemm_comparison as gc
from gb300_microbench_b200.cli import memory_paths as mp
from gb300_microbench_b200.cli import umma as um

ROOT = Path(__file__).resolve().parents[1]
GOLDEN = Path(__file__).resolve().parent / "golden"
REFERENCE = Path(os.environ["GB300_REFERENCE"]) if os.environ.get("GB300_REFERENCE") else None


def _ref_module(rel: str, name: str):
    if REFERENCE is None:
        pytest.skip("GB300_REFERENCE does not name the reference tree")
    path = REFERENCE / rel
    if not path.exists():
        pytest.skip("reference tree not present")
    sys.path.insert(0, str(path.parent))
    spec = importlib.util.spec_from_file_location(name, path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def test_csv_headers_equal_reference_schemas():
    g = json.loads((GOLDEN / "csv_headers.json").read_text())
    assert mp.CSV_HEADER.split(",") == g["memory_paths"] == g["memory_paths_tma"]
    assert um.CSV_HEADER.split(",") == g["umma"] == g["umma_2sm"]
    assert list(gc.CSV_FIELDS) == g["gemm"]


@pytest.mark.parametrize("argv,code", [(["ldgsts", "--help"], 0), (["tma", "--stages", "5"], 2),
                                       (["ldgsts", "--stages", "2"], 2), (["nope"], 2),
                                       (["ldgsts", "--self-test", "--stages", "2"], 2),
                                       (["tma", "--passes", "0", "--stages", "2"], 2)])
def test_memory_cli_usage_errors_exit_2(argv, code):
    assert mp.main(argv) == code


@pytest.mark.parametrize("argv,code", [(["umma_1sm", "--help"], 0), (["umma_2sm", "--n", "96"], 2),
                                       (["umma_1sm", "--depth", "8"], 2), (["umma_1sm", "--run-kind", "smoke"], 2)])
def test_umma_cli_usage_errors_exit_2(argv, code):
    assert um.main(argv) == code


def test_gemm_self_test_and_usage():
    assert gc.main(["--self-test"]) == 0
    assert gc.main(["--iterations", "0"]) == 2


def test_comparison_arithmetic_matches_reference():
    ref = _ref_module("gemm_comparison/gemm_comparison.py", "ref_gc")
    rnd = random.Random(7)
    order = [c[1] for c in gc.CANDIDATES]
    for trial in range(200):
        times = [rnd.choice([0.5, 1.0, 1.0, 2.0, rnd.uniform(0.1, 3.0)]) for _ in range(4)]
        mnkl = ref.FROZEN_SHAPES[trial % 5]
        want = ref.compute_shape_comparison(mnkl, times)
        got = gc.compute_shape_comparison(mnkl, times, gc.CUBLASLT_INDEX, (0, 1, 2), order)
        for w, g in zip(want, got):
            assert w["flop_count"] == g["flop_count"]
            assert w["rank_within_shape"] == g["rank_within_shape"]
            assert w["best_cutedsl_variant"] == g["best_cutedsl_variant"]
            assert w["is_best_cutedsl"] == g["is_best_cutedsl"]
            assert w["tflops"] == pytest.approx(g["tflops"], rel=1e-15)
            assert w["throughput_ratio_vs_cublaslt"] == pytest.approx(g["throughput_ratio_vs_cublaslt"], rel=1e-15)


def _fake_results(mnkl, rnd):
    cmp_info = {"layout": 1, "cublaslt_version": 120904, "lda": mnkl[2], "ldb": mnkl[2], "ldc": mnkl[1],
                "ldd": mnkl[1], "transa": 0, "transb": 1, "order_a": 1, "order_b": 1, "order_c": 1, "order_d": 1,
                "type_ab": 14, "type_d": 0, "compute_type": 68, "scale_type": 0, "pointer_mode": 0, "epilogue": 1,
                "search_mode": 0, "workspace_limit_bytes": 67108864, "workspace_bytes": 0,
                "heuristic_requested": 32, "heuristic_returned": 8, "heuristic_index": 0,
                "alignment_a_bytes": 256, "alignment_b_bytes": 256, "alignment_c_bytes": 256,
                "alignment_d_bytes": 256, "algo_id": 66, "tile_id": 18, "stages_id": 0, "split_k": 1,
                "reduction_scheme": 0, "cta_swizzling": 0, "custom_option": 0, "inner_shape_id": 0,
                "cluster_shape_id": 2, "waves_count": 1.73, "alpha": 1.0, "beta": 0.0}
    res = []
    for spec in gc.CANDIDATES:
        tile, cluster = spec[3], spec[4]
        info = None if spec[0] == "cublaslt" else {"mma_tiler_m": tile[0], "mma_tiler_n": tile[1],
                                                   "cluster_m": cluster[0], "max_active_clusters": 74}
        res.append({"spec": spec, "compile_ms": None if spec[0] == "cublaslt" else 12.5,
                    "setup_ms": 3.25 if spec[0] == "cublaslt" else None, "first_ms": 0.5,
                    "ms": rnd.uniform(0.05, 1.0), "max_abs": 0.0, "max_rel": 0.0, "info": info,
                    "cmp": cmp_info if spec[0] == "cublaslt" else None})
    return res


def test_our_rows_pass_reference_validators():
    ref = _ref_module("gemm_comparison/gemm_comparison.py", "ref_gc2")
    rnd = random.Random(3)
    prov = {"gpu_name": "NVIDIA B200", "gpu_uuid": "GPU-0123abcd-0000-1111-2222-333344445555",
            "compute_capability": "10.0", "driver_version": "580.159", "cuda_toolkit_version": "12.9",
            "torch_cuda_version": "12.8", "cutedsl_version": "0.1.0", "cutlass_commit": "a" * 40,
            "operand_factory_sha256": "b" * 64, "git_commit": "a" * 40, "git_dirty": "false"}
    order = [c[1] for c in gc.CANDIDATES]
    rows = []
    for si, mnkl in enumerate(gc.FROZEN_SHAPES):
        res = _fake_results(mnkl, rnd)
        comp = gc.compute_shape_comparison(mnkl, [r["ms"] for r in res], gc.CUBLASLT_INDEX, (0, 1, 2), order)
        rows += gc.build_rows("reference", si, mnkl, res, comp, prov, 5, 20)
    ref.validate_rows(rows)
    text = gc.serialize(rows)
    assert text.count("\n") == 21
    parsed = list(csv.DictReader(text.splitlines()))
    ref.validate_rows(parsed)


def test_committed_result_csvs_pass_campaign_validators():
    rc = _ref_module("scripts/run_campaign.py", "ref_rc")
    for name, validator in (("memory_paths_reference.csv", rc.validate_memory),
                            ("umma_reference.csv", rc.validate_umma),
                            ("gemm_comparison.csv", rc.validate_gemm)):
        path = ROOT / "results" / name
        rows = list(csv.DictReader(path.read_text().splitlines()))
        n = validator(path, commit=rows[0]["git_commit"], gpu_uuid=rows[0]["gpu_uuid"])
        assert n == len(rows)


def test_committed_result_csvs_feed_reference_analysis(tmp_path):
    """The reference's cross-campaign statistics (analysis/analyze.py:484-886)
    and figures (:1099) consume the committed B200 CSVs unchanged. The three
    records here are the same sweep CSVs three times, with no profiles; the
    three measured campaigns with their Nsight Compute captures are checked
    by tests/test_campaign.py."""
    an = _ref_module("analysis/analyze.py", "ref_analyze")

    def rows(name):
        return list(csv.DictReader((ROOT / "results" / name).read_text().splitlines()))

    records = [{"campaign_id": f"c{i}", "manifest": {}, "memory": rows("memory_paths_reference.csv"),
                "umma": rows("umma_reference.csv"), "gemm": rows("gemm_comparison.csv"),
                "profiles": {"memory_paths": {}, "umma_throughput": {}, "gemm_comparison": {}}}
               for i in range(3)]
    mem_rows, mem = an.memory_analysis(records)
    umma_rows, umma = an.umma_analysis(records)
    gemm_rows, gemm = an.gemm_analysis(records)
    assert len(mem["configurations"]) == 18  # {ldgsts, tma} x stages {2,4,8} x {16,32,64} KiB
    assert len(umma["configurations"]) == 24  # {1sm, 2sm} x N {64,128,256} x depth {4,16,64,256}
    assert [s["shape_index"] for s in gemm["shapes"]] == [1, 2, 3, 4, 5]
    assert all(s["best_cutedsl_variant_consensus"] for s in gemm["shapes"])
    assert mem_rows and umma_rows and gemm_rows
    an.figures(tmp_path, mem, umma, gemm)
    assert any(p.suffix == ".svg" for p in (tmp_path / "figures").iterdir())


@pytest.mark.parametrize("bad", ["12x3", "0x8x8", "axbxc", "8x8x8,"])
def test_multigpu_shapes_usage_errors(bad, capsys):
    from gb300_microbench_b200.cli import multigpu

    assert multigpu.main(["--shapes", bad]) == 2
    assert "--shapes" in capsys.readouterr().err
