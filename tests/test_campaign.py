"""The campaign driver's host logic: its profile plan names the cases and
kernels the reference's capture plan names (scripts/ncu_capture.py:42-79),
its metric lists equal the reference's, and bad identifiers are refused
before anything runs."""
import importlib.util
import os
import sys
from pathlib import Path

import pytest

from gb300_microbench_b200.cli import campaign as cp


def _ref_capture():
    ref = os.environ.get("GB300_REFERENCE")
    path = Path(ref, "scripts", "ncu_capture.py") if ref else None
    if path is None or not path.exists():
        pytest.skip("GB300_REFERENCE does not name the reference tree")
    spec = importlib.util.spec_from_file_location("ref_ncu_capture", path)
    mod = importlib.util.module_from_spec(spec)
    sys.modules["ref_ncu_capture"] = mod
    spec.loader.exec_module(mod)
    return mod


def test_plan_matches_reference_capture_plan():
    ref = _ref_capture()
    ours = [cp.case_record("memory_paths", i, c)[0] for i, c in enumerate(cp.MEMORY_CASES)]
    ours += [cp.case_record("umma_throughput", i, c)[0] for i, c in enumerate(cp.UMMA_CASES)]
    theirs = [{k: v for k, v in e.items() if k != "binary"} for e in (*ref.MEMORY_PLAN, *ref.UMMA_PLAN)]
    assert ours == theirs
    assert cp.MEMORY_METRICS == ref.MEMORY_METRICS and cp.UMMA_METRICS == ref.UMMA_METRICS
    assert cp.NCU_COLLECT == ref.COLLECTION_FLAGS and cp.NCU_EXPORT == ref.EXPORT_FLAGS


def test_plan_sizes_and_names():
    assert len(cp.MEMORY_CASES) == 6 and len(cp.UMMA_CASES) == 24
    rec, metrics = cp.case_record("umma_throughput", 23, ("umma_2sm", 256, 256))
    assert rec["kernel_name"] == "umma_2sm_m256n256k16_d256" and rec["case"] == "23_umma_2sm_n256_d256"
    assert "sm__cycles_elapsed.avg.per_second" in metrics


def test_useful_bytes_parsing():
    assert cp.useful_bytes_of("a,useful_bytes,b\n1,17226006528,3\n") == 17226006528.0
    assert cp.useful_bytes_of("no header here\n") is None


@pytest.mark.parametrize("argv", [["--kind", "final", "--output-root", "x", "--campaign-id", "bad"],
                                  ["--kind", "final", "--output-root", "x", "--campaign-id", "20261202T0101Z"]])
def test_bad_campaign_id_refused(argv, monkeypatch):
    monkeypatch.setenv("B200_GIT_COMMIT", "a" * 40)
    assert cp.main(argv) == 2


def _ref_analyze():
    ref = os.environ.get("GB300_REFERENCE")
    if not ref or not Path(ref, "analysis", "analyze.py").exists():
        pytest.skip("GB300_REFERENCE does not name the reference tree")
    for sub in ("scripts", "analysis"):
        sys.path.insert(0, str(Path(ref, sub)))
    spec = importlib.util.spec_from_file_location("ref_analyze_campaigns", Path(ref, "analysis", "analyze.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


CAMPAIGNS = Path(__file__).resolve().parents[1] / "results" / "campaigns"


def test_committed_campaigns_pass_reference_analysis():
    """The three committed campaigns pass the reference's campaign reader
    (manifest schema, artifact hashes, the row validators, the profile
    index and hashes) and its population check, and its analysis derives the
    counter-based figures from their profiles."""
    an = _ref_analyze()
    dirs = sorted(p for p in CAMPAIGNS.iterdir() if p.is_dir()) if CAMPAIGNS.exists() else []
    if len(dirs) != 3:
        pytest.skip("no committed campaigns")
    records = [an.campaign(d) for d in dirs]
    an.validate_population(records)
    assert all(r["profiles"]["state"] in ("COMPLETE", "PARTIAL") for r in records)
    _, mem = an.memory_analysis(records)
    _, umma = an.umma_analysis(records)
    assert len(mem["configurations"]) == 18 and len(umma["configurations"]) == 24
