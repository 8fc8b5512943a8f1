"""Regenerates the golden fixtures of tests/golden/ from the reference.

Run in a container that has the reference tree (GB300_REFERENCE or --reference)
and the CuTe DSL package the reference's driver uses:

    make -C oracle ref REFERENCE=$GB300_REFERENCE
    python tests/golden/make_golden.py [--reference PATH]

* gemm_reference_inputs.json: a small reference-mode operand draw made with
  the reference's own input helper, exactly as the pinned upstream
  create_tensors calls it (torch.manual_seed(1111); cutlass.torch.matrix for
  A then B; dense_gemm.py:1498-1506, gemm_comparison.py:2626-2655).
* umma_reference_d.json: samples of the reference's own reference_d
  (umma_throughput/umma_1sm.cu:566-575), through oracle/_ref/libref_umma.so,
  which is built from the reference source where it lies.
* pattern.json: SplitMix64 pattern vectors (memory_paths/ldgsts.cu:220-232),
  computed here with plain Python integers, independently of the C oracle.
"""
from __future__ import annotations

import argparse
import os
import json
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]
sys.path.insert(0, str(ROOT))

MASK = (1 << 64) - 1


def mix64_py(x: int) -> int:
    x = ((x ^ (x >> 30)) * 0xBF58476D1CE4E5B9) & MASK
    x = ((x ^ (x >> 27)) * 0x94D049BB133111EB) & MASK
    return x ^ (x >> 31)


def pattern_py(i: int) -> list[int]:
    lo, hi = mix64_py(i), mix64_py(i ^ 0xD1B54A32D192ED03)
    return [lo & 0xFFFFFFFF, lo >> 32, hi & 0xFFFFFFFF, hi >> 32]


def write_csv_headers(reference: Path) -> None:
    """csv_headers.json: the reference's three raw CSV schemas, read from its
    sources (memory_paths/ldgsts.cu:734-745, umma_throughput/umma_1sm.cu:
    965-973, gemm_comparison/gemm_comparison.py:319-429)."""
    import importlib.util
    import re

    def header_from_cu(path: Path) -> list[str]:
        text = path.read_text()
        block = text[text.index("void print_csv_header()"):]
        block = block[: block.index("}")]
        return "".join(re.findall(r'"([^"]*)"', block)).replace("\\n", "").strip().split(",")

    spec = importlib.util.spec_from_file_location("ref_gemm_comparison",
                                                  reference / "gemm_comparison" / "gemm_comparison.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    (HERE / "csv_headers.json").write_text(json.dumps({
        "source": "print_csv_header of memory_paths/ldgsts.cu, memory_paths/tma.cu, umma_throughput/umma_1sm.cu, "
                  "umma_throughput/umma_2sm.cu; CSV_FIELDS of gemm_comparison/gemm_comparison.py",
        "memory_paths": header_from_cu(reference / "memory_paths" / "ldgsts.cu"),
        "memory_paths_tma": header_from_cu(reference / "memory_paths" / "tma.cu"),
        "umma": header_from_cu(reference / "umma_throughput" / "umma_1sm.cu"),
        "umma_2sm": header_from_cu(reference / "umma_throughput" / "umma_2sm.cu"),
        "gemm": list(mod.CSV_FIELDS),
    }, indent=1) + "\n")


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("GB300_REFERENCE"), required=not os.environ.get("GB300_REFERENCE"))
    args = ap.parse_args()

    import torch
    import cutlass
    import cutlass.torch as cutlass_torch

    m, n, k, l = 8, 6, 16, 1
    torch.manual_seed(1111)
    a = cutlass_torch.matrix(l, m, k, False, cutlass.BFloat16)  # (m, k, l)
    b = cutlass_torch.matrix(l, n, k, False, cutlass.BFloat16)
    a_lmk = a.permute(2, 0, 1).contiguous()
    b_lnk = b.permute(2, 0, 1).contiguous()
    (HERE / "gemm_reference_inputs.json").write_text(json.dumps({
        "source": "torch.manual_seed(1111); cutlass.torch.matrix(l, m, k, False, BFloat16) then (l, n, k)",
        "mnkl": [m, n, k, l],
        "a": a_lmk.float().flatten().tolist(),
        "b": b_lnk.float().flatten().tolist(),
    }, indent=1) + "\n")

    import oracle

    oracle.build(reference=args.reference)
    ref = oracle.ref_umma_lib()
    if ref is None:
        raise SystemExit("oracle/_ref/libref_umma.so was not built")
    samples = {}
    for depth in (4, 16, 32, 64, 128, 256):
        samples[str(depth)] = [[r, c, ref.ref_umma_reference_d(r, c, depth)]
                               for r in range(0, 256, 37) for c in range(0, 256, 29)]
    (HERE / "umma_reference_d.json").write_text(json.dumps({
        "source": "reference_d of umma_throughput/umma_1sm.cu via oracle/_ref/libref_umma.so",
        "samples": samples}, indent=1) + "\n")

    vectors = {str(v0): [w for i in range(v0, v0 + 4) for w in pattern_py(i)]
               for v0 in (0, 1, 1000, 123456789, (1 << 32) + 7)}
    (HERE / "pattern.json").write_text(json.dumps({
        "source": "SplitMix64 pattern of memory_paths/ldgsts.cu:220-232, pure-Python restatement",
        "vectors": vectors}, indent=1) + "\n")
    write_csv_headers(Path(args.reference))
    print("golden fixtures written", file=sys.stderr)
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
