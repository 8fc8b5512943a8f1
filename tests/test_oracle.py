"""The CPU oracle, pinned before it is trusted.

* the SplitMix64 mixer against SplitMix64's published first output for
  seed 0;
* the UMMA known answer against the reference's own reference_d, compiled
  from umma_throughput/umma_1sm.cu (oracle/_ref), when present, and against
  the committed golden fixture;
* the reference-mode GEMM operand draw against the golden fixture made with
  the reference's input helper (tests/golden/make_golden.py);
* the checksum arithmetic against a direct numpy restatement.
"""
import json
from pathlib import Path

import numpy as np
import pytest
import torch

import oracle
from gb300_microbench_b200 import inputs

GOLDEN = Path(__file__).resolve().parent / "golden"


def test_splitmix64_published_vector():
    # SplitMix64 with state 0: state += 0x9E3779B97F4A7C15, output mix(state).
    assert oracle.mix64(0x9E3779B97F4A7C15) == 0xE220A8397B1DCDAF
    assert oracle.mix64(2 * 0x9E3779B97F4A7C15 % (1 << 64)) == 0x6E789E6AA1B965F4


def test_pattern_words_layout():
    w = oracle.pattern_words(5, 1)
    lo, hi = oracle.mix64(5), oracle.mix64(5 ^ 0xD1B54A32D192ED03)
    assert list(w) == [lo & 0xFFFFFFFF, lo >> 32, hi & 0xFFFFFFFF, hi >> 32]


def test_golden_pattern_fixture():
    g = json.loads((GOLDEN / "pattern.json").read_text())
    for vec0, words in g["vectors"].items():
        assert [int(x) for x in oracle.pattern_words(int(vec0), len(words) // 4)] == words


def test_umma_reference_d_pinned_to_reference_build():
    ref = oracle.ref_umma_lib()
    if ref is None:
        pytest.skip("oracle/_ref not built (no reference tree on this machine)")
    for depth in (4, 16, 64, 256):
        for row in range(0, 256, 7):
            for col in range(0, 256, 5):
                assert ref.ref_umma_reference_d(row, col, depth) == oracle.lib().bbo_umma_reference_d(row, col, depth)


def test_umma_golden_fixture():
    g = json.loads((GOLDEN / "umma_reference_d.json").read_text())
    for key, vals in g["samples"].items():
        depth = int(key)
        for (row, col, want) in vals:
            assert oracle.lib().bbo_umma_reference_d(row, col, depth) == want


def test_umma_general_matches_pattern():
    for cg in (1, 2):
        a, b = inputs.umma_pattern_operands(cg, 64)
        got = oracle.umma_expected(a.view(torch.int16).numpy().view(np.uint16),
                                   b.view(torch.int16).numpy().view(np.uint16), 16)
        assert np.array_equal(got, oracle.umma_reference_d(cg, 64, 16))


def test_reference_mode_operands_golden():
    g = json.loads((GOLDEN / "gemm_reference_inputs.json").read_text())
    m, n, k, l = g["mnkl"]
    a, b = inputs.reference_mode_operands(m, n, k, l)
    assert a.float().flatten().tolist() == g["a"]
    assert b.float().flatten().tolist() == g["b"]
    # Integer-valued operands in {-2,-1,0,1}.
    assert set(torch.unique(a.float()).tolist()) <= {-2.0, -1.0, 0.0, 1.0}


def test_checksums_match_numpy_restatement():
    words = oracle.uniform_u32(10_000, seed=3)
    for stage_bytes, grid in ((4096, 7), (2048, 3), (8192, 13)):
        got = oracle.copy_checksums(words, stage_bytes, grid, passes=3)
        tiles = -(-words.size * 4 // stage_bytes)
        for g_ in range(grid):
            t0, t1 = g_ * tiles // grid, (g_ + 1) * tiles // grid
            x = int(np.bitwise_xor.reduce(words[t0 * stage_bytes // 4: t1 * stage_bytes // 4], initial=0))
            total = 0
            for p in range(3):
                r = p % 32
                total ^= ((x << r) | (x >> (32 - r))) & 0xFFFFFFFF if r else x
            assert got[g_] == total
        assert int(np.bitwise_xor.reduce(oracle.copy_checksums(words, stage_bytes, grid))) == oracle.xor_all(words)


def test_gemm_oracles_agree_small():
    a, b = inputs.baseline_mode_operands(64, 48, 96)
    small = oracle.gemm_ref_small(a.view(torch.int16).numpy().view(np.uint16),
                                  b.view(torch.int16).numpy().view(np.uint16))
    fp32 = oracle.gemm_reference_fp32(a, b).numpy()
    assert np.allclose(small, fp32, rtol=1e-5, atol=1e-4)
    bad, max_abs, _ = oracle.validate_elementwise(fp32, small)
    assert bad == 0 and max_abs < 1e-3
