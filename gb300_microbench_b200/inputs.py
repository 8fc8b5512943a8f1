"""Seeded input generators for both input modes.

Reference mode (campaign-compatible CSVs): the reference draws GEMM operands
with ``torch.manual_seed(1111)`` and the CuTe DSL helper
``cutlass.torch.matrix`` (called by the upstream ``create_tensors``,
dense_gemm.py:1498-1506, as pinned by gemm_comparison.py:941-1031): an int32
tensor of shape (L, rows, K) filled by ``random_(-2, 2)`` (values -2..1),
converted to float and then to BF16, A first, then B. :func:`reference_mode_operands`
restates that draw without the helper.

Baseline mode: A (M, K) then B (N, K) from N(0, 1) with
``torch.Generator().manual_seed(0)`` on the CPU, cast to BF16.
"""
from __future__ import annotations

import torch

REFERENCE_SEED = 1111
BASELINE_SEED = 0


def reference_mode_operands(m: int, n: int, k: int, l: int = 1) -> tuple[torch.Tensor, torch.Tensor]:
    """(A, B) on the CPU as (L, M, K) and (L, N, K) BF16, integer-valued."""
    g = torch.Generator().manual_seed(REFERENCE_SEED)
    a = torch.empty(l, m, k, dtype=torch.int32).random_(-2, 2, generator=g).to(torch.float32)
    b = torch.empty(l, n, k, dtype=torch.int32).random_(-2, 2, generator=g).to(torch.float32)
    return a.to(torch.bfloat16), b.to(torch.bfloat16)


def baseline_mode_operands(m: int, n: int, k: int, seed: int = BASELINE_SEED) -> tuple[torch.Tensor, torch.Tensor]:
    """(A, B) on the CPU as (M, K) and (N, K) BF16 drawn from N(0, 1)."""
    g = torch.Generator().manual_seed(seed)
    a = torch.randn(m, k, generator=g, dtype=torch.float32).to(torch.bfloat16)
    b = torch.randn(n, k, generator=g, dtype=torch.float32).to(torch.bfloat16)
    return a, b


def umma_pattern_operands(cta_group: int, n: int) -> tuple[torch.Tensor, torch.Tensor]:
    """The reference's exact UMMA operands (umma_1sm.cu:394-401,
    umma_2sm.cu:495-509): A[r, k] = ((r + 3k) mod 7) - 3 over the global row
    r, B[c, k] = ((2k + c) mod 5) - 2 (stored N x K)."""
    m = 128 * cta_group
    r = torch.arange(m).view(-1, 1)
    kk = torch.arange(16).view(1, -1)
    a = ((r + 3 * kk) % 7 - 3).to(torch.bfloat16)
    c = torch.arange(n).view(-1, 1)
    b = ((2 * kk + c) % 5 - 2).to(torch.bfloat16)
    return a, b


def umma_random_operands(cta_group: int, n: int, seed: int = BASELINE_SEED) -> tuple[torch.Tensor, torch.Tensor]:
    """Baseline-mode UMMA operands: N(0, 1) BF16 from a seeded generator."""
    g = torch.Generator().manual_seed(seed)
    a = torch.randn(128 * cta_group, 16, generator=g).to(torch.bfloat16)
    b = torch.randn(n, 16, generator=g).to(torch.bfloat16)
    return a, b
