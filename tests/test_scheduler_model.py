"""CPU model of the GEMM tile scheduler (data-parallel tiles + split tail),
restating next_item and the host's choice of the split factor in
gemm_sm100.cu, checked for the properties the kernel relies on: every
(tile, k-block) is computed exactly once, all parts of a tail tile run in
the same (single) round on distinct clusters, and every part owns a column
slice that is a multiple of the epilogue chunk."""
import pytest


def choose(T, KB, P, BN=256):
    full, rem = divmod(T, P)
    waves = full + (1 if rem else 0)
    if not rem or KB < 48 or T / (waves * P) >= 0.95:
        return T, 0
    s = min(P // rem, 4)
    if s == 3:
        s = 2
    if s >= 2 and BN // s >= 64:
        return full * P, s
    return T, 0


def items(c, T, KB, P, dp_tiles, parts):
    n_dp = (dp_tiles - 1 - c) // P + 1 if c < dp_tiles else 0
    out = [(c + i * P, 0, KB, -1) for i in range(n_dp)]
    if parts and c < (T - dp_tiles) * parts:
        t, j = divmod(c, parts)
        out.append((dp_tiles + t, j * KB // parts, (j + 1) * KB // parts, j))
    return out


@pytest.mark.parametrize("T,KB,P", [(256, 64, 74), (128, 64, 74), (4, 64, 74), (1024, 128, 74), (300, 9, 74),
                                    (75, 8, 74), (37, 1000, 74), (140, 16, 148), (3, 8, 2), (256, 16, 74),
                                    (20, 64, 74), (256, 16, 74)])
def test_schedule_covers_everything_once(T, KB, P):
    dp_tiles, parts = choose(T, KB, P)
    seen = set()
    owners = {}
    for c in range(P):
        its = items(c, T, KB, P, dp_tiles, parts)
        assert sum(1 for it in its if it[3] >= 0) <= 1  # at most one part per cluster
        for tile, kb0, kb1, part in its:
            assert kb1 > kb0
            for kb in range(kb0, kb1):
                assert (tile, kb) not in seen
                seen.add((tile, kb))
            if part >= 0:
                owners.setdefault(tile, set()).add(c)
    assert len(seen) == T * KB
    assert all(len(v) == parts for v in owners.values())
    if parts:
        assert (256 // parts) % 64 == 0


def test_headline_shapes():
    assert choose(256, 64, 74) == (222, 2)      # 4096^3: 34-tile tail split in 2
    assert choose(128, 64, 74) == (128, 0)      # 16384x512: tail 73% full, kept whole
    assert choose(1024, 128, 74) == (1024, 0)   # 8192^3: last wave 84% full
    assert choose(20, 64, 74) == (0, 2)         # 20 tiles < 74 clusters: split in 2... (P//20 = 3 -> 2)
