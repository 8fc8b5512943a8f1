"""CPU model of the GEMM tile scheduler (data-parallel tiles, then a narrow
tail or a stream-K region), restating sk_begin, next_item, the fix-up's
piece range and the host's choose_stream_k / plan_tail in gemm_sm100.cu,
checked for the properties the kernel relies on: the narrow tail's half
items cover each tail tile's two column halves once, one per cluster; every (tile, k-block) is computed exactly once; the pieces
of a stream-K tile belong to consecutive clusters, so the last one can walk
them in k order; every piece's workspace slot (cluster + tile) is distinct
and inside the plan's 2 P slots (two per cluster: its first and last tile); no cluster ever waits for
another (nothing to check: the protocol has no wait)."""
import pytest

SNAP, OVH = 4, 17.0
EFF128 = 0.66
NARROW_RATE = 0.5 * 0.907 / EFF128


def sk_begin(c, P, sk_tiles, kb, snap):
    total = sk_tiles * kb
    if c <= 0:
        return 0
    if c >= P:
        return total
    x = (c * total) // P
    off = x % kb
    if off < snap:
        x -= off
    elif kb - off < snap:
        x += kb - off
    return x


def region_cost(P, sk_tiles, kb, snap, ovh):
    worst = 0.0
    for c in range(P):
        b0, b1 = sk_begin(c, P, sk_tiles, kb, snap), sk_begin(c + 1, P, sk_tiles, kb, snap)
        if b0 >= b1:
            continue
        cost = float(b1 - b0)
        t = b0 // kb
        while t * kb < b1:
            if b0 > t * kb or b1 < (t + 1) * kb:
                cost += ovh
            t += 1
        worst = max(worst, cost)
    return worst


def choose_stream_k(T, P, kb, snap=SNAP, ovh=OVH, force=False):
    snap = max(0, min(snap, kb // 4))
    full, rem = divmod(T, P)
    best = (0, float(full + (1 if rem else 0)) * kb)
    if rem == 0:
        return best[0], snap
    sk = (rem, full * kb + region_cost(P, rem, kb, snap, ovh))
    if full >= 1:
        c2 = (full - 1) * kb + region_cost(P, rem + P, kb, snap, ovh)
        if c2 < sk[1]:
            sk = (rem + P, c2)
    if force or sk[1] < 0.97 * best[1]:
        best = sk
    return best[0], snap


def plan_tail(T, P, kb, allow_narrow=True, narrow_mode=-1, sk_mode=-1, snap=SNAP, ovh=OVH):
    """(narrow_tiles, sk_tiles) as plan_tail chooses them."""
    snap = max(0, min(snap, kb // 4))
    full, rem = divmod(T, P)
    best = (0, 0, float(full + (1 if rem else 0)) * kb)
    if rem == 0:
        return best[:2]
    whole = best[2]
    if allow_narrow and narrow_mode != 0 and 2 * rem <= P:
        nt = (rem, 0, full * kb + kb * NARROW_RATE)
        if narrow_mode == 1 or nt[2] < 0.97 * whole:
            best = nt
        if narrow_mode == 1:
            return best[:2]
    if sk_mode != 0:
        sk, _ = choose_stream_k(T, P, kb, snap, ovh, sk_mode == 1)
        if sk:
            full_sk = (T - sk) // P
            cost = full_sk * kb + region_cost(P, sk, kb, snap, ovh)
            if sk_mode == 1 or cost < best[2]:
                best = (0, sk, cost)
    return best[:2]


def narrow_items(c, T, KB, P, narrow):
    dp = T - narrow
    n_dp = (dp - 1 - c) // P + 1 if c < dp else 0
    out = [(c + i * P, -1) for i in range(n_dp)]
    if narrow and c < 2 * narrow:
        out.append((dp + c // 2, c % 2))
    return out


@pytest.mark.parametrize("T,P", [(256, 74), (32, 74), (37, 74), (111, 74), (1, 74), (3, 2), (150, 74)])
def test_narrow_tail_covers_each_half_once(T, P):
    narrow, _ = plan_tail(T, P, 64, narrow_mode=1)
    if narrow == 0:
        assert T % P == 0 or 2 * (T % P) > P
        return
    seen = set()
    for c in range(P):
        its = narrow_items(c, T, 64, P, narrow)
        assert sum(1 for _, h in its if h >= 0) <= 1
        for tile, half in its:
            for hh in ((0, 1) if half < 0 else (half,)):
                assert (tile, hh) not in seen
                seen.add((tile, hh))
    assert len(seen) == 2 * T


def test_tail_plans_of_the_headline_shapes():
    # 4096^3, 256 x 256 tiles: the 34-tile partial wave runs as 68 half tiles
    assert plan_tail(256, 74, 64) == (34, 0)
    # 54-tile partial waves do not fit 74 clusters as half tiles; stream-K's
    # measured fix-up cost makes whole tiles the plan
    assert plan_tail(128, 74, 64) == (0, 0)
    # a single long-K tile: stream-K over the clusters pays for its fix-up
    assert plan_tail(1, 74, 256, allow_narrow=False)[1] == 1


def items(c, T, KB, P, sk_tiles, snap):
    dp = T - sk_tiles
    n_dp = (dp - 1 - c) // P + 1 if c < dp else 0
    out = [(c + i * P, 0, KB, -1) for i in range(n_dp)]
    if sk_tiles:
        b0, b1 = sk_begin(c, P, sk_tiles, KB, snap), sk_begin(c + 1, P, sk_tiles, KB, snap)
        if b0 < b1:
            t = b0 // KB
            while t * KB < b1:
                t0 = t * KB
                kb0, kb1 = max(b0, t0) - t0, min(b1, t0 + KB) - t0
                out.append((dp + t, kb0, kb1, -1 if (kb0 == 0 and kb1 == KB) else 1))
                t += 1
    return out


def piece_range(c, t_local, P, sk_tiles, KB, snap):
    """The fix-up's walk: clusters c_first..c_last around the last piece c."""
    tile0 = t_local * KB
    cf = cl = c
    while cf > 0 and sk_begin(cf, P, sk_tiles, KB, snap) > tile0:
        cf -= 1
    while cl + 1 < P and sk_begin(cl + 1, P, sk_tiles, KB, snap) < tile0 + KB:
        cl += 1
    return [co for co in range(cf, cl + 1)
            if sk_begin(co, P, sk_tiles, KB, snap) < sk_begin(co + 1, P, sk_tiles, KB, snap)]


CASES = [(256, 64, 74), (128, 64, 74), (4, 64, 74), (1024, 128, 74), (300, 9, 74), (75, 8, 74), (37, 1000, 74),
         (140, 16, 148), (3, 8, 2), (256, 16, 74), (20, 64, 74), (32, 64, 74), (16, 64, 74), (76, 64, 74),
         (64, 64, 148), (2, 3, 74), (150, 64, 74), (33, 130, 74)]


@pytest.mark.parametrize("T,KB,P", CASES)
@pytest.mark.parametrize("force", [False, True])
def test_schedule_covers_everything_once(T, KB, P, force):
    sk_tiles, snap = choose_stream_k(T, P, KB, force=force)
    dp = T - sk_tiles
    assert 0 <= sk_tiles <= T and (sk_tiles == 0 or dp % P == 0)
    seen = set()
    pieces = {}
    slots = set()
    for c in range(P):
        for tile, kb0, kb1, part in items(c, T, KB, P, sk_tiles, snap):
            assert kb1 > kb0
            for kb in range(kb0, kb1):
                assert (tile, kb) not in seen
                seen.add((tile, kb))
            if part >= 0:
                t_local = tile - dp
                first = sk_begin(c, P, sk_tiles, KB, snap) // KB == t_local
                slot = 2 * c + (0 if first else 1)
                assert slot not in slots and 0 <= slot < 2 * P
                slots.add(slot)
                pieces.setdefault(t_local, []).append((c, kb0, kb1))
    assert len(seen) == T * KB
    for t_local, ps in pieces.items():
        ps.sort(key=lambda x: x[1])
        # consecutive clusters, contiguous k ranges from 0 to KB
        assert ps[0][1] == 0 and ps[-1][2] == KB
        assert all(a[2] == b[1] for a, b in zip(ps, ps[1:]))
        owners = [p[0] for p in ps]
        assert owners == sorted(owners)
        # whichever piece finishes last walks exactly these owners in k order
        for c in owners:
            assert piece_range(c, t_local, P, sk_tiles, KB, snap) == owners


def test_headline_shapes():
    """choose_stream_k's region choice with a small per-piece cost."""
    # 4096^3 on 74 clusters of 256x256 tiles: 34-tile tail, stream-K over it
    assert choose_stream_k(256, 74, 64, ovh=4.0)[0] == 34
    # 8192^3 (1024 tiles): the 62-tile tail leaves the last wave 84 % full;
    # balancing it saves under 3 %, so whole tiles stay
    assert choose_stream_k(1024, 74, 128, ovh=4.0)[0] == 0
    # a 512-row shard of 4096^3 (32 tiles < 74 clusters): all stream-K
    assert choose_stream_k(32, 74, 64, ovh=4.0)[0] == 32
    # whole waves: nothing to balance
    assert choose_stream_k(148, 74, 64, ovh=4.0)[0] == 0


def test_stream_k_balances_sub_wave_shards():
    """The slowest cluster of a 32-tile, 64-k-block problem on 74 clusters
    carries about 32 * 64 / 74 k-blocks plus its fix-up, not a whole tile."""
    sk_tiles, snap = choose_stream_k(32, 74, 64)
    assert region_cost(74, sk_tiles, 64, snap, OVH) <= 32 * 64 / 74 + 2 * OVH + SNAP
