"""CPU checks of the split-KV schedule restatement (oracle/schedule_oracle.py).

The device scheduler (dsv4b_get_mla_metadata) is compared record for record
with this restatement by the GPU tests; here the restatement itself is held
to the invariants the decode and combine kernels rely on:
every tile of every query row is covered by exactly one part, in order;
the split indices of a row are consecutive and match num_splits; the
split flags agree with the covered range; parts past the plan are empty.
"""
import random

import pytest

from oracle import schedule_oracle as SO


def _check_plan(tiles, parts, cluster=1):
    recs, ns = SO.plan(tiles, parts, cluster)
    R = len(tiles)
    assert len(recs) == parts and len(ns) == R + 1 and ns[0] == 0
    covered = {r: [] for r in range(R)}   # row -> [(begin, end, split)]
    for rec in recs:
        br, er, bb, eb, split, first_sp, last_sp, nt = rec
        if er < br:
            assert rec == SO.EMPTY
            continue
        total = 0
        for r in range(br, er + 1):
            lo = bb if r == br else 0
            hi = eb if r == er else tiles[r]
            assert 0 <= lo < hi <= tiles[r], rec
            s = split if r == br else ns[r]
            covered[r].append((lo, hi, s))
            total += hi - lo
        assert nt == total
        assert first_sp == int(bb > 0)
        assert last_sp == int(eb < tiles[er])
    for r in range(R):
        segs = sorted(covered[r])
        assert segs[0][0] == 0 and segs[-1][1] == tiles[r]
        for (a0, a1, _), (b0, _, _) in zip(segs, segs[1:]):
            assert a1 == b0
        # a row covered by k parts owns splits ns[r] .. ns[r]+k-1
        if cluster == 1:
            assert ns[r + 1] - ns[r] == len(segs)
        firsts = [s for lo, _, s in segs]
        if cluster == 1:
            assert firsts == list(range(ns[r], ns[r + 1])) or len(segs) == 1
    return recs, ns


@pytest.mark.parametrize("seed", range(40))
def test_random_plans_cover_every_tile_once(seed):
    rng = random.Random(seed)
    R = rng.choice([1, 2, 3, 7, 32, 64, 150, 300])
    tiles = [rng.randint(1, 20) for _ in range(R)]
    parts = rng.choice([1, 7, 74, 148, 296])
    _check_plan(tiles, parts)


def test_row_aligned_when_rows_fit():
    # config-1 shape: 32 rows x 16 tiles on 148 parts -> cap 4, 128 parts
    recs, ns = _check_plan([16] * 32, 148)
    live = [r for r in recs if r[1] >= r[0]]
    assert len(live) == 128
    assert all(r[0] == r[1] and r[7] == 4 for r in live)
    assert ns[-1] == 128


def test_row_aligned_cap_is_minimal():
    tiles = [10, 3, 1, 7]
    recs, _ = _check_plan(tiles, 9)
    cap = max(r[7] for r in recs if r[1] >= r[0])
    assert sum(-(-n // cap) for n in tiles) <= 9
    assert sum(-(-n // (cap - 1)) for n in tiles) > 9


def test_contiguous_when_rows_exceed_parts():
    tiles = [2] * 10
    recs, ns = _check_plan(tiles, 4)
    assert [r[7] for r in recs] == [5, 5, 5, 5]
    assert any(r[0] != r[1] for r in recs)


def test_fewer_tiles_than_parts_leaves_empty_records():
    recs, ns = _check_plan([1, 1], 148)
    assert sum(1 for r in recs if r[1] >= r[0]) == 2
    assert ns == [0, 1, 2]


@pytest.mark.parametrize("cluster", [2, 4, 8])
def test_cluster_plan_keeps_rows_in_their_cluster(cluster):
    rng = random.Random(cluster)
    tiles = [rng.randint(1, 20) for _ in range(148 // cluster)]
    recs, ns = _check_plan(tiles, 148, cluster)
    assert ns == list(range(len(tiles) + 1))
    for part, rec in enumerate(recs):
        if rec[1] >= rec[0]:
            assert rec[0] == rec[1] == part // cluster
    # every rank gets floor or ceil of tiles / C
    for r, n in enumerate(tiles):
        got = [recs[r * cluster + j][7] for j in range(cluster)]
        assert sum(got) == n and max(got) - min(got) <= 1
