"""CPU restatement of the split-KV tile schedule (get_mla_metadata, K2).

TEST INFRASTRUCTURE ONLY (used by tests/ to check the device scheduler).

The reference has no scheduler (csrc/api/sparse_decode.cpp:147-158 fakes
num_sm_parts = 1); the record format is its DecodingSchedMeta
(csrc/common/params.h:17-32).  Plan: query row r = b*s_q + s owns
ceil(len_main/128) + ceil(len_extra/128) tiles, len_main =
max(min(topk_length[b], topk), 1) (tests/reference.py:107-109),
len_extra = clamp(extra_topk_length[b], 0, extra_topk).

* cluster size C >= 2 (chosen by the library from the shapes, the layout
  and the device: dsv4b_plan_cluster_size): row r owns parts r*C + j,
  j < C, with tiles [floor(j*n/C), floor((j+1)*n/C)) (empty ranges give the
  empty record); num_splits = [0, 1, ..., R] since each cluster merges its
  row itself.
* R <= num_sm_parts (row-aligned): t* = the smallest per-part tile cap with
  sum_r ceil(tiles_r / t*) <= num_sm_parts; row r gets k_r =
  ceil(tiles_r / t*) consecutive parts and its part j covers tiles
  [floor(j*n/k), floor((j+1)*n/k)).  No part spans two rows.
* otherwise (contiguous): the concatenated tile list is cut into
  P = min(num_sm_parts, T) ranges [floor(p*T/P), floor((p+1)*T/P)).

Parts past the last planned one get the empty record [0, -1, 0...].
"""
from __future__ import annotations

from typing import List, Optional, Sequence, Tuple

TILE = 128


def row_tiles(b: int, s_q: int, topk: int, topk_length: Optional[Sequence[int]],
              extra_topk: int = 0, extra_topk_length: Optional[Sequence[int]] = None,
              has_extra: bool = False) -> List[int]:
    out = []
    for bi in range(b):
        ln = topk if topk_length is None else min(topk, int(topk_length[bi]))
        ln = max(ln, 1)
        el = 0
        if has_extra:
            el = extra_topk if extra_topk_length is None else min(extra_topk, int(extra_topk_length[bi]))
            el = max(el, 0)
        n = -(-ln // TILE) + -(-el // TILE)
        out.extend([n] * s_q)
    return out


EMPTY = [0, -1, 0, 0, 0, 0, 0, 0]


def _plan_row_aligned(tiles: Sequence[int], num_sm_parts: int):
    R = len(tiles)
    lo, hi = 1, max(tiles)
    while lo < hi:
        mid = (lo + hi) // 2
        if sum(-(-n // mid) for n in tiles) <= num_sm_parts:
            hi = mid
        else:
            lo = mid + 1
    k = [-(-n // lo) for n in tiles]
    ns = [0]
    for kr in k:
        ns.append(ns[-1] + kr)
    recs = []
    for r in range(R):
        n = tiles[r]
        for j in range(k[r]):
            bb, eb = j * n // k[r], (j + 1) * n // k[r]
            recs.append([r, r, bb, eb, ns[r] + j, int(bb > 0), int(eb < n), eb - bb])
    recs += [list(EMPTY) for _ in range(num_sm_parts - len(recs))]
    return recs, ns


def _plan_cluster(tiles: Sequence[int], num_sm_parts: int, c: int):
    R = len(tiles)
    recs = []
    for part in range(num_sm_parts):
        r, j = divmod(part, c)
        rec = list(EMPTY)
        if r < R:
            n = tiles[r]
            bb, eb = j * n // c, (j + 1) * n // c
            if eb > bb:
                rec = [r, r, bb, eb, r, int(bb > 0), int(eb < n), eb - bb]
        recs.append(rec)
    return recs, list(range(R + 1))


def plan(tiles: Sequence[int], num_sm_parts: int,
         cluster: int = 1) -> Tuple[List[List[int]], List[int]]:
    """Returns (records [num_sm_parts][8], num_splits [R+1])."""
    R = len(tiles)
    if cluster > 1:
        assert R * cluster <= num_sm_parts
        return _plan_cluster(tiles, num_sm_parts, cluster)
    if R <= num_sm_parts:
        return _plan_row_aligned(tiles, num_sm_parts)
    off = [0]
    for n in tiles:
        off.append(off[-1] + n)
    T = off[-1]
    P = min(num_sm_parts, T)

    def part_of(t):
        return ((t + 1) * P + T - 1) // T - 1

    nsplit = [part_of(off[r + 1] - 1) - part_of(off[r]) + 1 for r in range(R)]
    ns = [0]
    for n in nsplit:
        ns.append(ns[-1] + n)

    def row_of(x):
        lo, hi = 0, R - 1
        while lo < hi:
            mid = (lo + hi + 1) // 2
            if off[mid] <= x:
                lo = mid
            else:
                hi = mid - 1
        return lo

    recs = []
    for p in range(num_sm_parts):
        if p >= P:
            recs.append(list(EMPTY))
            continue
        t0, t1 = p * T // P, (p + 1) * T // P
        br, er = row_of(t0), row_of(t1 - 1)
        bb, eb = t0 - off[br], t1 - off[er]
        recs.append([br, er, bb, eb, ns[br] + (p - part_of(off[br])),
                     int(bb > 0), int(off[er] + eb < off[er + 1]), t1 - t0])
    return recs, ns
