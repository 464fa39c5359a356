"""Index arithmetic of the expert-parallel combine's flagged-line protocol
(csrc/ep_combine.cu, calls of at most 64 tokens), restated on the CPU.

Rank q of W owns token rows [T q / W, T (q + 1) / W). In step A every rank
stores, for each row another rank owns, one fp32 row into the owner's
receive slot for it: row `src * ceil(T / W) + (t - first row of the owner)`
of a 72-row buffer (64 + 8 rows). The test checks, for every T <= 64 and
W in {2, 4, 8}, that those rows stay inside the buffer, that no two
(source, row) pairs share one, that every rank reads back exactly the rows
sent to it, and that the rank-order sum it forms equals the two-level sum
(each rank's shards, then the ranks) that the GPU tests compare against.
"""
from __future__ import annotations

import pytest
import torch

PART_ROWS = 64 + 8


def row_lo(q: int, T: int, W: int) -> int:
    return T * q // W


def row_owner(t: int, T: int, W: int) -> int:
    q = t * W // T
    while row_lo(q + 1, T, W) <= t:
        q += 1
    while row_lo(q, T, W) > t:
        q -= 1
    return q


@pytest.mark.parametrize("W", [2, 4, 8])
def test_receive_slots_in_range_and_disjoint(W):
    for T in range(1, 65):
        slot_rows = (T + W - 1) // W
        used = {}
        for src in range(W):
            mlo, mhi = row_lo(src, T, W), row_lo(src + 1, T, W)
            nmine = mhi - mlo
            for r in range(T - nmine):                      # step A's rows, in kernel order
                t = r if r < mlo else r + nmine
                q = row_owner(t, T, W)
                assert q != src and row_lo(q, T, W) <= t < row_lo(q + 1, T, W)
                dst = src * slot_rows + (t - row_lo(q, T, W))
                assert 0 <= dst < PART_ROWS, (T, W, src, t, dst)
                key = (q, dst)
                assert key not in used, (T, W, key, used.get(key), (src, t))
                used[key] = (src, t)
        # step B: owner q reads slot r * slot_rows + rr for each row rr of its own
        for q in range(W):
            mlo, mhi = row_lo(q, T, W), row_lo(q + 1, T, W)
            for rr in range(mhi - mlo):
                for r in range(W):
                    if r != q:
                        assert used[(q, r * slot_rows + rr)] == (r, mlo + rr)


def test_rank_order_sum_matches_two_level_sum():
    g = torch.Generator().manual_seed(5)
    W, S, T = 4, 2, 7
    shards = torch.randn(W, S, T, 16, generator=g)
    shards[1, 0, 3] = 0.0   # a row without a pick on that shard
    ref = torch.zeros(T, 16)
    for q in range(W):
        part = torch.zeros(T, 16)
        for s in range(S):
            part = part + shards[q, s]
        ref = ref + part
    # the protocol: each rank's partial (its shards from +0.0), the owner adds
    # the ranks' partials in rank order from +0.0
    partial = [torch.zeros(T, 16) for _ in range(W)]
    for q in range(W):
        for s in range(S):
            partial[q] = partial[q] + shards[q, s]
    out = torch.zeros(T, 16)
    for t in range(T):
        acc = torch.zeros(16)
        for r in range(W):
            acc = acc + partial[r][t]
        out[t] = acc
    assert torch.equal(out, ref)
