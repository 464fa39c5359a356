"""Work-unit decomposition of the swap-AB grouped GEMMs (csrc/gemm_sm100.cu,
decode_tile and the per-expert K splits), restated on the CPU.

Units run expert by expert (prefix over experts of tiles x row blocks x that
expert's K slices); inside an expert the token tile varies fastest, then the
K slice, then the row block; slice ks of `splits` covers K blocks
[ks K / splits, (ks + 1) K / splits). The last `tail` active experts use
`tail_splits`. For random per-expert counts the test checks that every
(expert, token tile, row block) gets every K block exactly once, so the
fp32 partial sums add up to the whole product whatever the splits.
"""
from __future__ import annotations

import random

import pytest

BN = 16


def expert_splits(counts, splits, tail_splits, tail):
    active = [e for e, c in enumerate(counts) if c > 0]
    last = set(active[-tail:]) if tail > 0 and tail_splits > splits else set()
    return [tail_splits if e in last else splits for e in range(len(counts))]


def units(counts, row_blocks, splits_e):
    pre = [0]
    for e, c in enumerate(counts):
        pre.append(pre[-1] + ((c + BN - 1) // BN) * row_blocks * splits_e[e])
    return pre


def decode_tile(u, pre, counts, splits_e, k_blocks):
    e = 0
    while pre[e + 1] <= u:
        e += 1
    nt = (counts[e] + BN - 1) // BN
    local = u - pre[e]
    tt = local % nt
    local //= nt
    ks = local % splits_e[e]
    blk = local // splits_e[e]
    return e, tt, blk, ks * k_blocks // splits_e[e], (ks + 1) * k_blocks // splits_e[e]


@pytest.mark.parametrize("k_blocks,row_blocks,splits,tail_splits", [(56, 16, 4, 8), (56, 16, 8, 8),
                                                                    (16, 28, 2, 4), (16, 28, 2, 0)])
def test_every_k_block_once(k_blocks, row_blocks, splits, tail_splits):
    rng = random.Random(k_blocks * 100 + splits)
    for _ in range(50):
        counts = [rng.choice([0, 0, 1, 3, 16, 17, 40, 64]) for _ in range(32)]
        splits_e = expert_splits(counts, splits, tail_splits, 2)
        pre = units(counts, row_blocks, splits_e)
        seen = {}
        for u in range(pre[-1]):
            e, tt, blk, kb0, kb1 = decode_tile(u, pre, counts, splits_e, k_blocks)
            assert counts[e] > 0 and 0 <= tt < (counts[e] + BN - 1) // BN and 0 <= blk < row_blocks
            assert 0 <= kb0 < kb1 <= k_blocks
            for kb in range(kb0, kb1):
                key = (e, tt, blk, kb)
                assert key not in seen, key
                seen[key] = u
        expect = sum(((c + BN - 1) // BN) * row_blocks * k_blocks for c in counts)
        assert len(seen) == expect
