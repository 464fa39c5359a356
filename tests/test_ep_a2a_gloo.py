"""Token-parallel expert parallelism on CPU: two gloo ranks with different
tokens, each owning four 32-expert shards, run the all-to-all protocol the
library's kernels implement -- per-destination numbering of the tokens that
have picks there (moe_oracle.a2a_plan), the exchange of the count matrix,
receive slabs of one row per (token, destination) in (source rank, token)
order carrying the token's picks on that destination, the shards run on
their slab rows with those picks, and each token's output as the sum of its
rows' results (each rank's shards in shard order, then the ranks in rank
order) -- with the CPU oracle as the layer. Each rank's result must equal
the single-process restatement (moe_oracle.token_parallel_forward) bit for
bit and the sum over all 8 shards of the ordinary layer on the rank's own
tokens within fp32 rounding."""
from __future__ import annotations

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import moe_oracle
import workloads

WORLD = 2
SHARDS = 4
TOKENS = (3, 2)     # a different batch on each rank


def _tokens(rank: int) -> dict:
    T = TOKENS[rank]
    r = workloads.make_routing_inputs(T, 60 + rank)
    hs, sc = workloads.make_hidden(T, 60 + rank)
    return dict(r, hidden_states=hs, hidden_states_scale=sc, routed_scaling_factor=2.5)


def _shard_weights(needed: dict) -> dict:
    """offset -> (w13, s13, w2, s2) as per-expert lists, only the experts any
    token picks materialised (the oracle indexes them by local id)."""
    out = {}
    for off in range(0, 256, 32):
        w13, s13, w2, s2 = [None] * 32, [None] * 32, [None] * 32, [None] * 32
        for le in needed.get(off, ()):
            w13[le], s13[le], w2[le], s2[le] = workloads.make_expert_weights(200 + off // 32, le)
        out[off] = (w13, s13, w2, s2)
    return out


def _needed(all_tokens) -> dict:
    need = {}
    for t in all_tokens:
        idx, _ = moe_oracle.route(t["routing_logits"], t["routing_bias"], 2.5)
        for e in idx.flatten().tolist():
            need.setdefault(e // 32 * 32, set()).add(e % 32)
    return need


def _worker(rank, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=WORLD)
    try:
        torch.set_num_threads(2)
        all_tokens = [_tokens(r) for r in range(WORLD)]
        mine = all_tokens[rank]
        weights = _shard_weights(_needed(all_tokens))
        idx, w = moe_oracle.route(mine["routing_logits"], mine["routing_bias"], 2.5)
        slot, counts = moe_oracle.a2a_plan(idx, WORLD, SHARDS)
        # the count matrix: every rank's row
        rows = [torch.zeros(WORLD, dtype=torch.int64) for _ in range(WORLD)]
        dist.all_gather(rows, counts)
        M = torch.stack(rows)
        # dispatch: wire format of one (token, destination) row = (token row,
        # 56 scales, its 8 picks with those on the destination kept)
        outgoing = [[] for _ in range(WORLD)]
        for t in range(idx.shape[0]):
            for d in range(WORLD):
                if int(slot[t, d]) < 0:
                    continue
                ids, ws = moe_oracle.a2a_row_picks(idx, w, t, d, SHARDS)
                # e4m3 rows travel as their bytes (pickling keeps plain dtypes)
                outgoing[d].append((int(slot[t, d]), t, mine["hidden_states"][t].view(torch.uint8).clone(),
                                    mine["hidden_states_scale"][:, t].clone(), ids, ws))
        sent = [None] * WORLD
        dist.all_gather_object(sent, outgoing)
        slab = [None] * int(M[:, rank].sum())
        for src in range(WORLD):
            for s_, t, row, sc, ids, ws in sent[src][rank]:
                slab[moe_oracle.a2a_slab(src, M, rank) + s_] = (src, t, row, sc, ids, ws)
        assert all(x is not None for x in slab)
        # this rank's shards on its slab rows, the rows' picks given
        hs = torch.stack([x[2] for x in slab]).view(torch.float8_e4m3fn)
        sc = torch.stack([x[3] for x in slab], dim=1)
        gi = torch.stack([x[4] for x in slab])
        gw = torch.stack([x[5] for x in slab])
        back = {}
        for s in range(SHARDS):
            off = 32 * (rank * SHARDS + s)
            y = moe_oracle.moe_forward(None, None, hs, sc, *weights[off], off, 1.0, return_fp32=True, given=(gi, gw))
            for j, x in enumerate(slab):
                back[(x[0], x[1], rank, s)] = y[j]
        # combine: each token's rows, each rank's shards in shard order, then
        # the ranks in rank order
        gathered = [None] * WORLD
        dist.all_gather_object(gathered, back)
        out = torch.zeros(idx.shape[0], 7168)
        for t in range(idx.shape[0]):
            for d in range(WORLD):
                part = torch.zeros(7168)
                for s in range(SHARDS):
                    if (rank, t, d, s) in gathered[d]:
                        part = part + gathered[d][(rank, t, d, s)]
                out[t] = out[t] + part
        q.put((rank, out.numpy().tobytes(), M.numpy().tobytes()))
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_token_parallel_protocol_on_gloo():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, port, q)) for r in range(WORLD)]
    for p in procs:
        p.start()
    import queue
    import time

    got = {}
    deadline = time.time() + 600
    while len(got) < WORLD and time.time() < deadline:
        try:
            rank, out, m = q.get(timeout=2)
            got[rank] = (torch.frombuffer(bytearray(out), dtype=torch.float32).view(TOKENS[rank], 7168), m)
        except queue.Empty:
            if any(p.exitcode not in (None, 0) for p in procs):
                break
    for p in procs:
        p.join(timeout=60)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    assert len(got) == WORLD
    assert got[0][1] == got[1][1], "the ranks saw different count matrices"
    all_tokens = [_tokens(r) for r in range(WORLD)]
    weights = _shard_weights(_needed(all_tokens))
    ref, slabs = moe_oracle.token_parallel_forward(all_tokens, weights, WORLD)
    # one row per (token, rank it has picks on): at most 4 ranks (4 groups)
    dests = 0
    for t_in in all_tokens:
        idx, _ = moe_oracle.route(t_in["routing_logits"], t_in["routing_bias"], 2.5)
        dests += int((torch.nn.functional.one_hot(moe_oracle.a2a_dest(idx, SHARDS), WORLD).sum(1) > 0).sum())
    assert sum(len(s) for s in slabs) == dests
    for r in range(WORLD):
        assert torch.equal(got[r][0], ref[r])
        # the same layer as expert parallelism on the rank's own tokens: the
        # sum over the 8 shards (another summation order, so fp32 rounding)
        t = all_tokens[r]
        ep = sum(moe_oracle.moe_forward(t["routing_logits"], t["routing_bias"], t["hidden_states"],
                                        t["hidden_states_scale"], *weights[off], off, 2.5, return_fp32=True)
                 for off in range(0, 256, 32))
        assert float((got[r][0] - ep).abs().max()) <= 1e-5 * float(ep.abs().max())
