"""Expert-parallel combine on CPU: two gloo ranks, each owning four of the
eight 32-expert shards, must reproduce the single-process sum over all
shards. The per-shard layer is the CPU oracle (host logic under test is
the shard assignment and the cross-rank reduction)."""
from __future__ import annotations

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import expert_parallel
import moe_oracle
import workloads

T = 2
SEED = 4


def _shard_weights(offsets, active_by_offset):
    out = {}
    for off in offsets:
        inp = workloads.make_inputs(T, SEED, "cpu", "uniform", off, 2.5, experts=active_by_offset[off],
                                    weight_seed=SEED + 100 + off)
        out[off] = (inp["gemm1_weights"], inp["gemm1_weights_scale"], inp["gemm2_weights"],
                    inp["gemm2_weights_scale"])
    return out


def _active(r):
    return {off: moe_oracle.active_local_experts(r["routing_logits"], r["routing_bias"], 2.5, off)
            for off in range(0, 256, 32)}


def _layer(*args):
    return moe_oracle.moe_forward(*args, return_fp32=True)


def _worker(rank, world, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        torch.set_num_threads(2)
        r = workloads.make_routing_inputs(T, SEED)
        hs, sc = workloads.make_hidden(T, SEED)
        tok = dict(r, hidden_states=hs, hidden_states_scale=sc, routed_scaling_factor=2.5)
        offs = expert_parallel.shard_offsets(world, rank)
        out = expert_parallel.ep_forward(_layer, tok, _shard_weights(offs, _active(r)), dist.group.WORLD)
        q.put((rank, out.view(torch.int16).numpy().tobytes()))
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_shard_offsets():
    assert expert_parallel.shard_offsets(1, 0) == list(range(0, 256, 32))
    assert expert_parallel.shard_offsets(2, 1) == [128, 160, 192, 224]
    assert expert_parallel.shard_offsets(8, 3) == [96]
    all_offsets = sorted(o for r in range(4) for o in expert_parallel.shard_offsets(4, r))
    assert all_offsets == list(range(0, 256, 32))
    with pytest.raises(ValueError):
        expert_parallel.shard_offsets(3, 0)


def test_two_rank_combine_matches_single_process():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=600) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert results[0] == results[1]
    # Expected: each rank sums its four shards in fp32, then the two rank
    # partials are added -- the same grouping as the distributed run.
    r = workloads.make_routing_inputs(T, SEED)
    hs, sc = workloads.make_hidden(T, SEED)
    tok = dict(r, hidden_states=hs, hidden_states_scale=sc, routed_scaling_factor=2.5)
    weights = _shard_weights(range(0, 256, 32), _active(r))
    halves = []
    for rank in range(2):
        acc = None
        for off in expert_parallel.shard_offsets(2, rank):
            w13, s13, w2, s2 = weights[off]
            part = _layer(tok["routing_logits"], tok["routing_bias"], hs, sc, w13, s13, w2, s2, off, 2.5)
            acc = part if acc is None else acc + part
        halves.append(acc)
    expected = (halves[0] + halves[1]).to(torch.bfloat16)
    got = torch.frombuffer(bytearray(results[0]), dtype=torch.int16).view(T, 7168)
    assert torch.equal(got, expected.view(torch.int16))
    # and the single-process helper agrees to within one bf16 rounding
    single = expert_parallel.ep_forward(_layer, tok, weights, None).float()
    assert float((single - expected.float()).abs().max()) <= 2.0 ** -7 * float(expected.float().abs().max())
