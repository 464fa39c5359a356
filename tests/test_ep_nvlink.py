"""Expert-parallel NVLink combine (moe_b200_ep_combine_shards) on 2-4 GPUs.

One process per GPU (up to four). In the first pass each rank owns one
32-expert shard (local_expert_offset = 32 * rank); in the second, two
shards each (offsets 64 * rank and 64 * rank + 32). The fused combine must
equal, bit for bit, the bf16 rounding of the fp32 sum of the shards' own
combine rows (read back from the workspaces and gathered; each rank's shards
summed in shard order, then those sums in rank order), agree
with an independent run of every shard within the operator's tolerance, be
identical on all ranks and leave the status words clear. The shared buffers
are plain cudaMalloc memory mapped through CUDA IPC (no multicast object),
and NCCL runs with NVLS off. Runs only where at least two GPUs are visible.
"""
import os
import socket
import sys

import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "flashinfer-bench-avengers_b200")

pytestmark = pytest.mark.gpu


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _shard_rows(ws, T):
    """A shard's fp32 combine rows, one per token (zeros without a local pick)."""
    import moe_host

    lay = moe_host.workspace_layout(T)
    y = ws[lay.y_acc: lay.y_acc + 4 * T * 7168].view(torch.float32).view(T, 7168)
    if T <= 64:   # decode plan: one row per token
        return y.clone()
    slot = ws[lay.tok_slot: lay.tok_slot + 4 * T].view(torch.int32).long()
    return torch.where((slot >= 0)[:, None], y[slot.clamp(min=0)], torch.zeros_like(y))


def _worker(rank: int, world: int, port: int, passes, results):
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    sys.path.insert(0, PKG)
    import torch.distributed as dist
    from datetime import timedelta

    import expert_parallel
    import moe_host
    import workloads

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60), device_id=dev)
    try:
        for spr, cases in passes:
            comb = expert_parallel.NvlinkCombiner(max(T for T, _ in cases), dev, shards_per_rank=spr)
            offsets = [32 * (rank * spr + s) for s in range(spr)]
            for T, variant in cases:
                inps = [workloads.make_inputs(T, 7, dev, variant, off, 2.5, weight_seed=100 + off // 32)
                        for off in offsets]
                tokens = {k: inps[0][k] for k in ("routing_logits", "routing_bias", "hidden_states",
                                                  "hidden_states_scale", "routed_scaling_factor")}
                shards = [(i["gemm1_weights"], i["gemm1_weights_scale"], i["gemm2_weights"],
                           i["gemm2_weights_scale"], off) for i, off in zip(inps, offsets)]
                fused = torch.empty(T, 7168, dtype=torch.bfloat16, device=dev)
                for _ in range(2):   # twice: the call counters must advance correctly
                    comb.forward_shards(tokens, shards, fused)
                torch.cuda.synchronize()
                status = comb.status()
                # exact reference: every shard's fp32 combine rows, each
                # rank's summed in shard order, those sums in rank order,
                # rounded once to bf16 (T <= 64 takes the flagged-line
                # protocol, larger T the staged one: both sum this way)
                mine = torch.stack([_shard_rows(ws, T) for ws in comb.workspaces])
                rows = [torch.empty_like(mine) for _ in range(world)]
                dist.all_gather(rows, mine)
                total = torch.zeros(T, 7168, dtype=torch.float32, device=dev)
                for q in range(world):
                    part = torch.zeros(T, 7168, dtype=torch.float32, device=dev)
                    for s in range(spr):
                        part = part + rows[q][s]
                    total = total + part
                exact = torch.equal(fused, total.to(torch.bfloat16))
                # the standard tolerance against an independent run of each shard
                ref = sum(moe_host.run(*workloads.as_args(i)).float() for i in inps)
                dist.all_reduce(ref)
                err = (fused.float() - ref).abs()
                within = float((err <= 1e-2 * ref.abs().max()).float().mean())
                other = fused.clone()
                dist.broadcast(other, src=0)
                results.put((rank, spr, T, variant, int(status), exact, within, torch.equal(fused, other),
                             float(ref.abs().max())))
            comb.close()
        torch.cuda.synchronize()
        dist.barrier()
    finally:
        dist.destroy_process_group()


def test_nvlink_combine_ranks():
    if not torch.cuda.is_available() or torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    world = min(torch.cuda.device_count(), 4)
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    results = ctx.Queue()
    # one shard per rank: decode plan (flagged lines, also with fewer tokens
    # than ranks: some own no row); compact combine rows; token-major GEMMs
    # (K split, compact rows). Two shards per rank: decode and token-major.
    passes = [(1, [(16, "uniform"), (64, "uniform"), (3, "uniform"), (200, "uniform"), (600, "uniform")]),
              (2, [(16, "uniform"), (600, "uniform")])]
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, passes, results)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=400)
    for p in procs:
        if p.is_alive():   # the kernels' waits are bounded; only a stuck host process is left here
            p.kill()
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    n = world * sum(len(c) for _, c in passes)
    got = [results.get(timeout=5) for _ in range(n)]
    for rank, spr, T, variant, status, exact, within, same, amax in got:
        assert status == 0, (rank, spr, T, status)
        assert exact, (rank, spr, T, variant)
        assert within >= 0.999, (rank, spr, T, variant, within)
        assert same, (rank, spr, T)
        assert amax > 0.0, (rank, spr, T)
