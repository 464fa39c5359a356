"""Expert-parallel NVLink combine (moe_b200_ep_combine) on 2-4 GPUs.

One process per GPU (up to four), each owning a different 32-expert shard
(local_expert_offset = 32 * rank) of the same tokens. The fused combine must
equal, bit for bit, the bf16 rounding of the fp32 sum in rank order of the
ranks' own combine rows (read back from the workspaces and gathered), agree
with an independent run of every shard within the operator's tolerance, be
identical on all ranks and leave the status word clear. Runs only where at
least two GPUs are visible.
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


def _worker(rank: int, world: int, port: int, cases, results):
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
        comb = expert_parallel.NvlinkCombiner(max(T for T, _ in cases), dev)
        for T, variant in cases:
            inp = workloads.make_inputs(T, 7, dev, variant, 32 * rank, 2.5, weight_seed=100 + rank)
            tokens = {k: inp[k] for k in ("routing_logits", "routing_bias", "hidden_states", "hidden_states_scale",
                                          "routed_scaling_factor")}
            fused = torch.empty(T, 7168, dtype=torch.bfloat16, device=dev)
            for _ in range(2):   # twice: the call counters must advance correctly
                comb.forward(tokens, inp["gemm1_weights"], inp["gemm1_weights_scale"], inp["gemm2_weights"],
                             inp["gemm2_weights_scale"], 32 * rank, fused)
            torch.cuda.synchronize()
            status = moe_host.read_status(comb.workspace)
            # exact reference: this rank's fp32 combine rows (per token), summed
            # over the ranks in fp32, rounded once to bf16
            lay = moe_host.workspace_layout(T)
            ws = comb.workspace
            y = ws[lay.y_acc: lay.y_acc + 4 * T * 7168].view(torch.float32).view(T, 7168)
            if T <= 64:   # decode plan: one row per token
                full = y.clone()
            else:
                slot = ws[lay.tok_slot: lay.tok_slot + 4 * T].view(torch.int32).long()
                full = torch.where((slot >= 0)[:, None], y[slot.clamp(min=0)], torch.zeros_like(y))
            rows = [torch.empty_like(full) for _ in range(world)]
            dist.all_gather(rows, full)
            total = torch.zeros_like(full)
            for q in range(world):   # rank order, as the kernel adds them
                total = total + rows[q]
            exact = torch.equal(fused, total.to(torch.bfloat16))
            # the standard tolerance against an independent run of each shard
            part = moe_host.run(*workloads.as_args(inp)).float()
            ref = part.clone()
            dist.all_reduce(ref)
            err = (fused.float() - ref).abs()
            within = float((err <= 1e-2 * ref.abs().max()).float().mean())
            other = fused.clone()
            dist.broadcast(other, src=0)
            results.put((rank, T, variant, int(status), exact, within, torch.equal(fused, other),
                         float(ref.abs().max())))
        del comb
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
    # decode plan; compact combine rows; token-major GEMMs (K split, compact rows)
    cases = [(16, "uniform"), (200, "uniform"), (600, "uniform")]
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, cases, results)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    for p in procs:
        if p.is_alive():
            p.kill()
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    got = [results.get(timeout=5) for _ in range(world * len(cases))]
    for rank, T, variant, status, exact, within, same, amax in got:
        assert status == 0, (rank, T, status)
        assert exact, (rank, T, variant)
        assert within >= 0.999, (rank, T, variant, within)
        assert same, (rank, T)
        assert amax > 0.0, (rank, T)
