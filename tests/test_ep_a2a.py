"""Token-parallel expert parallelism (all-to-all dispatch and combine) on B200s.

Single GPU: world 1 owns all 8 shards, so every token is dispatched to this
GPU's own slab as one row with all its picks; that exercises the plan, the
wire format, the routed layer on the slab and the combine without a peer.
Checked: the slab rows, scales, expert ids and weights against the oracle's
numbering of the (token, destination) rows (bit for bit), the output bit for
bit against the fp32 sum in shard order of the token's combine rows read
back from the shard workspaces, within the operator tolerance of the
oracle's restatement of the whole token-parallel layer, and the same on a
second call (the counters advance).

2-4 GPUs: every rank has its own tokens (a different batch per rank, in one
call none on the last rank) and 8/W shards; each rank's output must match, within the operator tolerance, the
expert-parallel layer (NvlinkCombiner) run by every rank on the gathered
batch of all ranks' tokens, be bit-identical to the fp32 sum of the token's
combine rows read back over peer memory (each rank's shards in shard order,
then the ranks in rank order), and leave the status words clear. Skipped
below two GPUs.
"""
from __future__ import annotations

import os
import socket
import sys

import pytest
import torch

import moe_oracle
import workloads

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "flashinfer-bench-avengers_b200")
REL_TOL = 1e-2
MATCH_FRAC = 0.999


def _shard_inputs(T, seed, dev, offsets):
    """Tokens (seed) and, per shard offset, that shard's weights (weight seed
    by shard), only the experts these tokens pick materialised."""
    r = workloads.make_routing_inputs(T, seed, dev)
    idx, _ = moe_oracle.route(r["routing_logits"].cpu(), r["routing_bias"].cpu(), 2.5)
    out = []
    for off in offsets:
        le = sorted({e - off for e in idx.flatten().tolist() if off <= e < off + 32})
        out.append(workloads.make_inputs(T, seed, dev, "uniform", off, 2.5, experts=le,
                                         weight_seed=300 + off // 32))
    return out


def _shard_rows(tp, s, rows):
    """fp32 combine rows of shard workspace s for slab rows `rows` (local)."""
    import moe_host

    lay = moe_host.routed_workspace_layout(tp.cap, 8)
    ws = tp.workspaces[s]
    rows = rows.to(ws.device)
    y = ws[lay.y_acc: lay.y_acc + 4 * 7168 * tp.cap].view(torch.float32).view(tp.cap, 7168)
    if tp.cap > 64:   # compact combine rows; a slab row without a pick here has none (zeros)
        slot = ws[lay.tok_slot: lay.tok_slot + 4 * tp.cap].view(torch.int32).long()[rows]
        return torch.where((slot >= 0)[:, None], y[slot.clamp(min=0)], torch.zeros_like(y[:1])).cpu()
    return y[rows].cpu()


def _readback(tp, T):
    """fp32 sum in shard order of each token's combine rows (one GPU owns all
    shards, every token is one slab row): the value the combine must round
    to bf16."""
    rows = tp.dest_rows(T)[:, 0].cpu().long()
    total = torch.zeros(T, 7168, dtype=torch.float32)
    part = torch.zeros(T, 7168, dtype=torch.float32)
    for s in range(8):
        part = part + _shard_rows(tp, s, rows)
    return total + part


@pytest.mark.parametrize("T", [40, 520])
def test_token_parallel_single_gpu(cuda_device, T):
    import expert_parallel
    import moe_host

    offsets = list(range(0, 256, 32))
    inps = _shard_inputs(T, 77, cuda_device, offsets)
    tok = {k: inps[0][k] for k in ("routing_logits", "routing_bias", "hidden_states", "hidden_states_scale",
                                   "routed_scaling_factor")}
    shards = [(i["gemm1_weights"], i["gemm1_weights_scale"], i["gemm2_weights"], i["gemm2_weights_scale"])
              for i in inps]
    tp = expert_parallel.TokenParallelEP(T, cuda_device)
    try:
        out = torch.full((T, 7168), float("nan"), dtype=torch.bfloat16, device=cuda_device)
        tp.forward(tok, shards, out)
        torch.cuda.synchronize()
        assert tp.status() == 0
        assert tp.slab_rows() == T
        # the slab: the oracle's numbering of the (token, destination) rows,
        # the wire format (one rank: every token is a row with all its picks)
        idx = tp.topk_idx[:T].cpu()
        w = tp.topk_w[:T].cpu()
        slot, counts = moe_oracle.a2a_plan(idx, 1, 8)
        assert int(counts[0]) == T
        rows = tp.dest_rows(T).cpu().long()
        assert torch.equal(rows, slot)
        lay = tp.layout
        area = tp.area
        s_idx = area[lay.slab_idx: lay.slab_idx + 4 * 8 * tp.cap].view(torch.int32).view(tp.cap, 8).cpu()
        s_w = area[lay.slab_w: lay.slab_w + 4 * 8 * tp.cap].view(torch.float32).view(tp.cap, 8).cpu()
        s_rows = area[lay.slab_rows: lay.slab_rows + tp.cap * 7168].view(tp.cap, 7168).cpu()
        s_sc = area[lay.slab_scale: lay.slab_scale + 4 * 56 * tp.cap].view(torch.float32).view(56, tp.cap).cpu()
        r0 = slot[:, 0]
        assert torch.equal(s_idx[r0], idx)
        assert torch.equal(s_w[r0], w)
        assert torch.equal(s_rows[r0], tok["hidden_states"].view(torch.uint8).cpu())
        assert torch.equal(s_sc[:, r0], tok["hidden_states_scale"].cpu())
        # the output: the shard-order sum of the token's combine rows, rounded once
        exact = _readback(tp, T)
        assert torch.equal(out.cpu(), exact.to(torch.bfloat16))
        # against the oracle's token-parallel restatement (one rank)
        cpu_tok = {k: (v.cpu() if torch.is_tensor(v) else v) for k, v in tok.items()}
        weights = {}
        for off, i in zip(offsets, inps):
            weights[off] = tuple(i[k].cpu() for k in ("gemm1_weights", "gemm1_weights_scale", "gemm2_weights",
                                                      "gemm2_weights_scale"))
        if T <= 64:
            ref = moe_oracle.token_parallel_forward([cpu_tok], weights, 1)[0][0]
            ok, matched, max_err, ref_max = moe_oracle.output_close(out, ref, REL_TOL, MATCH_FRAC)
            assert ok, f"T={T}: matched {matched:.5f}, max err {max_err:.4g}, max|ref| {ref_max:.4g}"
        # and against the sum over the 8 shards of the regular entry point
        ep = sum(moe_host.run(*workloads.as_args(i)).float() for i in inps)
        ok, matched, max_err, ref_max = moe_oracle.output_close(out, ep, REL_TOL, MATCH_FRAC)
        assert ok, f"T={T} vs shards: matched {matched:.5f}, max err {max_err:.4g}, max|ref| {ref_max:.4g}"
        # a second call: the counters advance, the result repeats
        out2 = torch.empty_like(out)
        tp.forward(tok, shards, out2)
        torch.cuda.synchronize()
        assert tp.status() == 0
        assert torch.equal(out2.cpu(), _readback(tp, T).to(torch.bfloat16))
    finally:
        tp.close()


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank: int, world: int, port: int, sizes, results):
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    sys.path.insert(0, PKG)
    import torch.distributed as dist
    from datetime import timedelta

    import expert_parallel
    import moe_host
    import workloads as wl

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60), device_id=dev)
    try:
        S = 8 // world
        offsets = [32 * (rank * S + s) for s in range(S)]
        for T_list in sizes:
            Tmax = max(T_list)
            # every rank's tokens (the same generators on every rank)
            toks = []
            for q in range(world):
                r = wl.make_routing_inputs(T_list[q], 500 + q, dev)
                hs, sc = wl.make_hidden(T_list[q], 500 + q, dev)
                toks.append(dict(r, hidden_states=hs, hidden_states_scale=sc))
            for q in range(1, world):   # one model: every rank routes with the same bias
                toks[q]["routing_bias"] = toks[0]["routing_bias"]
            Ttot = sum(T_list)
            # this rank's shard weights: every expert any token of any rank picks
            allr = torch.cat([toks[q]["routing_logits"] for q in range(world)])
            idx_all, _ = moe_host.route(allr, toks[0]["routing_bias"], 2.5)
            shard_inps = []
            for off in offsets:
                le = sorted({e - off for e in idx_all.flatten().tolist() if off <= e < off + 32})
                shard_inps.append(wl.make_inputs(1, 0, dev, "uniform", off, 2.5, experts=le,
                                                 weight_seed=300 + off // 32))
            shards = [(i["gemm1_weights"], i["gemm1_weights_scale"], i["gemm2_weights"], i["gemm2_weights_scale"])
                      for i in shard_inps]
            mine = toks[rank]
            tok = {"routing_logits": mine["routing_logits"], "routing_bias": mine["routing_bias"],
                   "hidden_states": mine["hidden_states"], "hidden_states_scale": mine["hidden_states_scale"],
                   "routed_scaling_factor": 2.5}
            tp = expert_parallel.TokenParallelEP(Tmax, dev)
            out = torch.empty(T_list[rank], 7168, dtype=torch.bfloat16, device=dev)
            for _ in range(2):   # twice: the call counters must advance correctly
                tp.forward(tok, shards, out)
            torch.cuda.synchronize()
            status = tp.status()
            # the fp32 sum of each token's combine rows: every source says
            # where its tokens went, every destination returns each of its
            # shards' rows for them from its own workspaces (local reads),
            # the source sums each rank's shards in shard order, then the
            # ranks in rank order
            rows = tp.dest_rows(T_list[rank]).cpu().long()
            asks = [None] * world
            dist.all_gather_object(asks, rows)
            answers = {}
            for src, s_rows in enumerate(asks):
                for t in range(s_rows.shape[0]):
                    r = int(s_rows[t, rank])
                    if r >= 0:
                        for s in range(S):
                            answers[(src, t, s)] = _shard_rows(tp, s, torch.tensor([r]))[0]
            replies = [None] * world
            dist.all_gather_object(replies, answers)
            exact = torch.zeros(T_list[rank], 7168, dtype=torch.float32)
            for t in range(T_list[rank]):
                for q, rep in enumerate(replies):
                    part = torch.zeros(7168, dtype=torch.float32)
                    for s in range(S):
                        if (rank, t, s) in rep:
                            part = part + rep[(rank, t, s)]
                    exact[t] = exact[t] + part
            is_exact = torch.equal(out.cpu(), exact.to(torch.bfloat16))
            tp.close()
            # expert-parallel reference on the gathered batch of all ranks' tokens
            g_tok = {"routing_logits": torch.cat([t_["routing_logits"] for t_ in toks]),
                     "routing_bias": toks[0]["routing_bias"],
                     "hidden_states": torch.cat([t_["hidden_states"] for t_ in toks]),
                     "hidden_states_scale": torch.cat([t_["hidden_states_scale"] for t_ in toks], dim=1),
                     "routed_scaling_factor": 2.5}
            comb = expert_parallel.NvlinkCombiner(Ttot, dev, shards_per_rank=S)
            ref_all = torch.empty(Ttot, 7168, dtype=torch.bfloat16, device=dev)
            comb.forward_shards(g_tok, [sh + (off,) for sh, off in zip(shards, offsets)], ref_all)
            torch.cuda.synchronize()
            comb.close()
            lo = sum(T_list[:rank])
            ref = ref_all[lo: lo + T_list[rank]].float()
            if T_list[rank] > 0:
                err = (out.float() - ref).abs()
                within = float((err <= REL_TOL * ref.abs().max()).float().mean())
            else:
                within = 1.0
            results.put((rank, tuple(T_list), int(status), is_exact, within))
        torch.cuda.synchronize()
        dist.barrier()
    finally:
        dist.destroy_process_group()


def test_token_parallel_ranks():
    if not torch.cuda.is_available() or torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    world = 4 if torch.cuda.device_count() >= 4 else 2
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    results = ctx.Queue()
    # a different batch on every rank: decode-size slabs and token-major
    # slabs, and a call in which the last rank has no tokens (it still takes
    # every step: the ranks meet in the dispatch and the combine)
    sizes = [tuple(5 + 3 * q for q in range(world)), tuple(90 + 7 * q for q in range(world)),
             tuple(0 if q == world - 1 else 6 + q for q in range(world))]
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, sizes, results)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=600)
    for p in procs:
        if p.is_alive():   # the kernels' waits are bounded; only a stuck host process is left here
            p.kill()
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    got = [results.get(timeout=5) for _ in range(world * len(sizes))]
    for rank, T_list, status, exact, within in got:
        assert status == 0, (rank, T_list, status)
        assert exact, (rank, T_list)
        assert within >= MATCH_FRAC, (rank, T_list, within)
