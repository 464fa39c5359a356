"""Failure detection of the token-parallel all-to-all on one GPU.

The dispatch waits, with a one-second limit, for every rank's announcement
of its send counts. Here a second "rank" exists only as an all-to-all area
that nothing ever writes, so that wait runs out (a flag that nothing sets; no
fault, no trap): the call must report status bit 1 << 7 and poison both
areas; the next call must return at once with bit 1 << 8 and write nothing;
after the counter blocks are zeroed a one-rank call must work again (status
clear, every token received as one slab row, bit for bit).
"""
from __future__ import annotations

import pytest
import torch

import workloads

pytestmark = pytest.mark.gpu

T = 16
CAP = 2 * T
POISON = 104          # int32 poison word inside the counter block


def test_a2a_gives_up_poisons_and_recovers(cuda_device):
    import moe_host

    inp = workloads.make_inputs(T, 31, cuda_device)
    idx, w = moe_host.route(inp["routing_logits"], inp["routing_bias"], inp["routed_scaling_factor"])
    hs = inp["hidden_states"]
    hss = inp["hidden_states_scale"].contiguous()
    area_bytes = moe_host.a2a_area_bytes(T, CAP)
    areas = [torch.zeros(area_bytes, dtype=torch.uint8, device=cuda_device) for _ in range(2)]
    ptrs = [a.data_ptr() for a in areas]
    # the shard workspaces the combine reads (no layer runs here: all zero)
    wss = [torch.zeros(moe_host.routed_workspace_bytes(CAP, 8), dtype=torch.uint8, device=cuda_device)
           for _ in range(8)]
    ws_ptrs = [x.data_ptr() for x in wss]
    out = torch.full((T, 7168), float("nan"), dtype=torch.bfloat16, device=cuda_device)

    # rank 0 of 2 (4 shards each); rank 1 never announces its counts
    moe_host.a2a_dispatch(idx, w, hs, hss, T, CAP, ptrs, 0, 4)
    moe_host.a2a_combine(idx, ws_ptrs, ptrs, 0, 4, T, CAP, out)
    torch.cuda.synchronize()
    st, _ = moe_host.a2a_read_status(areas[0])
    assert st & (1 << 7), hex(st)
    for a in areas:
        assert int(a[POISON:POISON + 4].view(torch.int32).item()) != 0
    assert torch.isnan(out.float()).all()

    # the next call on the poisoned areas returns at once, writing nothing
    moe_host.a2a_dispatch(idx, w, hs, hss, T, CAP, ptrs, 0, 4)
    moe_host.a2a_combine(idx, ws_ptrs, ptrs, 0, 4, T, CAP, out)
    torch.cuda.synchronize()
    st, _ = moe_host.a2a_read_status(areas[0])
    assert st == (1 << 8), hex(st)
    assert torch.isnan(out.float()).all()

    # recovery: zero the counter blocks; one rank owning all 8 shards then
    # receives every token as one row, in token order, and the combine of
    # the (zero) shard rows writes zeros
    for a in areas:
        a[:moe_host.A2A_COUNTER_BYTES].zero_()
    moe_host.a2a_dispatch(idx, w, hs, hss, T, CAP, ptrs[:1], 0, 8)
    moe_host.a2a_combine(idx, ws_ptrs, ptrs[:1], 0, 8, T, CAP, out)
    torch.cuda.synchronize()
    st, rows = moe_host.a2a_read_status(areas[0])
    assert st == 0, hex(st)
    assert rows == T
    lay = moe_host.a2a_layout(T, CAP)
    slab = areas[0][lay.slab_rows: lay.slab_rows + T * 7168].view(T, 7168)
    assert torch.equal(slab, hs.view(torch.uint8))
    slab_idx = areas[0][lay.slab_idx: lay.slab_idx + 4 * T * 8].view(torch.int32).view(T, 8)
    assert torch.equal(slab_idx, idx)
    assert torch.equal(out.float(), torch.zeros(T, 7168, device=cuda_device))
