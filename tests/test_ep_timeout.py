"""Failure detection of the expert-parallel combine on one GPU.

The combine waits for every peer with a one-second limit. Here a second
"rank" exists only as an EP area that nothing ever writes, so the wait for
its announcement runs out (a flag that nothing sets; no fault, no trap):
the call must report status bit 1 << 7, poison both areas, make the next
combine return at once with bit 1 << 8, and after the areas are zeroed a
combine must work again and reproduce the layer's own output. (T = 16 on two
ranks takes the flagged-line protocol: the wait that runs out is the poll
for the second rank's partial sums.)
"""
from __future__ import annotations

import pytest
import torch

import workloads

pytestmark = pytest.mark.gpu

T = 16


def test_combine_gives_up_poisons_and_recovers(cuda_device):
    import moe_host

    inp = workloads.make_inputs(T, 21, cuda_device)
    ws = torch.empty(moe_host.workspace_bytes(T), dtype=torch.uint8, device=cuda_device)
    area_bytes = moe_host.ep_area_bytes(T)
    areas = [torch.zeros(area_bytes, dtype=torch.uint8, device=cuda_device) for _ in range(2)]
    args = workloads.as_args(inp)
    ref = moe_host.run(*args)

    def layer():
        moe_host.run_dps(*args, None, workspace=ws)

    out = torch.full((T, 7168), float("nan"), dtype=torch.bfloat16, device=cuda_device)
    # rank 0 of 2; rank 1 never announces
    layer()
    moe_host.ep_combine_shards([ws.data_ptr(), ws.data_ptr()], 1, [a.data_ptr() for a in areas], 0, T, out)
    torch.cuda.synchronize()
    st = moe_host.read_status(ws)
    assert st & (1 << 7), hex(st)
    for a in areas:   # both areas poisoned (int32 at byte 76 of the counter block)
        assert int(a[76:80].view(torch.int32).item()) != 0
    # the next combine on the poisoned areas returns at once, writing nothing
    layer()
    out.fill_(float("nan"))
    moe_host.ep_combine_shards([ws.data_ptr(), ws.data_ptr()], 1, [a.data_ptr() for a in areas], 0, T, out)
    torch.cuda.synchronize()
    st = moe_host.read_status(ws)
    assert st == (1 << 8), hex(st)
    assert torch.isnan(out.float()).all()
    # recovery: zero the areas; a one-rank combine then equals the output
    # the layer itself wrote from the same combine rows
    for a in areas:
        a.zero_()
    own = torch.empty_like(out)
    moe_host.run_dps(*args, own, workspace=ws)
    moe_host.ep_combine_shards([ws.data_ptr()], 1, [areas[0].data_ptr()], 0, T, out)
    torch.cuda.synchronize()
    assert moe_host.read_status(ws) == 0
    assert torch.equal(out, own)
    err = (own.float() - ref.float()).abs().max().item()
    assert err <= 1e-2 * ref.float().abs().max().item()
