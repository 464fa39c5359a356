"""The upstream hidden-state quantiser (bf16 -> e4m3 + [56, T] scales).

CPU: the oracle quantiser reproduces, from the regenerated bf16 sources,
the e4m3 hidden states and scales of every committed golden fixture
(digests), and handles the edge blocks as its convention says.
GPU: moe_b200_quantize_hidden is bit-exact against the oracle, and
moe_b200_run_bf16_hidden (quantising inside the row copy) writes the same
permuted rows and scales and the same layer output as moe_b200_run on the
quantised inputs.
"""
from __future__ import annotations

import pytest
import torch

from conftest import digest, golden_files, golden_inputs, load_golden

import moe_oracle
import workloads

H = 7168


def _edge_rows(T: int, seed: int) -> torch.Tensor:
    """bf16 [T, 7168] N(0, 1) rows with per-block magnitudes spread over
    2^-60 .. 2^60 and edge blocks: all zero, a single nonzero element, a
    block of negative zeros, one huge value among small ones (results in the
    e4m3 subnormal range and below), exact ties of the maximum, and a block
    with scale 1 whose values sit exactly on e4m3 rounding midpoints."""
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(T, H, generator=g)
    mag = torch.pow(2.0, torch.randint(-60, 61, (T, H // 128), generator=g).float())
    x = (x.view(T, H // 128, 128) * mag.unsqueeze(2)).view(T, H)
    xb = x.view(T, H // 128, 128)
    if T >= 1:
        xb[0, 0] = 0.0
        xb[0, 1] = 0.0
        xb[0, 1, 77] = -3.0
        xb[0, 2] = -0.0
        xb[0, 3] = torch.randn(128, generator=g) * 1e-3
        xb[0, 3, 5] = 1000.0
        xb[0, 4] = 2.5
        xb[0, 4, ::3] = -2.5
        xb[0, 5] = torch.tensor(MIDPOINTS * 16)[:128]
    return x.to(torch.bfloat16)


# amax 448 gives scale 1, so these are their own quotients: midpoints between
# adjacent e4m3 values (normal and subnormal), which round to the even one
MIDPOINTS = [448.0, 1.0625, 1.1875, -2.125, 1.5 * 2.0 ** -9, 0.5 * 2.0 ** -9, 3.5 * 2.0 ** -9, -200.0]
MIDPOINT_BYTES = [0x7E, 0x38, 0x3A, 0xC0, 0x02, 0x00, 0x04, 0xF4]


# ------------------------------------------------------------------ CPU pins
@pytest.mark.parametrize("path", golden_files(), ids=lambda p: p.rsplit("/", 1)[-1][:-4])
def test_oracle_quantiser_reproduces_fixture_inputs(path):
    g = load_golden(path)
    x = workloads.make_hidden_bf16(g["T"], g["seed"], "cpu")
    q, s = moe_oracle.quantize_hidden(x)
    assert digest(q) == g["digests"]["hidden_states"]
    assert digest(s) == g["digests"]["hidden_states_scale"]


def test_oracle_quantiser_edge_blocks():
    x = _edge_rows(2, 3)
    q, s = moe_oracle.quantize_hidden(x)
    qb = q.view(torch.uint8).view(2, H // 128, 128)
    assert s[0, 0] == 1.0 and bool((qb[0, 0] == 0).all())                 # all-zero block
    assert s[1, 0] == 3.0 / 448.0 and qb[0, 1, 77] == 0xFE                  # -448 = 0xFE
    assert s[2, 0] == 1.0 and bool((qb[0, 2] == 0x80).all())               # negative zeros
    assert qb[0, 3, 5] == 0x7E and bool((qb[0, 3] != 0x7E).sum() == 127)   # 448 once
    assert bool((qb[0, 4].float() != 0).all())                             # ties of the max
    assert s[5, 0] == 1.0 and qb[0, 5, :8].tolist() == MIDPOINT_BYTES      # ties to even
    # every block's largest magnitude quantises to +-448
    mx = qb.view(torch.float8_e4m3fn).float().abs().amax(dim=2)
    nz = s.t() != 1.0
    assert bool((mx[nz] == 448.0).all())


# ------------------------------------------------------------------ GPU parity
@pytest.fixture(scope="module")
def host(cuda_device):
    import moe_host

    moe_host.load_library()
    return moe_host


@pytest.mark.gpu
@pytest.mark.parametrize("T,seed", [(1, 0), (37, 1), (1000, 2)])
def test_quantize_hidden_bit_exact(host, T, seed):
    x = _edge_rows(T, seed)
    q, s = host.quantize_hidden(x.cuda())
    torch.cuda.synchronize()
    rq, rs = moe_oracle.quantize_hidden(x)
    assert torch.equal(q.cpu().view(torch.uint8), rq.view(torch.uint8))
    assert torch.equal(s.cpu(), rs)


@pytest.mark.gpu
@pytest.mark.parametrize("T,variant,offset", [(16, "uniform", 0), (200, "uniform", 32), (600, "zipf", 128)])
def test_run_bf16_hidden_matches_quantised_run(host, T, variant, offset):
    """Decode, mid-size and token-major plans: the permuted rows and scales
    (and above 64 tokens the per-token e4m3 copy in the workspace) equal the
    oracle quantisation of the tokens' rows bit for bit, and the output
    equals moe_b200_run on the quantised inputs (within one bf16 ulp: both
    accumulate with fp32 atomics)."""
    inp = {k: (v.cuda() if torch.is_tensor(v) else v)
           for k, v in workloads.make_inputs(T, 3, "cpu", variant, offset, 2.5).items()}
    x = workloads.make_hidden_bf16(T, 62, "cpu")
    rq, rs = moe_oracle.quantize_hidden(x)
    args = workloads.as_args(inp)
    out = host.run_bf16_hidden(args[0], args[1], x.cuda(), *args[4:])
    torch.cuda.synchronize()
    ws = host.get_workspace(T, out.device)
    lay = host.workspace_layout(T)
    seg = ws[lay.seg_off: lay.seg_off + 33 * 4].view(torch.int32).cpu().long()
    n = int(seg[-1])
    perm_tok = ws[lay.perm_tok: lay.perm_tok + 4 * n].view(torch.int32).cpu().long()
    valid = perm_tok >= 0
    assert int(valid.sum()) > 0
    a_perm = ws[lay.a_perm: lay.a_perm + n * H].view(n, H).cpu()
    assert torch.equal(a_perm[valid], rq.view(torch.uint8)[perm_tok[valid]])
    sa = ws[lay.sa_perm: lay.sa_perm + 56 * lay.cap_rows * 4].view(torch.float32).view(56, lay.cap_rows).cpu()
    assert torch.equal(sa[:, :n][:, valid], rs[:, perm_tok[valid]])
    if T > 64:
        hq = ws[lay.hidden_q: lay.hidden_q + T * H].view(T, H).cpu()
        hqs = ws[lay.hidden_qs: lay.hidden_qs + 56 * T * 4].view(torch.float32).view(56, T).cpu()
        assert torch.equal(hq, rq.view(torch.uint8)) and torch.equal(hqs, rs)
    assert host.read_status(ws) == 0
    args[2], args[3] = rq.cuda(), rs.cuda()
    ref = host.run(*args)
    torch.cuda.synchronize()
    a, b = out.float(), ref.float()
    mag = torch.maximum(a.abs(), b.abs())
    assert bool(((a - b).abs() <= mag * 2.0 ** -7 + 1e-4 * float(b.abs().max())).all())


@pytest.mark.gpu
@pytest.mark.parametrize("path", golden_files(), ids=lambda p: p.rsplit("/", 1)[-1][:-4])
def test_golden_from_bf16_hidden(host, path):
    """The fixtures' outputs, reached from the bf16 hidden states their e4m3
    inputs were quantised from."""
    g = load_golden(path)
    if g["routing_method"] != 2:
        pytest.skip("the bf16-hidden entry point routes with DeepSeek-V3 only")
    inp, _ = golden_inputs(g, device="cuda")
    x = workloads.make_hidden_bf16(g["T"], g["seed"], "cpu").cuda()
    args = workloads.as_args(inp)
    out = host.run_bf16_hidden(args[0], args[1], x, *args[4:])
    torch.cuda.synchronize()
    ok, matched, max_err, ref_max = moe_oracle.output_close(out, g["output"], 1e-2, 0.999)
    assert ok, f"{g['name']}: matched {matched:.5f}, max err {max_err:.4g}, max|ref| {ref_max:.4g}"
