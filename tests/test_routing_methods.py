"""The other routing methods of the operator family (flashinfer's
RoutingMethodType: Default, Renormalize, Llama4, RenormalizeNaive, TopK)
ahead of the same permutation, GEMMs and combine.

The oracle is pinned to the installed flashinfer references through the
routing_*.npz fixtures (test_oracle_golden.py; the GPU runs them in
test_gpu_parity.py::test_golden_on_gpu). Here, on the GPU: the selections
are bit-exact against the oracle (with bf16, fp32 and no bias; ties to the
lower expert id), the weights agree to fp32 rounding, unused slots hold
-(1 << 30) and weight 0, and the full layer matches the oracle in the
decode, mid-size and token-major plans.
"""
from __future__ import annotations

import pytest
import torch

import moe_oracle
import workloads

pytestmark = pytest.mark.gpu

# (method, top_k)
METHODS = [(0, 8), (1, 8), (3, 1), (4, 8), (5, 8), (5, 3), (1, 2)]


@pytest.fixture(scope="module")
def host(cuda_device):
    import moe_host

    moe_host.load_library()
    return moe_host


@pytest.mark.parametrize("method,top_k", METHODS)
@pytest.mark.parametrize("bias_kind", ["bf16", "fp32", "none"])
def test_routing_method_bit_exact(host, method, top_k, bias_kind):
    r = workloads.make_routing_inputs(1000, 17 + method, "cuda")
    bias = {"bf16": r["routing_bias"], "fp32": r["routing_bias"].float() + 0.001, "none": None}[bias_kind]
    idx, w = host.route_method(method, top_k, r["routing_logits"], bias, 2.5)
    torch.cuda.synchronize()
    ref_idx, ref_w = moe_oracle.route_method(r["routing_logits"].cpu(), bias.cpu() if bias is not None else None,
                                             2.5, method, top_k)
    assert torch.equal(idx.cpu().long(), ref_idx)
    torch.testing.assert_close(w.cpu(), ref_w, rtol=2e-6, atol=1e-7)
    assert bool((idx[:, top_k:] == -(1 << 30)).all()) and bool((w[:, top_k:] == 0).all())


def test_routing_method_ties_go_to_lower_index(host):
    g = torch.Generator().manual_seed(5)
    logits = (torch.randint(-2, 3, (256, 256), generator=g).float() * 0.5)
    logits[0, 7] = -0.0
    logits[0, 9] = 0.0
    logits[1] = -1.0            # -0.0 and +0.0 compete for the first slot: equal, so 100 first
    logits[1, 100] = -0.0
    logits[1, 200] = 0.0
    for method, top_k in METHODS:
        idx, _ = host.route_method(method, top_k, logits.cuda(), None, 1.0)
        ref_idx, _ = moe_oracle.route_method(logits, None, 1.0, method, top_k)
        assert torch.equal(idx.cpu().long(), ref_idx), (method, top_k)


@pytest.mark.parametrize("method,top_k", [(0, 8), (1, 8), (3, 1), (4, 8), (5, 4)])
@pytest.mark.parametrize("T,offset", [(16, 0), (200, 32)])
def test_layer_with_routing_method(host, method, top_k, T, offset):
    inp = workloads.make_inputs(T, 23 + method, "cuda", "uniform", offset, 2.5)
    out = host.run_routing(method, top_k, *workloads.as_args(inp))
    torch.cuda.synchronize()
    ref = moe_oracle.moe_forward(*workloads.as_args(inp), routing_method=method, top_k=top_k)
    ok, matched, max_err, ref_max = moe_oracle.output_close(out, ref, 1e-2, 0.999)
    assert ok, f"method {method} T={T}: matched {matched:.5f}, max err {max_err:.4g}, max|ref| {ref_max:.4g}"
    assert host.read_status(host.get_workspace(T, out.device)) == 0


def test_layer_renormalize_token_major(host):
    """T = 600 (token-major GEMMs), no routing bias."""
    inp = workloads.make_inputs(600, 29, "cuda", "uniform", 64, 2.5)
    args = workloads.as_args(inp)
    args[1] = None
    out = host.run_routing(1, 8, *args)
    torch.cuda.synchronize()
    ref = moe_oracle.moe_forward(*args, routing_method=1, top_k=8)
    ok, matched, max_err, ref_max = moe_oracle.output_close(out, ref, 1e-2, 0.999)
    assert ok, f"matched {matched:.5f}, max err {max_err:.4g}, max|ref| {ref_max:.4g}"


def test_invalid_routing_arguments(host):
    r = workloads.make_routing_inputs(4, 1, "cuda")
    for method, top_k in [(2, 4), (3, 2), (1, 0), (1, 9), (6, 8)]:
        with pytest.raises(RuntimeError):
            host.route_method(method, top_k, r["routing_logits"], r["routing_bias"], 1.0)
    with pytest.raises(RuntimeError):   # DeepSeek-V3 needs its bias
        host.route_method(2, 8, r["routing_logits"], None, 1.0)
