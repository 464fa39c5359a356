"""The allocation-free entry point moe_b200_run_noalloc, called through the
C ABI, against the regular entry point.

It serves callers that may not allocate device memory when they call the
layer (their scratch is a fixed array inside the library). Two calls in a
row with different batches must both match moe_b200_run within the layer's
tolerance, which also shows that the previous call's leftovers in the shared
array do no harm. This file is collected last so that a stop at the first
failure has already run every other test.
"""
from __future__ import annotations

import ctypes

import pytest
import torch

import moe_oracle
import workloads

pytestmark = pytest.mark.gpu

REL_TOL = 1e-2
MATCH_FRAC = 0.999
MAX_TOKENS = 16


@pytest.fixture(scope="module")
def lib(cuda_device):
    import moe_host

    lib = moe_host.load_library()
    P, I64 = ctypes.c_void_p, ctypes.c_int64
    lib.moe_b200_run_noalloc.argtypes = [P, P, ctypes.c_int, P, P, P, P, P, P, I64, ctypes.c_double, I64,
                                         P, P]
    lib.moe_b200_run_noalloc.restype = ctypes.c_int
    return lib


def _noalloc(lib, inp, out):
    bias = inp["routing_bias"]
    code = lib.moe_b200_run_noalloc(
        inp["routing_logits"].data_ptr(), bias.data_ptr(), 0, inp["hidden_states"].data_ptr(),
        inp["hidden_states_scale"].data_ptr(), inp["gemm1_weights"].data_ptr(),
        inp["gemm1_weights_scale"].data_ptr(), inp["gemm2_weights"].data_ptr(),
        inp["gemm2_weights_scale"].data_ptr(), int(inp["local_expert_offset"]),
        float(inp["routed_scaling_factor"]), inp["routing_logits"].shape[0], out.data_ptr(),
        torch.cuda.current_stream().cuda_stream)
    return code


def _noalloc_status(lib) -> int:
    st = ctypes.c_uint32(0)
    lib.moe_b200_noalloc_read_status(ctypes.byref(st), torch.cuda.current_stream().cuda_stream)
    return int(st.value)


def test_noalloc_matches_regular_entry_point_twice(lib):
    import moe_host

    for T, seed in ((16, 101), (5, 102)):  # two calls in a row, different batches
        inp = workloads.make_inputs(T, seed, "cuda")
        out = torch.full((T, workloads.H), float("nan"), dtype=torch.bfloat16, device="cuda")
        assert _noalloc(lib, inp, out) == 0
        torch.cuda.synchronize()
        # the status word lives in the library's array; every bounded wait completed
        assert _noalloc_status(lib) == 0
        ref = moe_host.run(*workloads.as_args(inp))
        torch.cuda.synchronize()
        ok, matched, max_err, ref_max = moe_oracle.output_close(out, ref, REL_TOL, MATCH_FRAC)
        assert ok, f"T={T}: matched {matched:.5f}, max err {max_err:.4g}, max|ref| {ref_max:.4g}"
        if T == 5:  # one call also against the CPU oracle directly
            cpu = {k: (v.cpu() if isinstance(v, torch.Tensor) else v) for k, v in inp.items()}
            oref = moe_oracle.moe_forward(*workloads.as_args(cpu))
            ok, matched, max_err, ref_max = moe_oracle.output_close(out.cpu(), oref, REL_TOL, MATCH_FRAC)
            assert ok, f"oracle T={T}: matched {matched:.5f}, max err {max_err:.4g}, max|ref| {ref_max:.4g}"


def test_noalloc_rejects_batches_beyond_its_limit(lib):
    inp = workloads.make_inputs(MAX_TOKENS + 1, 103, "cuda", experts=[0])
    out = torch.empty(MAX_TOKENS + 1, workloads.H, dtype=torch.bfloat16, device="cuda")
    assert _noalloc(lib, inp, out) == 3  # MOE_B200_ERR_WORKSPACE_TOO_SMALL
