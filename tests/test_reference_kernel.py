"""The reference solution's own CUDA kernel as a second pin of the oracle.

baseline/build_reference.py compiles the reference's unchanged
solution/cuda/{kernel.cu,main.cpp} into baseline/_ref/moe_ref_ext*.so. On
config 0 of the benchmark (T=16, seed 0, 32 local experts at offset 0) its
output must agree with the CPU oracle within the operator tolerance, and
with this library's output. The reference computes GEMM2 in fp16 with the
W2 block scale folded into fp16 weights (solution/cuda/kernel.cu:1458-1507),
so it is compared within the tolerance, not bit for bit. Skipped when the
extension has not been built (the reference checkout is absent on the GPU
box; the built module travels with the tree).
"""
from __future__ import annotations

import os
import sys

import pytest
import torch

import moe_oracle
import workloads
from conftest import ROOT

pytestmark = pytest.mark.gpu

REL_TOL = 1e-2
MATCH_FRAC = 0.999


def _reference_module():
    sys.path.insert(0, os.path.join(ROOT, "baseline"))
    import build_reference

    if build_reference.built_path() is None:
        pytest.skip("reference extension not built (baseline/build_reference.py)")
    return build_reference.load_built()


def test_reference_kernel_pins_the_oracle(cuda_device):
    import moe_host

    ref_mod = _reference_module()
    inp = workloads.make_inputs(16, 0, cuda_device)
    args = workloads.as_args(inp)
    out_ref = ref_mod.run(*args)
    torch.cuda.synchronize()
    assert out_ref.dtype == torch.bfloat16 and tuple(out_ref.shape) == (16, 7168)
    cpu = {k: (v.cpu() if isinstance(v, torch.Tensor) else v) for k, v in inp.items()}
    oracle = moe_oracle.moe_forward(*workloads.as_args(cpu))
    ok, matched, max_err, ref_max = moe_oracle.output_close(out_ref.cpu(), oracle, REL_TOL, MATCH_FRAC)
    assert ok, f"reference kernel vs oracle: matched {matched:.5f}, max err {max_err:.4g}, max|ref| {ref_max:.4g}"
    ours = moe_host.run(*args)
    ok, matched, max_err, ref_max = moe_oracle.output_close(ours.cpu(), out_ref.cpu(), REL_TOL, MATCH_FRAC)
    assert ok, f"ours vs reference kernel: matched {matched:.5f}, max err {max_err:.4g}, max|ref| {ref_max:.4g}"
