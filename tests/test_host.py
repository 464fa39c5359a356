"""Host-side behaviour that needs no GPU: argument checks of the Python
entry points (they mirror the reference's TORCH_CHECKs, main.cpp:25-40),
the TVM-FFI registration, and the solution manifest."""
from __future__ import annotations

import os
import tomllib

import pytest
import torch

from conftest import PKG

import workloads


def _cpu_inputs(T=2):
    r = workloads.make_routing_inputs(T, 0, "cpu")
    hs, sc = workloads.quantize_rows_1x128(torch.zeros(T, 7168))
    return [r["routing_logits"], r["routing_bias"], hs, sc,
            torch.zeros(32, 4096, 7168, dtype=torch.float8_e4m3fn), torch.ones(32, 32, 56),
            torch.zeros(32, 7168, 2048, dtype=torch.float8_e4m3fn), torch.ones(32, 56, 16), 0, 2.5]


@pytest.fixture(scope="module")
def cpu_args():
    return _cpu_inputs()


def test_run_requires_cuda_tensors(cpu_args):
    import moe_host

    with pytest.raises(RuntimeError, match="must be CUDA"):
        moe_host.run(*cpu_args)


def test_all_to_all_wrappers_require_cuda_tensors():
    """The token-parallel dispatch and combine refuse host tensors before
    any library call (their kernels would dereference host pointers)."""
    import moe_host

    T = 4
    idx = torch.zeros(T, 8, dtype=torch.int32)
    w = torch.zeros(T, 8)
    hs = torch.zeros(T, 7168, dtype=torch.float8_e4m3fn)
    sc = torch.ones(56, T)
    with pytest.raises(RuntimeError, match="must be a CUDA tensor"):
        moe_host.a2a_dispatch(idx, w, hs, sc, T, 2 * T, [0, 0], 0, 4)
    with pytest.raises(RuntimeError, match="must be a CUDA tensor"):
        moe_host.a2a_combine(idx, [0] * 8, [0, 0], 0, 4, T, 2 * T, torch.zeros(T, 7168, dtype=torch.bfloat16))


def test_check_inputs_shapes_and_dtypes(cpu_args, monkeypatch):
    import moe_host

    # Pretend the tensors are on a GPU to reach the shape/dtype checks.
    monkeypatch.setattr(torch.Tensor, "is_cuda", property(lambda self: True))
    good = list(cpu_args[:8])
    assert moe_host._check_inputs(*good) == 2
    cases = [
        (0, torch.zeros(2, 255), "routing_logits must be"),
        (0, torch.zeros(2, 256, dtype=torch.float64), "float32"),
        (1, torch.zeros(255), "routing_bias"),
        (2, torch.zeros(2, 7168), "float8_e4m3fn"),
        (3, torch.ones(2, 56), "hidden_states_scale must be"),
        (4, torch.zeros(31, 4096, 7168, dtype=torch.float8_e4m3fn), "gemm1_weights must be"),
        (5, torch.ones(32, 32, 55), "gemm1_weights_scale"),
        (6, torch.zeros(32, 2048, 7168, dtype=torch.float8_e4m3fn), "gemm2_weights must be"),
        (7, torch.ones(32, 56, 16, dtype=torch.float16), "float32"),
    ]
    for i, bad, msg in cases:
        args = list(good)
        args[i] = bad
        with pytest.raises(RuntimeError, match=msg):
            moe_host._check_inputs(*args)
    args = list(good)
    args[2] = good[2].t()  # wrong shape and not contiguous
    with pytest.raises(RuntimeError):
        moe_host._check_inputs(*args)


def test_bias_dtype_codes():
    import moe_host

    b, code = moe_host._bias_arg(torch.zeros(256, dtype=torch.bfloat16))
    assert code == moe_host.BIAS_BF16 and b.dtype == torch.bfloat16
    b, code = moe_host._bias_arg(torch.zeros(256, dtype=torch.float16))
    assert code == moe_host.BIAS_FP32 and b.dtype == torch.float32


def test_tvm_ffi_registration(cpu_args):
    import tvm_ffi

    import binding

    f = tvm_ffi.get_global_func(binding.FUNC_NAME)
    assert f is not None
    out = torch.empty(2, 7168, dtype=torch.bfloat16)
    with pytest.raises(Exception, match="must be CUDA"):
        binding.kernel(*cpu_args, out)


def test_solution_manifest():
    with open(os.path.join(PKG, "config.toml"), "rb") as f:
        cfg = tomllib.load(f)
    assert cfg["solution"]["definition"] == "moe_fp8_block_scale_ds_routing_topk8_ng8_kg4_e32_h7168_i2048"
    assert cfg["build"]["entry_point"] == "main.py::run"
    assert cfg["build"]["destination_passing_style"] is False
    assert os.path.exists(os.path.join(PKG, cfg["build"]["entry_point"].split("::")[0]))


def test_entry_point_signature():
    import inspect

    import main

    names = list(inspect.signature(main.run).parameters)
    assert names == list(workloads.ARG_ORDER)
    assert list(inspect.signature(main.run_dps).parameters) == list(workloads.ARG_ORDER) + ["output"]
