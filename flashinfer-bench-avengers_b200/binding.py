"""TVM-FFI binding of the solution, registered as ``flashinfer.kernel``.

Fills in the reference's template (solution/cuda/binding.py:10-25, which
registers ``flashinfer.kernel`` with an empty body). The reference imports
``tvm.ffi``; this image ships the standalone ``tvm_ffi`` package, whose
``register_global_func`` is the same registry.

The registered function is destination-passing: the ten inputs of
``main.py::run`` followed by ``output`` (bf16 [T, 7168]). Tensors may arrive
as tvm_ffi tensors or anything else that speaks DLPack; they are viewed as
torch tensors without a copy and passed to ``moe_host.run_dps``.
"""
from __future__ import annotations

import os
import sys

import torch
import tvm_ffi

_HERE = os.path.dirname(os.path.abspath(__file__))
if _HERE not in sys.path:
    sys.path.insert(0, _HERE)

import moe_host  # noqa: E402

FUNC_NAME = "flashinfer.kernel"


def _as_torch(x):
    if isinstance(x, torch.Tensor):
        return x
    return torch.from_dlpack(x)


def kernel(routing_logits, routing_bias, hidden_states, hidden_states_scale, gemm1_weights,
           gemm1_weights_scale, gemm2_weights, gemm2_weights_scale, local_expert_offset,
           routed_scaling_factor, output):
    out = _as_torch(output)
    moe_host.run_dps(_as_torch(routing_logits), _as_torch(routing_bias), _as_torch(hidden_states),
                     _as_torch(hidden_states_scale), _as_torch(gemm1_weights),
                     _as_torch(gemm1_weights_scale), _as_torch(gemm2_weights),
                     _as_torch(gemm2_weights_scale), int(local_expert_offset),
                     float(routed_scaling_factor), out)


tvm_ffi.register_global_func(FUNC_NAME, kernel, override=True)
