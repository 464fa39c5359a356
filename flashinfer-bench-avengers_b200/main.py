"""Entry point of the solution: ``main.py::run`` (named by config.toml).

Same signature and meaning as the reference entry point
(solution/cuda/main.py:31-54): returns a new bf16 [T, 7168] tensor.
``run_dps`` is the destination-passing variant that writes ``output``.

Like the reference (solution/cuda/main.py:6-29), importing this module
compiles the CUDA sources from source when needed: it loads the sm_100a
library libmoe_b200.so next to this file, building it first with build.py
(nvcc, a few seconds) when it is missing or was built from other sources.
Unlike the reference it deletes no cache and recompiles nothing when the
build is current. It raises if the library cannot be built.
"""
from __future__ import annotations

import os
import sys

_HERE = os.path.dirname(os.path.abspath(__file__))
if _HERE not in sys.path:
    sys.path.insert(0, _HERE)

import moe_host  # noqa: E402

moe_host.load_library()


def run(routing_logits, routing_bias, hidden_states, hidden_states_scale, gemm1_weights,
        gemm1_weights_scale, gemm2_weights, gemm2_weights_scale, local_expert_offset,
        routed_scaling_factor):
    return moe_host.run(routing_logits, routing_bias, hidden_states, hidden_states_scale,
                        gemm1_weights, gemm1_weights_scale, gemm2_weights, gemm2_weights_scale,
                        local_expert_offset, routed_scaling_factor)


def run_dps(routing_logits, routing_bias, hidden_states, hidden_states_scale, gemm1_weights,
            gemm1_weights_scale, gemm2_weights, gemm2_weights_scale, local_expert_offset,
            routed_scaling_factor, output):
    return moe_host.run_dps(routing_logits, routing_bias, hidden_states, hidden_states_scale,
                            gemm1_weights, gemm1_weights_scale, gemm2_weights, gemm2_weights_scale,
                            local_expert_offset, routed_scaling_factor, output)
