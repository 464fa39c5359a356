"""Shared test setup.

Markers: ``gpu`` tests need an sm_100 GPU and the built library; everything
else runs on the CPU. Tests import the package modules by path (the
package directory name is not a Python identifier) and the oracle from
oracle/.
"""
from __future__ import annotations

import glob
import hashlib
import os
import sys

import numpy as np
import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "flashinfer-bench-avengers_b200")
for p in (PKG, os.path.join(ROOT, "oracle"), ROOT):
    if p not in sys.path:
        sys.path.insert(0, p)

GOLDEN_DIR = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an sm_100 (B200) GPU and the built CUDA library")


def golden_files():
    return sorted(glob.glob(os.path.join(GOLDEN_DIR, "*.npz")))


def load_golden(path: str) -> dict:
    z = np.load(path, allow_pickle=False)
    d = {k: z[k] for k in z.files}
    return {
        "name": os.path.basename(path)[:-4],
        "T": int(d["T"]),
        "seed": int(d["seed"]),
        "variant": str(d["variant"]),
        "local_expert_offset": int(d["local_expert_offset"]),
        "routed_scaling_factor": float(d["routed_scaling_factor"]),
        # routing method (flashinfer's RoutingMethodType numbering) and top_k;
        # fixtures without them use this operator's DeepSeek-V3 routing
        "routing_method": int(d["routing_method"]) if "routing_method" in d else 2,
        "top_k": int(d["top_k"]) if "top_k" in d else 8,
        "output": torch.from_numpy(d["output_bf16_bits"]).view(torch.bfloat16),
        "digests": dict(zip([str(k) for k in d["digest_keys"]], [str(v) for v in d["digest_values"]])),
    }


def digest(t: torch.Tensor) -> str:
    t = t.detach().to("cpu").contiguous()
    if t.dtype == torch.float8_e4m3fn:
        t = t.view(torch.uint8)
    elif t.dtype == torch.bfloat16:
        t = t.view(torch.int16)
    return hashlib.sha256(t.numpy().tobytes()).hexdigest()


def golden_inputs(g: dict, device="cpu"):
    """Regenerates a fixture's inputs (active experts only) and checks digests."""
    import moe_oracle
    import workloads

    r = workloads.make_routing_inputs(g["T"], g["seed"], "cpu", g["variant"], g["local_expert_offset"])
    active = moe_oracle.active_local_experts(r["routing_logits"], r["routing_bias"],
                                             g["routed_scaling_factor"], g["local_expert_offset"],
                                             g["routing_method"], g["top_k"])
    inp = workloads.make_inputs(g["T"], g["seed"], "cpu", g["variant"], g["local_expert_offset"],
                                g["routed_scaling_factor"], experts=active)
    dig = g["digests"]
    for k in ("routing_logits", "routing_bias", "hidden_states", "hidden_states_scale"):
        assert digest(inp[k]) == dig[k], f"{g['name']}: regenerated {k} differs from the fixture"
    for e in active:
        assert digest(inp["gemm1_weights"][e]) == dig[f"w13_{e}"], f"{g['name']}: w13[{e}] differs"
        assert digest(inp["gemm2_weights"][e]) == dig[f"w2_{e}"], f"{g['name']}: w2[{e}] differs"
        assert digest(inp["gemm1_weights_scale"][e]) == dig[f"s13_{e}"]
        assert digest(inp["gemm2_weights_scale"][e]) == dig[f"s2_{e}"]
    if device != "cpu":
        inp = {k: (v.to(device) if isinstance(v, torch.Tensor) else v) for k, v in inp.items()}
    return inp, active


def gpu_available() -> bool:
    if not torch.cuda.is_available():
        return False
    major, minor = torch.cuda.get_device_capability(0)
    return (major, minor) == (10, 0)


@pytest.fixture(scope="session")
def cuda_device():
    if not gpu_available():
        pytest.skip("needs an sm_100 GPU")
    return torch.device("cuda", 0)
