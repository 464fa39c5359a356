"""Writes the golden fixtures tests/golden/*.npz.

Each fixture holds the output of an independent implementation of the same
operator -- the DeepSeek-routing FP8 block-scale MoE reference in the
installed flashinfer-python package
(flashinfer/trace/templates/moe.py::_trtllm_fp8_block_scale_moe_ds_routing_reference,
flashinfer-python 0.6.11.post2), imported, not copied -- on seeded inputs
from flashinfer-bench-avengers_b200/workloads.py, with all 32 local experts
materialised. Inputs are not stored (the weights alone are 1.4 GB); the
fixture keeps the generator arguments and SHA-256 digests of the generated
tensors so a test can check that it regenerated the very same inputs.

The routing_*.npz fixtures hold, the same way, the outputs of the sibling
references of the other routing methods in the same module
(_trtllm_fp8_block_scale_moe_{default,renormalize,llama4,renormalize_naive,
topk}_routing_reference) with the method and top_k stored beside them.

Run from the repository root (CPU only, a few minutes, ~25 GB RAM):
    python tests/golden/make_golden.py             # DeepSeek-V3 routing fixtures
    python tests/golden/make_golden.py --routing   # the other routing methods
"""
from __future__ import annotations

import hashlib
import os
import sys

import numpy as np
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, os.path.join(ROOT, "flashinfer-bench-avengers_b200"))

import workloads  # noqa: E402

CASES = [
    # name, T, seed, variant, local_expert_offset, routed_scaling_factor
    ("config0_t16_seed0", 16, 0, "uniform", 0, 2.5),
    ("t1_seed1", 1, 1, "uniform", 0, 2.5),
    ("t7_seed2_offset32", 7, 2, "uniform", 32, 2.5),
    ("t8_seed3_hot", 8, 3, "hot", 0, 2.5),
    ("t12_seed5_zipf_offset224", 12, 5, "zipf", 224, 1.0),
]


def digest(t: torch.Tensor) -> str:
    t = t.detach().to("cpu").contiguous()
    if t.dtype in (torch.float8_e4m3fn, torch.bfloat16):
        t = t.view(torch.uint8) if t.dtype == torch.float8_e4m3fn else t.view(torch.int16)
    return hashlib.sha256(t.numpy().tobytes()).hexdigest()


def input_digests(inp: dict, experts) -> dict:
    d = {
        "routing_logits": digest(inp["routing_logits"]),
        "routing_bias": digest(inp["routing_bias"]),
        "hidden_states": digest(inp["hidden_states"]),
        "hidden_states_scale": digest(inp["hidden_states_scale"]),
    }
    for e in experts:
        d[f"w13_{e}"] = digest(inp["gemm1_weights"][e])
        d[f"s13_{e}"] = digest(inp["gemm1_weights_scale"][e])
        d[f"w2_{e}"] = digest(inp["gemm2_weights"][e])
        d[f"s2_{e}"] = digest(inp["gemm2_weights_scale"][e])
    return d


# name, T, seed, variant, local_expert_offset, routed_scaling_factor, method, top_k
# (methods numbered as flashinfer's RoutingMethodType)
ROUTING_CASES = [
    ("routing_default_t8_seed7", 8, 7, "uniform", 0, 2.5, 0, 8),
    ("routing_renormalize_t8_seed8_offset32", 8, 8, "uniform", 32, 1.0, 1, 8),
    ("routing_llama4_t32_seed9", 32, 9, "uniform", 0, 2.5, 3, 1),
    ("routing_renormalize_naive_t8_seed10", 8, 10, "hot", 0, 2.5, 4, 8),
    ("routing_topk_t8_seed11_top4", 8, 11, "uniform", 0, 2.5, 5, 4),
]
ROUTING_REFS = {0: "default", 1: "renormalize", 3: "llama4", 4: "renormalize_naive", 5: "topk"}


def main_routing() -> None:
    import flashinfer.trace.templates.moe as ext

    torch.set_num_threads(os.cpu_count() or 1)
    for name, T, seed, variant, off, rsf, method, top_k in ROUTING_CASES:
        fn_name = f"_trtllm_fp8_block_scale_moe_{ROUTING_REFS[method]}_routing_reference"
        ext_ref = getattr(ext, fn_name)
        inp = workloads.make_inputs(T, seed, "cpu", variant, off, rsf)
        out = ext_ref(inp["routing_logits"], inp["routing_bias"], inp["hidden_states"],
                      inp["hidden_states_scale"], inp["gemm1_weights"], inp["gemm1_weights_scale"],
                      inp["gemm2_weights"], inp["gemm2_weights_scale"], top_k, off, rsf)
        dig = input_digests(inp, range(workloads.E_LOCAL))
        keys = sorted(dig)
        np.savez_compressed(
            os.path.join(os.path.dirname(os.path.abspath(__file__)), f"{name}.npz"),
            T=T, seed=seed, variant=variant, local_expert_offset=off, routed_scaling_factor=rsf,
            routing_method=method, top_k=top_k,
            output_bf16_bits=out.view(torch.int16).numpy(),
            digest_keys=np.array(keys), digest_values=np.array([dig[k] for k in keys]),
            generator=f"flashinfer-python 0.6.11.post2 trace.templates.moe.{fn_name}",
            torch_version=torch.__version__,
        )
        print(name, tuple(out.shape), float(out.float().abs().max()))
        del inp, out


def main() -> None:
    from flashinfer.trace.templates.moe import _trtllm_fp8_block_scale_moe_ds_routing_reference as ext_ref

    torch.set_num_threads(os.cpu_count() or 1)
    for name, T, seed, variant, off, rsf in CASES:
        inp = workloads.make_inputs(T, seed, "cpu", variant, off, rsf)
        out = ext_ref(inp["routing_logits"], inp["routing_bias"], inp["hidden_states"],
                      inp["hidden_states_scale"], inp["gemm1_weights"], inp["gemm1_weights_scale"],
                      inp["gemm2_weights"], inp["gemm2_weights_scale"], 8, 8, 4, off, rsf)
        dig = input_digests(inp, range(workloads.E_LOCAL))
        keys = sorted(dig)
        np.savez_compressed(
            os.path.join(os.path.dirname(os.path.abspath(__file__)), f"{name}.npz"),
            T=T, seed=seed, variant=variant, local_expert_offset=off, routed_scaling_factor=rsf,
            output_bf16_bits=out.view(torch.int16).numpy(),
            digest_keys=np.array(keys), digest_values=np.array([dig[k] for k in keys]),
            generator="flashinfer-python 0.6.11.post2 "
                      "trace.templates.moe._trtllm_fp8_block_scale_moe_ds_routing_reference",
            torch_version=torch.__version__,
        )
        print(name, tuple(out.shape), float(out.float().abs().max()))
        del inp, out


if __name__ == "__main__":
    if "--routing" in sys.argv[1:]:
        main_routing()
    else:
        main()
