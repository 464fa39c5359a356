"""Seeded synthetic inputs for the MoE layer (the contest dataset is not
available, so these stand in for its workloads).

Distributions follow the benchmark configurations of this build:

* ``routing_logits`` fp32 [T, 256] ~ N(0, 1)
* ``routing_bias``   bf16 [256] = bf16(N(0, 0.1)); the "hot" variant adds
  +1.0 to four experts inside the local range (local ids 3, 11, 19, 27)
* ``hidden_states``  bf16 N(0, 1) quantised per 1x128 block to e4m3 with
  fp32 scale amax/448, scales stored block-major [56, T]
* ``gemm1_weights``  N(0, 0.02) [32, 4096, 7168] quantised per 128x128
  block, scales [32, 32, 56]; ``gemm2_weights`` likewise [32, 7168, 2048],
  scales [32, 56, 16]
* the "zipf" variant adds alpha * log p(rank) to the logits, p a Zipf(1.2)
  law over a seeded permutation of the 256 experts (alpha = 1.0)

Every tensor is drawn from its own seeded generator, so a subset of experts
can be materialised on its own (the CPU tests build only the experts that
the routing activates; the others stay zero and are never read).
"""
from __future__ import annotations

import torch

H = 7168
I = 2048
E_GLOBAL = 256
E_LOCAL = 32
BLOCK = 128
FP8_MAX = 448.0
HOT_LOCAL_EXPERTS = (3, 11, 19, 27)
ZIPF_S = 1.2
ZIPF_ALPHA = 1.0

_PIECE_LOGITS = 1
_PIECE_BIAS = 2
_PIECE_HIDDEN = 3
_PIECE_ZIPF = 4
_PIECE_W13 = 1000
_PIECE_W2 = 2000


def _gen(seed: int, piece: int, device) -> torch.Generator:
    g = torch.Generator(device=device)
    g.manual_seed(seed * 100003 + piece)
    return g


def quantize_rows_1x128(x: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """x [T, H] -> (e4m3 [T, H], fp32 scales [H/128, T]) with scale = amax/448."""
    T, h = x.shape
    xb = x.float().view(T, h // BLOCK, BLOCK)
    amax = xb.abs().amax(dim=2)
    scale = torch.where(amax > 0, amax / FP8_MAX, torch.ones_like(amax))
    q = (xb / scale.unsqueeze(2)).to(torch.float8_e4m3fn).view(T, h)
    return q, scale.t().contiguous()


def quantize_blocks_128x128(w: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """w [R, C] fp32 -> (e4m3 [R, C], fp32 scales [R/128, C/128])."""
    R, C = w.shape
    wb = w.view(R // BLOCK, BLOCK, C // BLOCK, BLOCK)
    amax = wb.abs().amax(dim=(1, 3))
    scale = torch.where(amax > 0, amax / FP8_MAX, torch.ones_like(amax))
    q = (wb / scale[:, None, :, None]).to(torch.float8_e4m3fn).view(R, C)
    return q, scale


def make_routing_inputs(T: int, seed: int = 0, device="cpu", variant: str = "uniform",
                        local_expert_offset: int = 0) -> dict:
    """routing_logits fp32 [T, 256] and routing_bias bf16 [256]."""
    logits = torch.randn(T, E_GLOBAL, generator=_gen(seed, _PIECE_LOGITS, device), device=device)
    bias = torch.randn(E_GLOBAL, generator=_gen(seed, _PIECE_BIAS, device), device=device) * 0.1
    if variant == "hot":
        for le in HOT_LOCAL_EXPERTS:
            bias[local_expert_offset + le] += 1.0
    elif variant == "zipf":
        g = _gen(seed, _PIECE_ZIPF, "cpu")
        perm = torch.randperm(E_GLOBAL, generator=g)
        ranks = torch.empty(E_GLOBAL, dtype=torch.float64)
        ranks[perm] = torch.arange(1, E_GLOBAL + 1, dtype=torch.float64)
        p = ranks.pow(-ZIPF_S)
        p = p / p.sum()
        logits = logits + (ZIPF_ALPHA * p.log()).to(torch.float32).to(device)
    elif variant != "uniform":
        raise ValueError(f"unknown routing variant {variant!r}")
    return {"routing_logits": logits.contiguous(), "routing_bias": bias.to(torch.bfloat16)}


def make_hidden_bf16(T: int, seed: int = 0, device="cpu") -> torch.Tensor:
    """The bf16 [T, 7168] hidden states that make_hidden quantises."""
    return torch.randn(T, H, generator=_gen(seed, _PIECE_HIDDEN, device), device=device).to(torch.bfloat16)


def make_hidden(T: int, seed: int = 0, device="cpu") -> tuple[torch.Tensor, torch.Tensor]:
    return quantize_rows_1x128(make_hidden_bf16(T, seed, device))


def make_expert_weights(seed: int, le: int, device="cpu"):
    """(w13 e4m3 [4096, 7168], s13 [32, 56], w2 e4m3 [7168, 2048], s2 [56, 16]) of local expert le."""
    w13 = torch.randn(2 * I, H, generator=_gen(seed, _PIECE_W13 + le, device), device=device) * 0.02
    q13, s13 = quantize_blocks_128x128(w13)
    del w13
    w2 = torch.randn(H, I, generator=_gen(seed, _PIECE_W2 + le, device), device=device) * 0.02
    q2, s2 = quantize_blocks_128x128(w2)
    return q13, s13, q2, s2


def make_inputs(T: int, seed: int = 0, device="cpu", variant: str = "uniform",
                local_expert_offset: int = 0, routed_scaling_factor: float = 2.5,
                experts=None, weight_seed: int | None = None) -> dict:
    """All ten arguments of run(...). ``experts`` lists the local experts whose
    weights are materialised (default: all 32); the others are zero.
    ``weight_seed`` (default ``seed``) seeds the expert weights separately,
    so expert-parallel ranks can share tokens but own different experts."""
    wseed = seed if weight_seed is None else weight_seed
    device = torch.device(device)
    out = make_routing_inputs(T, seed, device, variant, local_expert_offset)
    hs, hs_scale = make_hidden(T, seed, device)
    w13 = torch.zeros(E_LOCAL, 2 * I, H, dtype=torch.float8_e4m3fn, device=device)
    s13 = torch.ones(E_LOCAL, 2 * I // BLOCK, H // BLOCK, dtype=torch.float32, device=device)
    w2 = torch.zeros(E_LOCAL, H, I, dtype=torch.float8_e4m3fn, device=device)
    s2 = torch.ones(E_LOCAL, H // BLOCK, I // BLOCK, dtype=torch.float32, device=device)
    for le in (range(E_LOCAL) if experts is None else experts):
        q13, sc13, q2, sc2 = make_expert_weights(wseed, le, device)
        w13[le].copy_(q13)
        s13[le].copy_(sc13)
        w2[le].copy_(q2)
        s2[le].copy_(sc2)
        del q13, q2
    out.update(
        hidden_states=hs,
        hidden_states_scale=hs_scale,
        gemm1_weights=w13,
        gemm1_weights_scale=s13,
        gemm2_weights=w2,
        gemm2_weights_scale=s2,
        local_expert_offset=local_expert_offset,
        routed_scaling_factor=routed_scaling_factor,
    )
    return out


ARG_ORDER = (
    "routing_logits",
    "routing_bias",
    "hidden_states",
    "hidden_states_scale",
    "gemm1_weights",
    "gemm1_weights_scale",
    "gemm2_weights",
    "gemm2_weights_scale",
    "local_expert_offset",
    "routed_scaling_factor",
)


def as_args(inputs: dict) -> list:
    """The inputs in the positional order of run(...)."""
    return [inputs[k] for k in ARG_ORDER]
