"""Expert parallelism over the 256 experts of the layer.

The operator's entry point handles 32 local experts per call, selected by
``local_expert_offset`` (reference: main.py:40, main.cpp:22,
kernel.cu:2473,2488 -- the reference has the argument but no communication).
Here the 8 shards of 32 experts are spread over the ranks of a process
group: rank r of N owns shards [8r/N, 8(r+1)/N). Every rank sees the same
tokens and computes the same routing; each computes the partial output of
its shards, and the partials are summed across ranks (NCCL all-reduce over
NVLink on B200, gloo on CPU).
"""
from __future__ import annotations

import torch
import torch.distributed as dist

E_GLOBAL = 256
E_LOCAL = 32
NUM_SHARDS = E_GLOBAL // E_LOCAL


def shard_offsets(world_size: int, rank: int) -> list[int]:
    """local_expert_offset values owned by `rank` (ranks must divide 8 shards evenly)."""
    if world_size < 1 or NUM_SHARDS % world_size != 0:
        raise ValueError(f"world size {world_size} must divide {NUM_SHARDS}")
    per = NUM_SHARDS // world_size
    return [E_LOCAL * s for s in range(rank * per, (rank + 1) * per)]


def ep_forward(layer_fn, token_inputs: dict, shard_weights: dict, group=None,
               reduce_dtype: torch.dtype = torch.float32) -> torch.Tensor:
    """Sum of the owned shards' partial outputs, then summed over the group.

    layer_fn(routing_logits, routing_bias, hidden_states, hidden_states_scale,
    w13, s13, w2, s2, local_expert_offset, routed_scaling_factor) -> [T, 7168]
    computes one 32-expert shard. token_inputs holds the token-side
    arguments; shard_weights maps each owned offset to (w13, s13, w2, s2).
    Returns the combined bf16 [T, 7168] output (identical on every rank).
    """
    acc = None
    for off, (w13, s13, w2, s2) in sorted(shard_weights.items()):
        part = layer_fn(token_inputs["routing_logits"], token_inputs["routing_bias"],
                        token_inputs["hidden_states"], token_inputs["hidden_states_scale"],
                        w13, s13, w2, s2, off, token_inputs["routed_scaling_factor"])
        part = part.to(reduce_dtype)
        acc = part if acc is None else acc + part
    if acc is None:
        T = token_inputs["routing_logits"].shape[0]
        acc = torch.zeros(T, 7168, dtype=reduce_dtype, device=token_inputs["routing_logits"].device)
    if group is not None and dist.get_world_size(group) > 1:
        dist.all_reduce(acc, op=dist.ReduceOp.SUM, group=group)
    return acc.to(torch.bfloat16)
