"""Expert parallelism over the 256 experts of the layer.

The operator's entry point handles 32 local experts per call, selected by
``local_expert_offset`` (reference: main.py:40, main.cpp:22,
kernel.cu:2473,2488 -- the reference has the argument but no communication).
Here the 8 shards of 32 experts are spread over the ranks of a process
group: rank r of N owns shards [8r/N, 8(r+1)/N). Every rank sees the same
tokens and computes the same routing; each computes the partial output of
its shards, and the partials are summed across ranks.

Two forms: ``ep_forward`` sums bf16/fp32 partial outputs with a collective
of the process group (gloo on CPU, NCCL on GPUs) for any number of shards
per rank; ``NvlinkCombiner`` (one shard per rank, B200 + NVLink) keeps each
rank's fp32 combine rows in a workspace that every rank maps (symmetric
memory) and forms the bf16 output on every rank with one kernel of the
library (moe_b200_ep_combine: peer loads, an fp32 sum, one bf16 rounding,
peer stores).
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


class NvlinkCombiner:
    """One 32-expert shard per rank, combined over NVLink by the library.

    One symmetric-memory allocation per rank (mapped in every process of
    the group), sized for ``max_tokens``, holds the EP area (counters +
    staging, at offset 0) and the layer workspace after it; ``forward`` runs
    this rank's shard with the fp32 combine rows left in the workspace and
    then ``moe_b200_ep_combine``, which writes the whole layer's bf16 output
    into ``out`` on every rank. Every rank must call ``forward`` with the
    same token count, in the same order.
    """

    def __init__(self, max_tokens: int, device: torch.device, group=None):
        import moe_host
        import torch.distributed._symmetric_memory as symm_mem

        group = group if group is not None else dist.group.WORLD
        self.device = device
        self.max_tokens = int(max_tokens)
        area = moe_host.ep_area_bytes(self.max_tokens)
        layer = moe_host.workspace_bytes(self.max_tokens)
        if area == 0 or layer == 0:
            raise ValueError(f"max_tokens {max_tokens} out of range")
        self.ws_off = (area + 255) // 256 * 256
        nbytes = self.ws_off + layer
        self.buf = symm_mem.empty(nbytes, dtype=torch.uint8, device=device)
        self.buf.zero_()   # the EP area's counters start at zero
        self.handle = symm_mem.rendezvous(self.buf, group)
        self.rank = int(self.handle.rank)
        self.world = int(self.handle.world_size)
        self.area_ptrs = [int(p) for p in self.handle.buffer_ptrs]
        self.ws_ptrs = [p + self.ws_off for p in self.area_ptrs]
        self.workspace = self.buf[self.ws_off:]
        torch.cuda.synchronize(device)
        dist.barrier(group)

    def forward(self, token_inputs: dict, w13, s13, w2, s2, local_expert_offset: int,
                out: torch.Tensor) -> torch.Tensor:
        import moe_host

        T = token_inputs["routing_logits"].shape[0]
        if T > self.max_tokens:
            raise ValueError(f"{T} tokens exceed the combiner's {self.max_tokens}")
        moe_host.run_dps(token_inputs["routing_logits"], token_inputs["routing_bias"],
                         token_inputs["hidden_states"], token_inputs["hidden_states_scale"], w13, s13, w2, s2,
                         local_expert_offset, token_inputs["routed_scaling_factor"], None,
                         workspace=self.workspace)
        return moe_host.ep_combine(self.ws_ptrs, self.area_ptrs, self.rank, T, out)
