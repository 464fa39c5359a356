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
per rank; ``NvlinkCombiner`` (B200s + NVLink) keeps every shard's fp32
combine rows in a workspace that every rank maps (plain cudaMalloc buffers
shared through CUDA IPC handles, no multicast object) and forms the bf16
output on every rank with one kernel of the library
(moe_b200_ep_combine_shards: peer loads, an fp32 sum in shard order, one
bf16 rounding, peer stores).
"""
from __future__ import annotations

import ctypes

import torch
import torch.distributed as dist

E_GLOBAL = 256
E_LOCAL = 32
NUM_SHARDS = E_GLOBAL // E_LOCAL
STATUS_COMBINE_TIMEOUT = 1 << 7
STATUS_COMBINE_POISONED = 1 << 8


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


class _DeviceBytes:
    """A raw device allocation presented through the CUDA array interface,
    so torch can view it as a uint8 tensor without copying."""

    def __init__(self, ptr: int, nbytes: int):
        self.__cuda_array_interface__ = {"shape": (nbytes,), "typestr": "|u1", "data": (ptr, False),
                                         "strides": None, "version": 3}


def _round256(n: int) -> int:
    return (n + 255) // 256 * 256


class NvlinkCombiner:
    """``shards_per_rank`` 32-expert shards per rank, combined over NVLink.

    Each rank allocates one device buffer (moe_b200_ep_buffer_alloc: plain
    cudaMalloc, zero-filled) sized for ``max_tokens``: its EP area
    (counters + bf16 staging) followed by one layer workspace per shard.
    The buffers' IPC handles are exchanged through the process group and
    every rank maps every peer's buffer. ``forward_shards`` runs each of
    this rank's shards with the fp32 combine rows left in that shard's
    workspace, then ``moe_b200_ep_combine_shards`` writes the whole layer's
    bf16 output into ``out`` on every rank. Every rank must make the same
    calls with the same token count, in the same order. ``close`` is
    collective (it waits for every rank before freeing memory the peers map).
    """

    def __init__(self, max_tokens: int, device: torch.device, group=None, shards_per_rank: int = 1):
        import moe_host

        # without an initialised process group the combiner is a single rank
        # (all shards on this GPU, no peers)
        if group is None and dist.is_available() and dist.is_initialized():
            group = dist.group.WORLD
        self.group = group
        self.device = torch.device(device)
        self.max_tokens = int(max_tokens)
        self.shards_per_rank = int(shards_per_rank)
        self.rank = dist.get_rank(group) if group is not None else 0
        self.world = dist.get_world_size(group) if group is not None else 1
        if self.world * self.shards_per_rank > NUM_SHARDS or self.shards_per_rank < 1:
            raise ValueError(f"{self.world} ranks x {shards_per_rank} shards exceed {NUM_SHARDS} shards")
        area = moe_host.ep_area_bytes(self.max_tokens)
        layer = moe_host.workspace_bytes(self.max_tokens)
        if area == 0 or layer == 0:
            raise ValueError(f"max_tokens {max_tokens} out of range")
        self.area_bytes = _round256(area)
        self.ws_bytes = _round256(layer)
        self.nbytes = self.area_bytes + self.shards_per_rank * self.ws_bytes
        lib = moe_host.load_library()
        self._lib = lib
        self._closed = False
        self._opened: list[int] = []
        with torch.cuda.device(self.device):
            ptr = ctypes.c_void_p()
            moe_host._raise_on(lib.moe_b200_ep_buffer_alloc(self.nbytes, ctypes.byref(ptr)),
                               "moe_b200_ep_buffer_alloc")
            self._ptr = int(ptr.value)
            handle = ctypes.create_string_buffer(64)
            moe_host._raise_on(lib.moe_b200_ipc_get_handle(ctypes.c_void_p(self._ptr), handle),
                               "moe_b200_ipc_get_handle")
            handles = [None] * self.world
            if self.world > 1:
                dist.all_gather_object(handles, handle.raw, group=self.group)
            else:
                handles[0] = handle.raw
            bases = []
            for q, h in enumerate(handles):
                if q == self.rank:
                    bases.append(self._ptr)
                    continue
                peer = ctypes.c_void_p()
                moe_host._raise_on(lib.moe_b200_ipc_open_handle(ctypes.create_string_buffer(h, 64),
                                                                ctypes.byref(peer)), "moe_b200_ipc_open_handle")
                self._opened.append(int(peer.value))
                bases.append(int(peer.value))
            self.buf = torch.as_tensor(_DeviceBytes(self._ptr, self.nbytes), device=self.device)
            if self.buf.data_ptr() != self._ptr:
                raise RuntimeError("device buffer view does not alias the allocation")
        self.area_ptrs = bases
        self.ws_ptrs = [b + self.area_bytes + s * self.ws_bytes for b in bases for s in range(self.shards_per_rank)]
        self.area = self.buf[:self.area_bytes]
        self.workspaces = [self.buf[self.area_bytes + s * self.ws_bytes: self.area_bytes + (s + 1) * self.ws_bytes]
                           for s in range(self.shards_per_rank)]
        self.workspace = self.workspaces[0]
        torch.cuda.synchronize(self.device)
        self._barrier()

    def _barrier(self) -> None:
        if self.world > 1:
            dist.barrier(group=self.group)

    def run_shard(self, s: int, token_inputs: dict, w13, s13, w2, s2, local_expert_offset: int) -> None:
        """This rank's shard ``s``: the layer with its combine rows left in workspace ``s``."""
        import moe_host

        T = token_inputs["routing_logits"].shape[0]
        if T > self.max_tokens:
            raise ValueError(f"{T} tokens exceed the combiner's {self.max_tokens}")
        moe_host.run_dps(token_inputs["routing_logits"], token_inputs["routing_bias"],
                         token_inputs["hidden_states"], token_inputs["hidden_states_scale"], w13, s13, w2, s2,
                         local_expert_offset, token_inputs["routed_scaling_factor"], None,
                         workspace=self.workspaces[s])

    def combine(self, num_tokens: int, out: torch.Tensor) -> torch.Tensor:
        """The bf16 sum over every shard of every rank into ``out`` (this rank's)."""
        import moe_host

        return moe_host.ep_combine_shards(self.ws_ptrs, self.shards_per_rank, self.area_ptrs, self.rank,
                                          num_tokens, out)

    def forward_shards(self, token_inputs: dict, shards: list, out: torch.Tensor) -> torch.Tensor:
        """shards: this rank's (w13, s13, w2, s2, local_expert_offset), one per shard."""
        if len(shards) != self.shards_per_rank:
            raise ValueError(f"expected {self.shards_per_rank} shards, got {len(shards)}")
        for s, (w13, s13, w2, s2, off) in enumerate(shards):
            self.run_shard(s, token_inputs, w13, s13, w2, s2, off)
        return self.combine(token_inputs["routing_logits"].shape[0], out)

    def forward(self, token_inputs: dict, w13, s13, w2, s2, local_expert_offset: int,
                out: torch.Tensor) -> torch.Tensor:
        """One shard per rank."""
        return self.forward_shards(token_inputs, [(w13, s13, w2, s2, local_expert_offset)], out)

    def status(self) -> int:
        """OR of the status words of this rank's shard workspaces (the combine
        writes into the first one); synchronises the current stream."""
        import moe_host

        st = 0
        for ws in self.workspaces:
            st |= moe_host.read_status(ws)
        return st

    def reset(self) -> None:
        """Collective: clears every rank's combine counters after a combine
        gave up a wait (status bits 1 << 7 / 1 << 8)."""
        torch.cuda.synchronize(self.device)
        self._barrier()
        self.area[:256].zero_()
        torch.cuda.synchronize(self.device)
        self._barrier()

    def close(self) -> None:
        """Collective: unmaps the peers' buffers and frees this rank's, once
        every rank has finished using them."""
        if self._closed:
            return
        torch.cuda.synchronize(self.device)
        self._barrier()
        self.buf = self.area = self.workspace = None
        self.workspaces = []
        with torch.cuda.device(self.device):
            for p in self._opened:
                self._lib.moe_b200_ipc_close_handle(ctypes.c_void_p(p))
            self._opened = []
            torch.cuda.synchronize(self.device)
        self._barrier()
        with torch.cuda.device(self.device):
            self._lib.moe_b200_ep_buffer_free(ctypes.c_void_p(self._ptr))
        self._closed = True
