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


class PeerBuffers:
    """One device buffer per rank, mapped in every rank's process.

    Each rank allocates ``nbytes`` of plain cudaMalloc memory
    (moe_b200_ep_buffer_alloc, zero-filled), the buffers' CUDA IPC handles
    are exchanged through the process group and every rank opens the peers'
    (peer access enabled); no multicast object is created. ``ptrs[q]`` is
    rank q's buffer in this process, ``buf`` this rank's own as a uint8
    tensor. ``close`` is collective: it waits for every rank before
    unmapping and freeing, since the peers may still read this memory.
    Without an initialised process group it is a single rank.
    """

    def __init__(self, nbytes: int, device: torch.device, group=None):
        import moe_host

        if group is None and dist.is_available() and dist.is_initialized():
            group = dist.group.WORLD
        self.group = group
        self.device = torch.device(device)
        self.rank = dist.get_rank(group) if group is not None else 0
        self.world = dist.get_world_size(group) if group is not None else 1
        self.nbytes = int(nbytes)
        self._lib = moe_host.load_library()
        self._closed = False
        self._opened: list[int] = []
        with torch.cuda.device(self.device):
            ptr = ctypes.c_void_p()
            moe_host._raise_on(self._lib.moe_b200_ep_buffer_alloc(self.nbytes, ctypes.byref(ptr)),
                               "moe_b200_ep_buffer_alloc")
            self._ptr = int(ptr.value)
            handle = ctypes.create_string_buffer(64)
            moe_host._raise_on(self._lib.moe_b200_ipc_get_handle(ctypes.c_void_p(self._ptr), handle),
                               "moe_b200_ipc_get_handle")
            handles = [None] * self.world
            if self.world > 1:
                dist.all_gather_object(handles, handle.raw, group=self.group)
            else:
                handles[0] = handle.raw
            ptrs = []
            for q, h in enumerate(handles):
                if q == self.rank:
                    ptrs.append(self._ptr)
                    continue
                peer = ctypes.c_void_p()
                moe_host._raise_on(self._lib.moe_b200_ipc_open_handle(ctypes.create_string_buffer(h, 64),
                                                                      ctypes.byref(peer)),
                                   "moe_b200_ipc_open_handle")
                self._opened.append(int(peer.value))
                ptrs.append(int(peer.value))
            self.buf = torch.as_tensor(_DeviceBytes(self._ptr, self.nbytes), device=self.device)
            if self.buf.data_ptr() != self._ptr:
                raise RuntimeError("device buffer view does not alias the allocation")
        self.ptrs = ptrs
        torch.cuda.synchronize(self.device)
        self.barrier()

    def barrier(self) -> None:
        if self.world > 1:
            dist.barrier(group=self.group)

    def close(self) -> None:
        if self._closed:
            return
        torch.cuda.synchronize(self.device)
        self.barrier()
        self.buf = None
        with torch.cuda.device(self.device):
            for p in self._opened:
                self._lib.moe_b200_ipc_close_handle(ctypes.c_void_p(p))
            self._opened = []
            torch.cuda.synchronize(self.device)
        self.barrier()
        with torch.cuda.device(self.device):
            self._lib.moe_b200_ep_buffer_free(ctypes.c_void_p(self._ptr))
        self._closed = True


class NvlinkCombiner:
    """``shards_per_rank`` 32-expert shards per rank, combined over NVLink.

    Each rank's PeerBuffers buffer, sized for ``max_tokens``, holds its EP
    area (counters + bf16 staging) followed by one layer workspace per shard.
    ``forward_shards`` runs each of this rank's shards with the fp32 combine
    rows left in that shard's workspace, then ``moe_b200_ep_combine_shards``
    writes the whole layer's bf16 output into ``out`` on every rank. Every
    rank must make the same calls with the same token count, in the same
    order. ``close`` is collective.
    """

    def __init__(self, max_tokens: int, device: torch.device, group=None, shards_per_rank: int = 1):
        import moe_host

        self.max_tokens = int(max_tokens)
        self.shards_per_rank = int(shards_per_rank)
        area = moe_host.ep_area_bytes(self.max_tokens)
        layer = moe_host.workspace_bytes(self.max_tokens)
        if area == 0 or layer == 0:
            raise ValueError(f"max_tokens {max_tokens} out of range")
        if self.shards_per_rank < 1:
            raise ValueError("shards_per_rank must be at least 1")
        self.area_bytes = _round256(area)
        self.ws_bytes = _round256(layer)
        self.peers = PeerBuffers(self.area_bytes + self.shards_per_rank * self.ws_bytes, device, group)
        self.device, self.rank, self.world = self.peers.device, self.peers.rank, self.peers.world
        if self.world * self.shards_per_rank > NUM_SHARDS:
            self.peers.close()
            raise ValueError(f"{self.world} ranks x {shards_per_rank} shards exceed {NUM_SHARDS} shards")
        bases = self.peers.ptrs
        self.area_ptrs = bases
        self.ws_ptrs = [b + self.area_bytes + s * self.ws_bytes for b in bases for s in range(self.shards_per_rank)]
        buf = self.peers.buf
        self.area = buf[:self.area_bytes]
        self.workspaces = [buf[self.area_bytes + s * self.ws_bytes: self.area_bytes + (s + 1) * self.ws_bytes]
                           for s in range(self.shards_per_rank)]
        self.workspace = self.workspaces[0]

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
        """Collective: clears every rank's EP area (combine counters and
        flagged lines) after a combine gave up a wait (status bits 1 << 7 /
        1 << 8)."""
        torch.cuda.synchronize(self.device)
        self.peers.barrier()
        self.area.zero_()
        torch.cuda.synchronize(self.device)
        self.peers.barrier()

    def close(self) -> None:
        """Collective: unmaps the peers' buffers and frees this rank's."""
        self.area = self.workspace = None
        self.workspaces = []
        self.peers.close()


class TokenParallelEP:
    """Token-parallel expert parallelism (all-to-all dispatch and combine).

    Every rank holds its own tokens (up to ``max_tokens`` per call, a
    different batch on every rank) and owns S = 8 / world 32-expert shards:
    rank q owns global experts [32 S q, 32 S (q + 1)). One ``forward``:
    route the own tokens over all 256 experts (moe_b200_route), dispatch
    every token once to each rank it has picks on (moe_b200_a2a_dispatch:
    the token's e4m3 row, its 56 block scales and its picks on that rank,
    written by peer stores into that rank's receive slab), run each owned
    shard on the received rows with the given routing (moe_b200_run_routed
    with 8 picks per row; its combine rows stay in the shard's workspace),
    and combine (moe_b200_a2a_combine: each own token's output is the fp32
    sum of its combine rows on the destination ranks' shards, each rank's
    shards in shard order and then the ranks in rank order, rounded once to
    bf16).

    Each rank's PeerBuffers buffer holds the all-to-all area (counters,
    send plan, receive slab of ``recv_capacity`` rows) and one layer
    workspace per shard sized for the slab. ``recv_capacity`` defaults to
    world * max_tokens, which can never overflow. Every rank must call
    ``forward`` the same number of times (with any token count up to
    ``max_tokens``, also zero). ``close`` is collective.
    """

    def __init__(self, max_tokens: int, device: torch.device, group=None, recv_capacity: int | None = None):
        import moe_host

        world = dist.get_world_size(group) if group is not None else (
            dist.get_world_size() if dist.is_available() and dist.is_initialized() else 1)
        if NUM_SHARDS % world != 0:
            raise ValueError(f"world size {world} must divide {NUM_SHARDS}")
        self.max_tokens = int(max_tokens)
        self.shards_per_rank = NUM_SHARDS // world
        self.cap = int(recv_capacity) if recv_capacity is not None else world * self.max_tokens
        a2a = moe_host.a2a_area_bytes(self.max_tokens, self.cap)
        layer = moe_host.routed_workspace_bytes(self.cap, 8)
        if a2a == 0 or layer == 0:
            raise ValueError(f"max_tokens {max_tokens} / recv_capacity {self.cap} out of range")
        self.a2a_bytes = _round256(a2a)
        self.ws_bytes = _round256(layer)
        self.layout = moe_host.a2a_layout(self.max_tokens, self.cap)
        self.peers = PeerBuffers(self.a2a_bytes + self.shards_per_rank * self.ws_bytes, device, group)
        self.device, self.rank, self.world = self.peers.device, self.peers.rank, self.peers.world
        bases = self.peers.ptrs
        self.area_ptrs = bases
        self.ws_ptrs = [b + self.a2a_bytes + s * self.ws_bytes for b in bases for s in range(self.shards_per_rank)]
        buf = self.peers.buf
        self.area = buf[:self.a2a_bytes]
        self.workspaces = [buf[self.a2a_bytes + s * self.ws_bytes: self.a2a_bytes + (s + 1) * self.ws_bytes]
                           for s in range(self.shards_per_rank)]
        self.topk_idx = torch.empty(self.max_tokens, 8, dtype=torch.int32, device=self.device)
        self.topk_w = torch.empty(self.max_tokens, 8, dtype=torch.float32, device=self.device)

    def shard_offsets(self) -> list[int]:
        """local_expert_offset of each of this rank's shards."""
        return [E_LOCAL * (self.rank * self.shards_per_rank + s) for s in range(self.shards_per_rank)]

    def slab_rows(self) -> int:
        """Rows received by the last dispatch (synchronises)."""
        import moe_host

        return moe_host.a2a_read_status(self.area)[1]

    def status(self) -> int:
        """OR of the all-to-all status word and the shard workspaces' status words."""
        import moe_host

        st = moe_host.a2a_read_status(self.area)[0]
        for ws in self.workspaces:
            st |= moe_host.read_status(ws)
        return st

    def reset(self) -> None:
        """Collective: clears every rank's counter block after an all-to-all
        wait gave up (status bits 1 << 7 / 1 << 8); call numbers restart."""
        import moe_host

        torch.cuda.synchronize(self.device)
        self.peers.barrier()
        self.area[:moe_host.A2A_COUNTER_BYTES].zero_()
        torch.cuda.synchronize(self.device)
        self.peers.barrier()

    def forward(self, token_inputs: dict, shards: list, out: torch.Tensor) -> torch.Tensor:
        """token_inputs: this rank's routing_logits [T, 256], routing_bias,
        hidden_states e4m3 [T, 7168], hidden_states_scale [56, T],
        routed_scaling_factor; shards: this rank's (w13, s13, w2, s2) in
        shard order. Writes this rank's bf16 [T, 7168] output into ``out``."""
        import moe_host

        if len(shards) != self.shards_per_rank:
            raise ValueError(f"expected {self.shards_per_rank} shards, got {len(shards)}")
        T = int(token_inputs["routing_logits"].shape[0])
        if T > self.max_tokens:
            raise ValueError(f"{T} tokens exceed max_tokens {self.max_tokens}")
        idx, w = self.topk_idx[:T], self.topk_w[:T]
        if T > 0:
            ri, rw = moe_host.route(token_inputs["routing_logits"], token_inputs["routing_bias"],
                                    token_inputs["routed_scaling_factor"])
            idx.copy_(ri)
            w.copy_(rw)
        hs = token_inputs["hidden_states"]
        hss = token_inputs["hidden_states_scale"].contiguous()
        moe_host.a2a_dispatch(idx, w, hs, hss, self.max_tokens, self.cap, self.area_ptrs, self.rank,
                              self.shards_per_rank)
        base = self.peers.buf.data_ptr()
        lay = self.layout
        for s, (w13, s13, w2, s2) in enumerate(shards):
            moe_host.run_routed_ptrs(base + lay.slab_idx, base + lay.slab_w, 8, base + lay.slab_rows,
                                     base + lay.slab_scale, w13, s13, w2, s2,
                                     E_LOCAL * (self.rank * self.shards_per_rank + s), self.cap,
                                     self.workspaces[s])
        return moe_host.a2a_combine(idx, self.ws_ptrs, self.area_ptrs, self.rank, self.shards_per_rank,
                                    self.max_tokens, self.cap, out)

    def dest_rows(self, T: int) -> torch.Tensor:
        """int32 [T, world]: the slab row of each of this rank's tokens on
        every destination rank (-1 where it has no pick), from the last
        dispatch."""
        lay = self.layout
        return self.area[lay.dest_row: lay.dest_row + 4 * T * 8].view(torch.int32).view(T, 8)[:, :self.world]

    def close(self) -> None:
        """Collective: unmaps the peers' buffers and frees this rank's."""
        self.area = None
        self.workspaces = []
        self.peers.close()
