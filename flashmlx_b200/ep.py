"""Expert parallelism: one process per GPU, experts split across ranks, rows moved by
all-to-all collectives (NCCL over NVLink on GPUs, any torch.distributed backend).

The reference runs the whole MoE layer in one process (model.cpp:750-807); this module
has no reference counterpart.  One expert-parallel layer on rank r of W:

  1. dispatch   route the rank's T tokens; the T*k routed pairs in stable
                expert-major order, so the rows owned by each rank are contiguous
                (libflashmoe: fm_ep_dispatch)
  2. counts     all-to-all of the per-(owner, expert) pair counts
  3. rows       all-to-all of the token rows (H bf16 per pair)
  4. experts    the owner runs gate/up/down of its local experts on the rows it
                received, one tile group per (source rank, expert) segment, plus the
                shared expert on its own tokens (fm_ep_experts)
  5. return     all-to-all of bf16(d) back to the token's rank, in the order sent
  6. combine    y = sum_j bf16(d * score_j) in order j = 0..k-1, plus the gated shared
                expert (fm_ep_combine)

`ep_forward` is the protocol; the stage objects supply 1, 4 and 6 (DeviceStages: the
C ABI on this rank's GPU; the tests also drive it with an oracle on CPU ranks).

`MoEBlockEPPeer` runs the same layer with steps 2, 3 and 5 done by the kernels
themselves over NVLink peer memory (fm_ep_p2p_*): routed rows are written straight into
their owners' receive buffers and d rows straight back, ordered by epoch flags, with no
host synchronization and no collective library inside a call.
"""
from __future__ import annotations

import ctypes as C

import numpy as np
import torch
import torch.distributed as dist

__all__ = ["expert_range", "local_layer", "Exchange", "ep_forward", "DeviceStages", "MoEBlockEP", "MoEBlockEPPeer"]


def expert_range(num_experts: int, rank: int, world: int) -> tuple[int, int]:
    """(first, count) of the contiguous experts rank owns: the first E % W ranks own
    one expert more (the rule of fm_ep_range)."""
    if world <= 0 or not 0 <= rank < world or num_experts <= 0:
        raise ValueError("bad expert-parallel rank / world")
    base, rem = divmod(num_experts, world)
    return rank * base + min(rank, rem), base + (1 if rank < rem else 0)


def local_layer(layer: dict, rank: int, world: int) -> dict:
    """The arrays of one synthetic layer a rank keeps: router and shared expert whole,
    the stacked routed experts sliced to the rank's range."""
    E = layer["gate"][0].shape[0]
    first, count = expert_range(E, rank, world)
    out = dict(layer)
    for name in ("gate", "up", "down"):
        w, s, b = layer[name]
        out[name] = (w[first:first + count], s[first:first + count], None if b is None else b[first:first + count])
    return out


class Exchange:
    """The collectives of an expert-parallel layer on a torch.distributed group.  Rows
    travel on `device` (CUDA for NCCL, CPU for gloo)."""

    def __init__(self, num_experts: int, group=None, device=None):
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.E = num_experts
        self.ranges = [expert_range(num_experts, r, self.world) for r in range(self.world)]
        self.E_local = self.ranges[self.rank][1]
        self.device = device

    def send_splits(self, expert_counts) -> list[int]:
        """Pairs bound for each owner (expert_counts: pairs per global expert)."""
        c = [int(v) for v in expert_counts]
        return [sum(c[f:f + n]) for f, n in self.ranges]

    def exchange_counts(self, expert_counts) -> list[int]:
        """Rows this rank receives per (source rank, local expert), source-major."""
        send = torch.as_tensor(np.asarray(expert_counts, dtype=np.int32), device=self.device)
        recv = torch.empty(self.world * self.E_local, dtype=torch.int32, device=self.device)
        dist.all_to_all_single(recv, send, output_split_sizes=[self.E_local] * self.world,
                               input_split_sizes=[n for _, n in self.ranges], group=self.group)
        return [int(v) for v in recv.cpu()]

    def recv_splits(self, recv_counts) -> list[int]:
        e = self.E_local
        return [sum(recv_counts[s * e:(s + 1) * e]) for s in range(self.world)]

    def all_to_all(self, rows: torch.Tensor, send_splits, recv_splits) -> torch.Tensor:
        """Rows [n, H] (2-byte elements, H even) move as int32 pairs, a type every backend
        carries (gloo has no 16-bit types)."""
        rows = rows.contiguous()
        wide = rows.view(torch.int32)
        out = torch.empty((sum(recv_splits),) + tuple(wide.shape[1:]), dtype=torch.int32, device=rows.device)
        dist.all_to_all_single(out, wide, output_split_sizes=list(recv_splits),
                               input_split_sizes=list(send_splits), group=self.group)
        return out.view(rows.dtype)


def ep_forward(stages, exch: Exchange, x):
    """One expert-parallel MoE layer for this rank's tokens x (see the module doc)."""
    counts, send = stages.dispatch(x)
    send_splits = exch.send_splits(counts)
    recv_counts = exch.exchange_counts(counts)
    recv_splits = exch.recv_splits(recv_counts)
    recv = exch.all_to_all(send, send_splits, recv_splits)
    d = stages.experts(recv, recv_counts)
    ret = exch.all_to_all(d, recv_splits, send_splits)
    return stages.combine(ret)


class _DeviceRows:
    """A [rows, H] bf16 view of library-owned device memory (via the CUDA array
    interface; int16 storage, viewed as bfloat16)."""

    def __init__(self, ptr: int, rows: int, cols: int):
        self.__cuda_array_interface__ = {"shape": (rows, cols), "typestr": "<i2", "data": (ptr, False),
                                         "version": 3, "strides": None}


class DeviceStages:
    """Stages 1, 4 and 6 on libflashmoe (fm_ep_dispatch / fm_ep_experts / fm_ep_combine)
    for one rank.  `weights` holds the router and shared expert whole and the rank's
    local experts stacked (see local_layer)."""

    def __init__(self, shape, weights, rank: int, world: int, handle=None):
        from . import ops
        self.shape = shape
        self.block = ops.MoEBlock(shape, weights, handle)  # config + weight structs
        self.rank, self.world = rank, world
        self._h = handle
        self._T = 0

    def _handle(self, device):
        from . import ops
        h = self._h or ops.default_handle(device.index)
        h.bind_stream()
        h.check(h.lib.fm_ep_set(h.h, self.rank, self.world))
        return h

    def dispatch(self, x: torch.Tensor):
        H, E, k = self.shape.hidden, self.shape.num_experts, self.shape.top_k
        if x.dtype != torch.bfloat16 or not x.is_cuda or x.shape[-1] != H:
            raise ValueError("x must be a CUDA bf16 tensor [T, hidden]")
        x = x.contiguous()
        h = self._handle(x.device)
        T = x.numel() // H
        counts = (C.c_int32 * E)()
        send = C.c_void_p()
        h.check(h.lib.fm_ep_dispatch(h.h, C.byref(self.block.cfg), C.byref(self.block.W), C.c_void_p(x.data_ptr()),
                                     T, counts, C.byref(send)))
        self._T, self._dev, self._h_active = T, x.device, h
        P = T * k
        rows = (torch.as_tensor(_DeviceRows(send.value or 0, P, H), device=x.device).view(torch.bfloat16)
                if P else torch.empty(0, H, dtype=torch.bfloat16, device=x.device))
        return list(counts), rows

    def experts(self, recv: torch.Tensor, recv_counts) -> torch.Tensor:
        h = self._h_active
        H = self.shape.hidden
        d = torch.empty(recv.shape[0], H, dtype=torch.bfloat16, device=self._dev)
        rc = (C.c_int32 * len(recv_counts))(*recv_counts)
        h.check(h.lib.fm_ep_experts(h.h, C.byref(self.block.cfg), C.byref(self.block.W),
                                    C.c_void_p(recv.data_ptr() if recv.numel() else 0), rc,
                                    C.c_void_p(d.data_ptr() if d.numel() else 0)))
        return d

    def combine(self, ret: torch.Tensor) -> torch.Tensor:
        h = self._h_active
        y = torch.empty(self._T, self.shape.hidden, dtype=torch.bfloat16, device=self._dev)
        h.check(h.lib.fm_ep_combine(h.h, C.byref(self.block.cfg), C.c_void_p(ret.data_ptr() if ret.numel() else 0),
                                    C.c_void_p(y.data_ptr() if y.numel() else 0)))
        return y


class MoEBlockEP:
    """LlamaModel::moe_block with its experts split across the ranks of a process group
    (one process per GPU).  Every rank calls it collectively with its own tokens."""

    def __init__(self, shape, local_weights, group=None, handle=None):
        world = dist.get_world_size(group)
        rank = dist.get_rank(group)
        self.stages = DeviceStages(shape, local_weights, rank, world, handle)
        self.exchange = Exchange(shape.num_experts, group, device=local_weights.router_w.device)

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        return ep_forward(self.stages, self.exchange, x)


class MoEBlockEPPeer:
    """LlamaModel::moe_block with its experts split across the ranks of a process group
    (one process per GPU of one NVLink domain, at most 8) and the rows moved over peer
    memory by the kernels (fm_ep_p2p_*).  Constructed collectively: every rank allocates
    its exchange region for up to `max_tokens` tokens per call and the CUDA IPC handles
    travel once over the group.  Every rank then makes the same sequence of calls, each
    with its own tokens; `close` (collective) releases the regions."""

    def __init__(self, shape, local_weights, max_tokens: int, group=None):
        from . import ops
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.shape = shape
        self.device = local_weights.router_w.device
        self.block = ops.MoEBlock(shape, local_weights)  # config + weight structs
        self.h = ops.Handle(self.device.index)  # owns the region: one per layer object
        self.h.bind_stream()
        lib = self.h.lib
        self.h.check(lib.fm_ep_set(self.h.h, self.rank, self.world))
        ipc = (C.c_uint8 * 64)()
        self.h.check(lib.fm_ep_p2p_alloc(self.h.h, C.byref(self.block.cfg), int(max_tokens), ipc))
        key = (shape.hidden, shape.num_experts, shape.top_k, int(max_tokens))
        got = [None] * self.world
        dist.all_gather_object(got, (bytes(ipc), key), group=group)
        if any(k != key for _, k in got):
            self.h.check(lib.fm_ep_p2p_close(self.h.h))
            raise ValueError("ranks disagree on (hidden, num_experts, top_k, max_tokens)")
        handles = b"".join(b for b, _ in got)
        self.h.check(lib.fm_ep_p2p_open(self.h.h, handles))
        dist.barrier(group)
        self.max_tokens = int(max_tokens)

    def __call__(self, x: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        H = self.shape.hidden
        if x.dtype != torch.bfloat16 or x.device != self.device or x.shape[-1] != H:
            raise ValueError("x must be a bf16 tensor [T, hidden] on this rank's device")
        x = x.contiguous()
        T = x.numel() // H
        y = out if out is not None else torch.empty_like(x)
        self.h.bind_stream()
        self.h.check(self.h.lib.fm_ep_p2p_forward(self.h.h, C.byref(self.block.cfg), C.byref(self.block.W),
                                                  C.c_void_p(x.data_ptr() if T else 0), T,
                                                  C.c_void_p(y.data_ptr() if T else 0)))
        return y

    def sync(self):
        """Wait for this rank's calls and raise on a device-side error (a peer that did not
        take part shows up here as a timeout)."""
        self.h.sync()

    def close(self):
        """Collective: every rank's calls complete, then the regions are unmapped and freed."""
        if self.h is None:
            return
        torch.cuda.synchronize(self.device)
        dist.barrier(self.group)
        self.h.check(self.h.lib.fm_ep_p2p_close(self.h.h))
        self.h.close()
        self.h = None
