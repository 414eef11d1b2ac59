"""A CPU model of the peer-memory expert-parallel layer (fm_ep_p2p_forward), for tests.

Every rank owns one region with the device layout of flashmlx_b200/csrc/ep.cu -- flags
[3][W] u32 (per kind and source rank, the epoch of the last post), board [W][E] i32,
recv [cap_recv][H] and ret [cap_ret][H] bf16 rows -- here in POSIX shared memory that
every rank process maps.  One call (epoch e) on rank r runs the steps of the kernels with
their index arithmetic restated:

  dispatch  (ep_dispatch_kernel)     post r's per-expert counts into every board and
                                     flag 0; wait for flag 0 of all ranks; write each
                                     routed row into its owner's recv at the offset the
                                     board gives (owner o's rows from r follow those of
                                     ranks < r), walking the rows from r's own owner on;
                                     flag 1 on every rank
  plan      (ep_p2p_plan_kernel)     as an owner, wait for flag 1 of all sources; the
                                     (source, local expert) counts and, per received row,
                                     its source and position in that source's send order
  experts   (the expert GEMMs)       d rows of the received rows, each stored straight
                                     into its source's ret row
  release   (ep_release_kernel)      flag 2 on every rank
  combine   (ep_combine_p2p_kernel)  wait for flag 2 of all owners; y from ret

The expert arithmetic comes from the CPU oracle (the stages object); what the model
checks is the exchange: where rows land, the counts, and that the epoch flags order the
calls so that no region is overwritten while another rank still reads it.  Waits are
bounded: a wait that runs out returns False, as the device waits record FM_ETIMEOUT.
Test infrastructure only."""
from __future__ import annotations

import time
from multiprocessing import shared_memory

import numpy as np


def owner_range(E: int, r: int, W: int) -> tuple[int, int]:
    """(first, count) of rank r's experts (fm_ep.cuh: ep_owner_range)."""
    base, rem = divmod(E, W)
    return r * base + min(r, rem), base + (1 if r < rem else 0)


class Layout:
    """Byte layout of one rank's region (ep.cu, fm_ep_p2p_alloc): cap_recv = W *
    max_tokens * min(k, ceil(E / W)) rows, cap_ret = max_tokens * k rows."""

    def __init__(self, W: int, E: int, k: int, H: int, max_tokens: int):
        self.W, self.E, self.k, self.H = W, E, k, H
        self.cap_recv = W * max_tokens * min(k, -(-E // W))
        self.cap_ret = max_tokens * k
        off = 0

        def take(nbytes):
            nonlocal off
            start = off
            off = (off + nbytes + 255) // 256 * 256
            return start
        self.off_flags = take(3 * W * 4)
        self.off_board = take(W * E * 4)
        self.off_recv = take(self.cap_recv * H * 2)
        self.off_ret = take(self.cap_ret * H * 2)
        self.nbytes = off


class Region:
    """Views of one rank's region in a shared-memory block."""

    def __init__(self, shm: shared_memory.SharedMemory, lay: Layout):
        b = shm.buf
        self.flags = np.ndarray((3, lay.W), np.uint32, b, lay.off_flags)
        self.board = np.ndarray((lay.W, lay.E), np.int32, b, lay.off_board)
        self.recv = np.ndarray((lay.cap_recv, lay.H), np.uint16, b, lay.off_recv)
        self.ret = np.ndarray((lay.cap_ret, lay.H), np.uint16, b, lay.off_ret)


class PeerRank:
    """One rank of the model: `regions[q]` is rank q's region as this rank maps it."""

    def __init__(self, rank: int, lay: Layout, regions: list[Region], wait_s: float = 10.0, jitter=None,
                 planted_early_release: bool = False):
        self.me, self.lay, self.regions, self.wait_s = rank, lay, regions, wait_s
        self.jitter = jitter or (lambda: None)
        # a planted protocol mistake, for the test that checks the model can fail: flag 2
        # released before the d rows are returned
        self.planted_early_release = planted_early_release

    def wait_all(self, kind: int, epoch: int) -> bool:
        """Until flag [kind][s] of this rank's region holds the epoch for every source s
        (fm_ep.cuh: ep_wait_all); False when the budget runs out."""
        f = self.regions[self.me].flags[kind]
        t0 = time.monotonic()
        while not np.all(f == np.uint32(epoch)):
            if time.monotonic() - t0 > self.wait_s:
                return False
            time.sleep(1e-4)
        return True

    def release(self, kind: int, epoch: int) -> None:
        for reg in self.regions:
            reg.flags[kind, self.me] = epoch

    def forward(self, stages, x: np.ndarray, epoch: int):
        """One layer call on this rank's tokens x (may be empty); returns (y, status),
        status "ok" or "timeout"."""
        lay, me, W, E = self.lay, self.me, self.lay.W, self.lay.E
        T = x.shape[0]
        # ---- dispatch
        if T:
            counts, send = stages.dispatch(x)
            counts = np.asarray(counts, np.int64)
            send = send.numpy().view(np.uint16) if hasattr(send, "numpy") else send
        else:
            counts, send = np.zeros(E, np.int64), np.zeros((0, lay.H), np.uint16)
        for reg in self.regions:
            reg.board[me, :] = counts
        self.release(0, epoch)
        if not self.wait_all(0, epoch):
            return None, "timeout"
        self.jitter()
        cnt = self.regions[me].board.astype(np.int64)
        s_start, s_off = np.zeros(W, np.int64), np.zeros(W, np.int64)
        for r in range(W):
            first, count = owner_range(E, r, W)
            s_start[r] = cnt[me, :first].sum()
            rows = cnt[me, first:first + count].sum()
            s_off[r] = cnt[:me, first:first + count].sum()
            assert s_off[r] + rows <= lay.cap_recv, "receive capacity exceeded"
        P = int(counts.sum())
        rot = int(s_start[me]) if s_start[me] < P else 0
        for p0 in range(P):
            p = p0 + rot if p0 + rot < P else p0 + rot - P
            r = 0
            while r + 1 < W and p >= s_start[r + 1]:
                r += 1
            self.regions[r].recv[s_off[r] + (p - s_start[r])] = send[p]
        self.release(1, epoch)
        # ---- plan (owner): the board is read again here, as the plan kernel reads it
        if not self.wait_all(1, epoch):
            return None, "timeout"
        self.jitter()
        cnt = self.regions[me].board.astype(np.int64)
        first, count = owner_range(E, me, W)
        rc = [int(cnt[s, first + e]) for s in range(W) for e in range(count)]
        src_start = [int(cnt[s, :first].sum()) for s in range(W)]
        src_off = np.concatenate([[0], np.cumsum([sum(rc[s * count:(s + 1) * count]) for s in range(W)])])
        R = int(src_off[-1])
        dst = []
        for p in range(R):
            s = int(np.searchsorted(src_off, p, side="right") - 1)
            pos = src_start[s] + (p - int(src_off[s]))
            assert pos < lay.cap_ret, "return capacity exceeded"
            dst.append((s, pos))
        # ---- experts: d rows straight into their sources' ret rows
        if self.planted_early_release:
            self.release(2, epoch)
        if R:
            import torch
            recv = torch.from_numpy(self.regions[me].recv[:R].copy().view(np.int16))
            d = stages.experts(recv, rc).numpy().view(np.uint16)
            self.jitter()
            if self.planted_early_release:
                time.sleep(0.2)
            for p, (s, pos) in enumerate(dst):
                self.regions[s].ret[pos] = d[p]
        # ---- release, then combine
        self.release(2, epoch)
        if not self.wait_all(2, epoch):
            return None, "timeout"
        if not T:
            return np.zeros((0, lay.H), np.uint16), "ok"
        import torch
        return stages.combine(torch.from_numpy(self.regions[me].ret[:P].copy().view(np.int16))), "ok"
