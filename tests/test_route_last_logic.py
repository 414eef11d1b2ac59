"""Logic of the small-batch routing forms, restated on the CPU.

The last-block kernel's arrival (route.cu, route_last_body): each block counts itself in
with atomicInc(counter, gridDim.x - 1), whose PTX semantics are old = *p;
*p = (old >= limit) ? 0 : old + 1.  For any arrival order exactly one block -- the last to
arrive -- sees gridDim.x - 1 and goes on to phases 2-4, and the counter is back at 0 for
the next launch, whatever that launch's grid size.

The cluster kernel's one-CTA tail (route.cu, tail_fused): pair positions from per-expert
token bitmasks equal the stable sort by expert that the grid form produces.

The last-block tail's column scan (phase_column_scan_one_block) against the grid form's
(phase_column_scan): the same chunk offsets and totals."""
from __future__ import annotations

import numpy as np


def atomic_inc(mem, limit):
    old = mem[0]
    mem[0] = 0 if old >= limit else old + 1
    return old


def test_one_last_block_per_launch_and_the_counter_returns_to_zero():
    rng = np.random.default_rng(0)
    counter = [0]
    for grid in [1, 2, 3, 7, 16, 148, 1, 64, 5, 296]:
        order = rng.permutation(grid)  # the blocks' arrival order
        last = [b for b in order if atomic_inc(counter, grid - 1) == grid - 1]
        assert last == [order[-1]], (grid, last)
        assert counter[0] == 0


def _tail_fused_positions(ids: np.ndarray, E: int, T: int, k: int) -> np.ndarray:
    """The cluster form's one-CTA tail (route.cu, tail_fused), restated: a 128-bit token mask
    per expert (bit t set when token t routes to it), exclusive starts of the experts'
    popcounts, and pair (t, j) at start[e] + popc(mask[e] below bit t); -1 for dropped
    pairs (id < 0)."""
    words = 4  # kTailTokens / 32
    mask = np.zeros((E, words), np.uint64)
    for i, e in enumerate(ids):
        if e >= 0:
            t = i // k
            mask[e, t >> 5] |= np.uint64(1) << np.uint64(t & 31)
    popc = lambda v: bin(int(v)).count("1")
    counts = np.array([sum(popc(mask[e, w]) for w in range(words)) for e in range(E)])
    starts = np.concatenate([[0], np.cumsum(counts)])[:-1]
    pos = np.full(len(ids), -1, np.int64)
    for i, e in enumerate(ids):
        if e < 0:
            continue
        t = i // k
        w, b = t >> 5, t & 31
        rank = popc(int(mask[e, w]) & ((1 << b) - 1)) + sum(popc(mask[e, ww]) for ww in range(w))
        pos[i] = starts[e] + rank
    return pos


def test_fused_tail_positions_equal_the_stable_expert_sort():
    """Positions from the token bitmasks equal a stable sort of the pairs by expert id (the
    order the grid form's chunked count / column scan / scatter produces), for batches up to
    128 tokens, top-k up to 16, with dropped pairs."""
    rng = np.random.default_rng(1)
    for T, E, k in [(1, 4, 1), (7, 60, 4), (32, 60, 4), (100, 128, 8), (128, 512, 16), (128, 3, 2)]:
        ids = np.stack([rng.permutation(E)[:k] for _ in range(T)]).reshape(-1).astype(np.int64)
        drop = rng.random(ids.shape) < 0.1
        ids[drop] = -1
        pos = _tail_fused_positions(ids, E, T, k)
        kept = np.flatnonzero(ids >= 0)
        order = kept[np.argsort(ids[kept], kind="stable")]  # flat pair indices in sorted order
        expect = np.full(len(ids), -1, np.int64)
        expect[order] = np.arange(len(order))
        assert np.array_equal(pos, expect), (T, E, k)


def _column_scan_grid(counts: np.ndarray, cap: int, nthreads: int = 256):
    """phase_column_scan restated: per expert, the chunks in passes of `cap`, each pass an
    exclusive block scan (thread i takes a contiguous range of ceil(n / nthreads) chunks,
    the per-thread sums scanned across threads) plus the carry of earlier passes."""
    nch, E = counts.shape
    out = counts.copy()
    totals = np.zeros(E, np.int64)
    for e in range(E):
        carry = 0
        for c0 in range(0, nch, cap):
            n = min(cap, nch - c0)
            buf = out[c0:c0 + n, e].copy()
            per = -(-n // nthreads)
            local = [int(buf[min(n, t * per):min(n, t * per + per)].sum()) for t in range(nthreads)]
            excl_thread = np.concatenate([[0], np.cumsum(local)])[:-1]
            for t in range(nthreads):
                run = int(excl_thread[t])
                for i in range(min(n, t * per), min(n, t * per + per)):
                    x = int(buf[i])
                    buf[i] = run
                    run += x
            out[c0:c0 + n, e] = buf + carry
            carry += sum(local)
        totals[e] = carry
    return out, totals


def _column_scan_one_block(counts: np.ndarray, max_chunks: int = 8):
    """phase_column_scan_one_block restated: each thread scans its experts' (at most
    max_chunks) counts in registers."""
    nch, E = counts.shape
    assert nch <= max_chunks
    out = counts.copy()
    totals = np.zeros(E, np.int64)
    for e in range(E):
        run = 0
        for i in range(max_chunks):
            c = int(counts[i, e]) if i < nch else 0
            if i < nch:
                out[i, e] = run
            run += c
        totals[e] = run
    return out, totals


def test_one_block_column_scan_equals_the_grid_scan():
    """The last-block form's one-block column scan gives the grid form's chunk offsets and
    totals (chunk-major counts [chunk][expert]); the grid scan is exercised with passes
    shorter than the chunk count, so its carry between passes is covered too."""
    rng = np.random.default_rng(2)
    for nch, E in [(1, 4), (3, 60), (8, 128), (8, 512), (5, 1)]:
        counts = rng.integers(0, 17, size=(nch, E)).astype(np.int64)
        g_out, g_tot = _column_scan_grid(counts, cap=3, nthreads=4)
        o_out, o_tot = _column_scan_one_block(counts)
        assert np.array_equal(g_out, o_out) and np.array_equal(g_tot, o_tot), (nch, E)
        assert np.array_equal(g_out, np.cumsum(counts, axis=0) - counts)
