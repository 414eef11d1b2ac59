"""The last-block routing kernel's arrival logic (route.cu, route_last_body), restated on
the CPU: each block counts itself in with atomicInc(counter, gridDim.x - 1), whose PTX
semantics are old = *p; *p = (old >= limit) ? 0 : old + 1.  For any arrival order exactly
one block -- the last to arrive -- sees gridDim.x - 1 and goes on to phases 2-4, and the
counter is back at 0 for the next launch, whatever that launch's grid size."""
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
