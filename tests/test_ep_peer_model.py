"""The peer-memory expert-parallel protocol (ep.cu: epoch flags, counts board, rows
written straight into the owners' receive buffers and the d rows straight back) as a
CPU model over shared host memory (tests/ep_peer_model.py), run by 2 and 3 rank
processes with random delays between the steps: every call's output equals the
single-process oracle bit for bit, over several calls with token counts that differ
across ranks and calls (one rank at 0 tokens), so no region is overwritten while
another rank still reads it; and a rank that skips a call makes the others' bounded
waits run out instead of hanging."""
from __future__ import annotations

import random
from multiprocessing import shared_memory

import numpy as np
import pytest
import torch.multiprocessing as mp

from flashmlx_b200 import synthetic as S
from tests.ep_peer_model import Layout, PeerRank, Region
from tests.test_ep import SMALL, OracleStages

CALLS = 3


def _tokens(rank: int, world: int, call: int) -> int:
    T = SMALL.tokens - 4 * call + 3 * rank
    return 0 if (call == 1 and rank == world - 1) else T


def _rank_main(rank, world, names, results, skip_call, planted=False):
    lay = Layout(world, SMALL.num_experts, SMALL.top_k, SMALL.hidden, SMALL.tokens + 3 * world)
    shms = [shared_memory.SharedMemory(name=n) for n in names]
    try:
        regions = [Region(s, lay) for s in shms]
        rng = random.Random(1000 + rank)
        model = PeerRank(rank, lay, regions, wait_s=2.0 if skip_call is not None else 20.0,
                         jitter=lambda: __import__("time").sleep(rng.uniform(0, 0.004)),
                         planted_early_release=planted and rank == 0)
        layer = S.make_layer(SMALL, 3)
        stages = OracleStages(SMALL, layer, rank, world)
        out = []
        for call in range(CALLS):
            if skip_call == call and rank == world - 1:
                out.append(("skipped", 0))
                break
            T = _tokens(rank, world, call)
            x = S.make_x(SMALL, 100 * call + rank, tokens=max(T, 1))[:T]
            y, status = model.forward(stages, x, epoch=call + 1)
            if status != "ok":
                out.append((status, 0))
                break
            mism = int(np.count_nonzero(y != stages.full.moe_block(x)[0])) if T else 0
            out.append(("ok", mism))
        results[rank] = out
    finally:
        for s in shms:
            s.close()


def _run(world, skip_call=None, planted=False):
    lay = Layout(world, SMALL.num_experts, SMALL.top_k, SMALL.hidden, SMALL.tokens + 3 * world)
    shms = [shared_memory.SharedMemory(create=True, size=lay.nbytes) for _ in range(world)]
    try:
        for s in shms:
            np.ndarray((lay.nbytes,), np.uint8, s.buf)[:] = 0
        ctx = mp.get_context("spawn")
        results = ctx.Manager().dict()
        mp.start_processes(_rank_main, args=(world, [s.name for s in shms], results, skip_call, planted), nprocs=world,
                           join=True, start_method="spawn")
        return dict(results)
    finally:
        for s in shms:
            s.close()
            s.unlink()


@pytest.mark.parametrize("world", [2, 3])
def test_peer_protocol_matches_single_process_oracle(world):
    res = _run(world)
    assert len(res) == world
    for r in range(world):
        assert [st for st, _ in res[r]] == ["ok"] * CALLS, res[r]
        assert all(m == 0 for _, m in res[r]), f"rank {r}: outputs differ from the oracle: {res[r]}"


def test_peer_protocol_skipped_call_times_out():
    res = _run(2, skip_call=1)
    assert res[1] == [("ok", 0), ("skipped", 0)]
    assert res[0][0] == ("ok", 0) and res[0][1][0] == "timeout"


def test_planted_early_release_is_caught():
    """The model can fail: an owner that releases flag 2 before returning its d rows lets
    the token ranks combine stale rows, and the comparison with the oracle sees it."""
    res = _run(2, planted=True)
    assert any(m > 0 for r in range(2) for _, m in res[r]), res
