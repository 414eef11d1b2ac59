"""Expert parallelism on CPU: the expert split rule (Python vs the C ABI) and the whole
exchange protocol of flashmlx_b200.ep.ep_forward run by gloo ranks with oracle stages,
checked bit-exact against the single-process oracle on each rank's tokens."""
from __future__ import annotations

import dataclasses
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from flashmlx_b200 import synthetic as S
from flashmlx_b200.ep import Exchange, ep_forward, expert_range, local_layer

SMALL = S.MoEShape("ep_small", hidden=256, inter=256, num_experts=10, top_k=3, tokens=20, norm_topk_prob=True,
                   shared_inter=256)


def test_expert_range_rule():
    for E in (1, 7, 8, 10, 60, 128):
        for world in (1, 2, 3, 4, 8):
            got = [expert_range(E, r, world) for r in range(world)]
            assert sum(n for _, n in got) == E
            assert [f for f, _ in got] == list(np.cumsum([0] + [n for _, n in got])[:-1])
            assert max(n for _, n in got) - min(n for _, n in got) <= 1


def test_expert_range_matches_c_abi():
    import ctypes as C
    from flashmlx_b200 import _lib
    lib = _lib.load()
    f, n = C.c_int(), C.c_int()
    for E in (7, 10, 60, 128):
        for world in (1, 3, 8):
            for r in range(world):
                assert lib.fm_ep_range(E, r, world, C.byref(f), C.byref(n)) == 0
                assert (f.value, n.value) == expert_range(E, r, world)
    assert lib.fm_ep_range(10, 3, 3, C.byref(f), C.byref(n)) != 0


def test_local_layer_slices_experts():
    layer = S.make_layer(SMALL, 0)
    for r, (first, count) in enumerate(expert_range(10, r, 3) for r in range(3)):
        sub = local_layer(layer, r, 3)
        for name in ("gate", "up", "down"):
            np.testing.assert_array_equal(sub[name][0], layer[name][0][first:first + count])
        assert sub["router_w"] is layer["router_w"]


class OracleStages:
    """Stages 1, 4 and 6 of ep_forward evaluated by the CPU oracle (test only)."""

    def __init__(self, shape, layer, rank, world):
        from oracle import oracle as O
        self.O, self.shape, self.layer = O, shape, layer
        self.full = O.Layer(shape, layer)
        self.first, self.count = expert_range(shape.num_experts, rank, world)
        self.world = world
        sub = local_layer(layer, rank, world)
        lshape = dataclasses.replace(shape, num_experts=self.count, top_k=1, shared_inter=0, norm_topk_prob=False)
        self.local = O.Layer(lshape, {"router_w": layer["router_w"][self.first:self.first + self.count],
                                      "gate": sub["gate"], "up": sub["up"], "down": sub["down"]})

    def dispatch(self, x):
        O, sh = self.O, self.shape
        self.x = x
        ids, sc, _, _ = O.route(x, self.layer["router_w"], sh.top_k, norm_topk=sh.norm_topk_prob,
                                router_bias=self.layer.get("router_bias"))
        st, sf, off = O.sort_pairs(ids, sh.num_experts)
        self.ids, self.sc = ids, sc
        self.pos = np.empty_like(sf)
        self.pos[sf] = np.arange(sf.size, dtype=sf.dtype)
        return np.diff(off), torch.from_numpy(np.ascontiguousarray(x[st]).view(np.int16))

    def experts(self, recv, recv_counts):
        rows = recv.numpy().view(np.uint16)
        d = np.empty_like(rows)
        p = 0
        for s in range(self.world):
            for e in range(self.count):
                n = recv_counts[s * self.count + e]
                if n:
                    d[p:p + n] = self.local.moe_block(rows[p:p + n], forced_ids=np.full((n, 1), e, np.int32),
                                                      forced_scores=np.full((n, 1), 0x3F80, np.uint16))[0]
                p += n
        return torch.from_numpy(d.view(np.int16))

    def combine(self, ret):
        T, k = self.ids.shape
        r = S.bf16_to_f32(ret.numpy().view(np.uint16))
        sc = S.bf16_to_f32(self.sc)
        rbf = lambda a: S.bf16_to_f32(S.f32_to_bf16(a))  # noqa: E731
        acc = np.zeros((T, self.shape.hidden), np.float32)
        pos = self.pos.reshape(T, k)
        for j in range(k):
            acc += rbf(r[pos[:, j]] * sc[:, j:j + 1])
        y = rbf(acc)
        if self.shape.shared_inter:
            term = S.bf16_to_f32(self.full.moe_block(self.x, forced_ids=self.ids,
                                                     forced_scores=np.zeros_like(self.sc))[0])
            y = rbf(y + term)
        return S.f32_to_bf16(y)


def _rank_main(rank, world, port, shape, results):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        layer = S.make_layer(shape, 3)
        x = S.make_x(shape, 100 + rank)
        if rank == world - 1:
            x = x[:5]  # ragged token counts across ranks
        stages = OracleStages(shape, layer, rank, world)
        y = ep_forward(stages, Exchange(shape.num_experts, device="cpu"), x)
        want = stages.full.moe_block(x)[0]
        results[rank] = (int(np.count_nonzero(y != want)), y.shape)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_ep_protocol_matches_single_process_oracle(world):
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    mgr = ctx.Manager()
    results = mgr.dict()
    mp.start_processes(_rank_main, args=(world, port, SMALL, results), nprocs=world, join=True, start_method="spawn")
    assert len(results) == world
    for r in range(world):
        mism, shp = results[r]
        assert mism == 0, f"rank {r}: {mism} elements differ from the single-process oracle"
        assert shp[1] == SMALL.hidden
