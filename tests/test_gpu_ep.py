"""Expert parallelism on GPUs through the C ABI: the staged calls (fm_ep_dispatch /
fm_ep_experts / fm_ep_combine) with NCCL all-to-alls, and the peer-memory layer
(fm_ep_p2p_*) whose kernels move the rows themselves.  A one-rank group runs on any GPU
box; two ranks need two GPUs.  Each rank's output is checked against the single-GPU
fm_moe_block on the same tokens and against the oracle under that routing."""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from flashmlx_b200 import synthetic as S

pytestmark = pytest.mark.gpu

SHAPES = {
    "qwen15": S.CONFIGS["qwen15_decode"],
    "qwen3": S.CONFIGS["qwen3_decode"],
}


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _check_rank(rank, world, shape_name, tokens, path):
    from flashmlx_b200 import ops
    from flashmlx_b200.ep import MoEBlockEP, local_layer
    from oracle import oracle as O
    from tests._parity import EXACT_FLOOR, assert_close
    from tests.gpu_util import check_vs_oracle, form_of, host_bf16
    shape = SHAPES[shape_name]
    layer = S.make_layer(shape, 7)
    dev = torch.device("cuda", rank)
    h = ops.default_handle(rank)
    h.set_path({"auto": 0, "gemv": 1, "tcgen05": 2}[path])
    try:
        local = ops.MoEWeightsT.from_numpy(local_layer(layer, rank, world), dev)
        block = MoEBlockEP(shape, local)
        x_np = S.make_x(shape, 40 + rank, tokens=tokens)
        x = ops.bf16_from_numpy(x_np, dev)
        y_ep = host_bf16(block(x))
        form = form_of(h)
        # single-GPU reference on the same tokens, with the full layer
        full = ops.MoEBlock(shape, ops.MoEWeightsT.from_numpy(layer, dev))
        y1, r = full(x, return_routing=True)
        torch.cuda.synchronize(dev)
        assert_close(y_ep, host_bf16(y1), f"rank {rank}: ep vs fm_moe_block", **EXACT_FLOOR)
        ids, sc = r["topk_ids"].cpu().numpy(), host_bf16(r["topk_scores"])
        check_vs_oracle(y_ep, lambda: O.Layer(shape, layer).moe_block(x_np, forced_ids=ids, forced_scores=sc),
                        f"rank {rank}: ep vs oracle", form)
    finally:
        h.set_path(0)


def _check_rank_peer(rank, world, shape_name, tokens, path):
    """Several calls on one peer-memory layer (the epochs advance), with token counts that
    differ across ranks and calls, one of them 0 on the last rank."""
    from flashmlx_b200 import ops
    from flashmlx_b200.ep import MoEBlockEPPeer, local_layer
    from oracle import oracle as O
    from tests._parity import EXACT_FLOOR, assert_close
    from tests.gpu_util import check_vs_oracle, form_of, host_bf16
    shape = SHAPES[shape_name]
    layer = S.make_layer(shape, 7)
    dev = torch.device("cuda", rank)
    local = ops.MoEWeightsT.from_numpy(local_layer(layer, rank, world), dev)
    block = MoEBlockEPPeer(shape, local, max_tokens=tokens + 8 * world)
    block.h.set_path({"auto": 0, "gemv": 1, "tcgen05": 2}[path])
    full = ops.MoEBlock(shape, ops.MoEWeightsT.from_numpy(layer, dev))
    try:
        for call in range(3):
            T = tokens - 8 * call + 4 * rank
            if call == 1 and rank == world - 1 and world > 1:
                T = 0
            x_np = S.make_x(shape, 100 * call + 40 + rank, tokens=max(T, 1))[:T]
            x = ops.bf16_from_numpy(x_np, dev) if T else torch.empty(0, shape.hidden, dtype=torch.bfloat16,
                                                                   device=dev)
            y = block(x)
            block.sync()
            form = form_of(block.h)
            assert y.shape == (T, shape.hidden)
            if T == 0:
                continue
            y_ep = host_bf16(y)
            y1, r = full(x, return_routing=True)
            torch.cuda.synchronize(dev)
            assert_close(y_ep, host_bf16(y1), f"rank {rank} call {call}: peer ep vs fm_moe_block", **EXACT_FLOOR)
            if call == 0:
                ids, sc = r["topk_ids"].cpu().numpy(), host_bf16(r["topk_scores"])
                check_vs_oracle(y_ep, lambda: O.Layer(shape, layer).moe_block(x_np, forced_ids=ids, forced_scores=sc),
                                f"rank {rank}: peer ep vs oracle", form)
    finally:
        block.close()


def _check_rank_peer_timeout(rank, world):
    """The last rank skips one call: the others' bounded waits run out and report a
    timeout at sync (no fault, the context stays usable), then everyone closes."""
    from flashmlx_b200 import ops
    from flashmlx_b200._lib import FlashMoEError, FM_ETIMEOUT
    from flashmlx_b200.ep import MoEBlockEPPeer, local_layer
    shape = SHAPES["qwen15"]
    layer = S.make_layer(shape, 7)
    dev = torch.device("cuda", rank)
    local = ops.MoEWeightsT.from_numpy(local_layer(layer, rank, world), dev)
    block = MoEBlockEPPeer(shape, local, max_tokens=16)
    try:
        x = ops.bf16_from_numpy(S.make_x(shape, 5 + rank, tokens=16), dev)
        if rank != world - 1:
            block(x)
            with pytest.raises(FlashMoEError) as ei:
                block.sync()
            assert ei.value.status == FM_ETIMEOUT, ei.value
            # the context still works
            y = torch.ones(4, device=dev) * 2
            assert float(y.sum().item()) == 8.0
    finally:
        block.close()


def _rank_main(rank, world, port, shape_name, tokens, path, results, impl="nccl"):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", rank))
    try:
        if impl == "peer":
            _check_rank_peer(rank, world, shape_name, tokens, path)
        elif impl == "peer_timeout":
            _check_rank_peer_timeout(rank, world)
        else:
            _check_rank(rank, world, shape_name, tokens, path)
        results[rank] = "ok"
    except Exception as e:  # reported by the parent
        results[rank] = f"{type(e).__name__}: {e}"
    finally:
        dist.barrier()
        dist.destroy_process_group()


def _run(world, shape_name, tokens, path, impl="nccl"):
    if not torch.cuda.is_available() or torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPU(s)")
    os.environ["NCCL_NVLS_ENABLE"] = "0"  # children inherit: no multicast objects in these tests
    ctx = mp.get_context("spawn")
    results = ctx.Manager().dict()
    mp.start_processes(_rank_main, args=(world, _free_port(), shape_name, tokens, path, results, impl),
                       nprocs=world, join=True, start_method="spawn")
    for r in range(world):
        assert results.get(r) == "ok", f"rank {r}: {results.get(r)}"


@pytest.mark.parametrize("path", ["gemv", "tcgen05"])
@pytest.mark.parametrize("shape_name", ["qwen15", "qwen3"])
def test_ep_one_rank(shape_name, path):
    _run(1, shape_name, 40, path)


@pytest.mark.parametrize("path", ["gemv", "tcgen05"])
def test_ep_two_ranks(path):
    _run(2, "qwen15", 48, path)


@pytest.mark.parametrize("path", ["gemv", "tcgen05"])
@pytest.mark.parametrize("shape_name", ["qwen15", "qwen3"])
def test_ep_peer_one_rank(shape_name, path):
    _run(1, shape_name, 40, path, impl="peer")


@pytest.mark.parametrize("path", ["gemv", "tcgen05"])
def test_ep_peer_two_ranks(path):
    _run(2, "qwen15", 48, path, impl="peer")


def test_ep_peer_two_ranks_timeout():
    _run(2, "qwen15", 16, "auto", impl="peer_timeout")
