"""GPU test of fm_moe_block_noalloc, the entry point for callers that cannot let a
library allocate device memory (their device memory belongs to a runtime's memory
planner or caching allocator, or they cannot afford the device-wide synchronization of
cudaMalloc / cudaFree).  It is called through the C ABI and must match the handle-based
fm_moe_block on the same inputs, on two calls in a row sharing the fixed scratch.

The file name sorts last so that a run stopping at the first failure has already run
every other test; it also passes alone in a fresh process.
"""
from __future__ import annotations

import ctypes as C

import numpy as np
import pytest
import torch

from flashmlx_b200 import synthetic as S
from tests._parity import TIGHT, assert_close

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def setup():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from flashmlx_b200 import _lib, ops
    shape = S.CONFIGS["qwen15_decode"]  # 32 decode tokens
    weights = ops.MoEWeightsT.from_numpy(S.make_layer(shape, 3), "cuda")
    block = ops.MoEBlock(shape, weights)
    return _lib, ops, shape, block


def run_noalloc(lib_mod, ops, block, x):
    y = torch.empty_like(x)
    stream = torch.cuda.current_stream()
    st = lib_mod.load().fm_moe_block_noalloc(torch.cuda.current_device(), C.c_void_p(stream.cuda_stream),
                                             C.byref(block.cfg), C.byref(block.W), C.c_void_p(x.data_ptr()),
                                             x.shape[0], C.c_void_p(y.data_ptr()))
    assert st == lib_mod.FM_OK, lib_mod.load().fm_status_string(st)
    torch.cuda.synchronize()
    return ops.bf16_to_numpy(y)


def test_noalloc_matches_handle_path_twice(setup):
    lib_mod, ops, shape, block = setup
    from oracle import oracle as O
    from tests.gpu_util import check_vs_oracle
    layer = S.make_layer(shape, 3)
    for call, seed in enumerate((11, 12)):  # two calls in a row reuse the same scratch
        x_np = S.make_x(shape, seed)
        x = ops.bf16_from_numpy(x_np, "cuda")
        y_ref, r = block(x, return_routing=True)
        y_ref = ops.bf16_to_numpy(y_ref)
        ops.synchronize()
        y = run_noalloc(lib_mod, ops, block, x)
        assert np.isfinite(S.bf16_to_f32(y)).all()
        m = assert_close(y, y_ref, f"no-alloc call {call} vs fm_moe_block", **TIGHT)
        print(f"no-alloc call {call}: {m}")
        # and against the CPU oracle directly: 32 tokens run the dequant GEMV, whose
        # arithmetic is MLX's exact-weight (qmv) form
        ids, sc = r["topk_ids"].cpu().numpy(), ops.bf16_to_numpy(r["topk_scores"])
        check_vs_oracle(y, lambda: O.Layer(shape, layer).moe_block(x_np, forced_ids=ids, forced_scores=sc),
                        f"no-alloc call {call}", "exact")


def test_noalloc_rejects_oversize_batch(setup):
    lib_mod, ops, shape, block = setup
    T = 1 << 15  # needs far more than the fixed scratch
    x = torch.zeros(T, shape.hidden, dtype=torch.bfloat16, device="cuda")
    y = torch.full_like(x, 7.0)
    st = lib_mod.load().fm_moe_block_noalloc(torch.cuda.current_device(),
                                             C.c_void_p(torch.cuda.current_stream().cuda_stream),
                                             C.byref(block.cfg), C.byref(block.W), C.c_void_p(x.data_ptr()), T,
                                             C.c_void_p(y.data_ptr()))
    assert st == lib_mod.FM_ETOOLARGE
    torch.cuda.synchronize()
    assert bool((y == 7.0).all()), "a rejected call must not launch anything"
