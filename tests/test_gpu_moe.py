"""GPU parity of fm_moe_block (the whole MoE layer) against the CPU oracle, through the
C ABI: routing ids (sets, near-ties excluded) and scores bit-exact, the expert-major
permutation bit-exact, activations within the north-star tolerances, on both
expert-product paths and every BASELINE configuration's layer shape."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from flashmlx_b200 import synthetic as S
from tests.gpu_util import GpuLayer, dev_bf16, host_bf16

pytestmark = pytest.mark.gpu
PATHS = {"auto": 0, "gemv": 1, "tcgen05": 2}


@pytest.fixture(scope="module")
def ops():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from flashmlx_b200 import ops as _ops
    return _ops


_layers = {}


def layer(name, seed=0):
    key = (name, seed)
    if key not in _layers:
        _layers.clear()  # keep one resident layer at a time
        torch.cuda.empty_cache()
        _layers[key] = GpuLayer(S.CONFIGS[name], seed)
    return _layers[key]


def with_path(ops, path):
    h = ops.default_handle()
    h.set_path(PATHS[path])
    return h


@pytest.mark.parametrize("path", ["gemv", "tcgen05"])
@pytest.mark.parametrize("T", [1, 15, 16, 32, 200])
def test_qwen15_block(ops, path, T):
    L = layer("qwen15_decode")
    h = with_path(ops, path)
    try:
        x = S.make_x(L.shape, 100 + T, tokens=T)
        L.check(x, f"qwen15 {path} T={T}")
    finally:
        h.set_path(0)


def test_qwen15_decode_config0(ops):
    """BASELINE configs[0] exactly: 32 decode tokens, seed 0."""
    L = layer("qwen15_decode")
    x = S.make_x(L.shape, 0)
    m, ties = L.check(x, "configs[0]")
    print("configs[0]", m, "near-ties", ties)


@pytest.mark.parametrize("path", ["gemv", "tcgen05"])
@pytest.mark.parametrize("T", [64, 700])
def test_qwen3_block(ops, path, T):
    L = layer("qwen3_decode")
    h = with_path(ops, path)
    try:
        x = S.make_x(L.shape, 200 + T, tokens=T)
        L.check(x, f"qwen3 {path} T={T}")
    finally:
        h.set_path(0)


@pytest.mark.parametrize("path", ["gemv", "tcgen05"])
def test_mixtral_block(ops, path):
    from tests._parity import MIXTRAL_TC
    L = layer("mixtral_prefill")
    h = with_path(ops, path)
    try:
        x = S.make_x(L.shape, 300, tokens=48)
        # the named exception to max_rel 1e-2 (one or two bf16 ulps at the largest output)
        L.check(x, f"mixtral {path}", tight=MIXTRAL_TC if path == "tcgen05" else None)
    finally:
        h.set_path(0)


def test_qwen15_prefill_config1_full(ops):
    """BASELINE configs[1] at full size (T=4096): routing for every token, the
    permutation exactly, activations on a sample of rows (tokens are independent)."""
    L = layer("qwen15_prefill")
    x = S.make_x(L.shape, 0)
    sample = np.random.default_rng(0).choice(x.shape[0], 96, replace=False)
    m, ties = L.check(x, "configs[1]", sample=np.sort(sample))
    print("configs[1]", m, "near-ties", ties)


def test_qwen3_prefill_full_sample(ops):
    L = layer("qwen3_prefill")
    x = S.make_x(L.shape, 0)
    sample = np.sort(np.random.default_rng(1).choice(x.shape[0], 48, replace=False))
    L.check(x, "configs[3] prefill", sample=sample)


def test_qwen3_decode_config3_exact(ops):
    """BASELINE configs[3] decode exactly: 256 tokens, seed 0, every token's routing and
    every output row (the automatic path choice)."""
    L = layer("qwen3_decode")
    x = S.make_x(L.shape, 0)
    assert x.shape[0] == 256
    m, ties = L.check(x, "configs[3] decode T=256")
    print("configs[3] decode", m, "near-ties", ties)


def test_mixtral_config4_full_routing_sample(ops):
    """BASELINE configs[4] at full size: the Zipf(1.2)-skewed 8192-token batch of the
    Mixtral-shaped layer (8 experts, top-2 renormalised, H 4096, I 14336).  Routing for
    every token and the permutation exactly; activations on a 512-token sample."""
    L = layer("mixtral_prefill")
    x = S.make_x(L.shape, 0)
    assert x.shape[0] == 8192
    sample = np.sort(np.random.default_rng(4).choice(x.shape[0], 512, replace=False))
    m, ties = L.check(x, "configs[4] T=8192 (512-row sample)", sample=sample)
    print("configs[4]", m, "near-ties", ties)


def test_all_tokens_one_expert(ops):
    """Heavy skew: a large router bias sends every token to the same expert."""
    L = layer("qwen15_decode", seed=5)
    bias = np.zeros(L.shape.num_experts, np.float32)
    bias[7] = 30.0
    L.np["router_bias"] = S.f32_to_bf16(bias)
    from flashmlx_b200 import ops as _ops
    from oracle import oracle as O
    L.weights.router_bias = dev_bf16(L.np["router_bias"])
    L.block = _ops.MoEBlock(L.shape, L.weights)
    L.oracle = O.Layer(L.shape, L.np)
    for path in ("gemv", "tcgen05"):
        h = with_path(ops, path)
        try:
            x = S.make_x(L.shape, 9, tokens=300)
            y, r = L.run(x)
            assert (r["topk_ids"] == 7).any(axis=1).all()
            L.check(x, f"one hot expert {path}")
        finally:
            h.set_path(0)
    _layers.clear()


def test_deterministic_repeat(ops):
    L = layer("qwen15_decode")
    x = S.make_x(L.shape, 77, tokens=256)
    for path in ("gemv", "tcgen05"):
        h = with_path(ops, path)
        try:
            y1, r1 = L.run(x)
            y2, r2 = L.run(x)
            np.testing.assert_array_equal(r1["topk_ids"], r2["topk_ids"])
            np.testing.assert_array_equal(r1["sorted_token"], r2["sorted_token"])
            assert np.mean(y1 == y2) > 0.999, f"{path}: run-to-run differences beyond fp32 atomic order"
        finally:
            h.set_path(0)


def test_paths_agree(ops):
    L = layer("qwen15_decode")
    x = S.make_x(L.shape, 55, tokens=128)
    outs = []
    for path in ("gemv", "tcgen05"):
        h = with_path(ops, path)
        try:
            outs.append(L.run(x))
        finally:
            h.set_path(0)
    (ya, ra), (yb, rb) = outs
    np.testing.assert_array_equal(ra["topk_ids"], rb["topk_ids"])
    # the two paths follow MLX's two arithmetic forms (exact vs bf16-rounded weights)
    from tests._parity import EXACT_FLOOR, assert_close
    assert_close(ya, yb, "gemv vs tcgen05", **EXACT_FLOOR)


def test_moe_block_argument_errors(ops):
    L = layer("qwen15_decode")
    with pytest.raises(ValueError):
        L.block(torch.zeros(4, 100, dtype=torch.bfloat16, device="cuda"))
    y = L.block(torch.zeros(0, L.shape.hidden, dtype=torch.bfloat16, device="cuda"))
    assert y.shape[0] == 0
    _ = host_bf16
