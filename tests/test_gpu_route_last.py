"""The small-batch routing kernels against the cooperative grid-barrier kernel: the
last-block form (fm_set_route_mode(FM_ROUTE_LAST_BLOCK): the router GEMV over the grid,
then top-k, the stable expert-major sort and the tile plan in the block that finishes
last) and the cluster form (FM_ROUTE_CLUSTER: one cluster of 8 CTAs, router and top-k
over the cluster, sort and plan in its first CTA): the same ids,
scores, expert offsets and permutation bit for bit, and the same layer output up to the
order of the fp32 atomic adds, for softmax routing (model.cpp:757-775), grouped sigmoid
routing (nemotron_h.cpp:1018-1050) and gather_qmm's given indices (model.cpp:703-721);
batches above 128 tokens take the grid form in either mode."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from flashmlx_b200 import synthetic as S
from flashmlx_b200 import _lib
from tests.gpu_util import GpuLayer, dev_bf16, dev_u32, host_bf16

pytestmark = pytest.mark.gpu


def _in_mode(mode, fn):
    from flashmlx_b200 import ops
    h = ops.default_handle()
    h.set_route_mode(mode)
    try:
        return fn()
    finally:
        h.set_route_mode(_lib.FM_ROUTE_AUTO)


def _same_up_to_atomic_order(ya, yb, what):
    assert np.mean(ya == yb) > 0.999, f"{what}: outputs differ beyond fp32 atomic order"


@pytest.fixture(scope="module")
def qwen():
    return GpuLayer(S.CONFIGS["qwen15_decode"], 3)


SMALL_FORMS = {"last-block": _lib.FM_ROUTE_LAST_BLOCK, "cluster": _lib.FM_ROUTE_CLUSTER}


@pytest.mark.parametrize("form", sorted(SMALL_FORMS))
@pytest.mark.parametrize("T", [1, 5, 16, 17, 32, 100, 128, 129, 200])
def test_softmax_routing_forms_agree(qwen, T, form):
    x = S.make_x(qwen.shape, 300 + T, tokens=T)
    ya, ra = _in_mode(_lib.FM_ROUTE_GRID, lambda: qwen.run(x))
    yb, rb = _in_mode(SMALL_FORMS[form], lambda: qwen.run(x))
    assert ra.keys() == rb.keys()
    for k in ra:
        np.testing.assert_array_equal(ra[k], rb[k], err_msg=f"T={T} {k}")
    _same_up_to_atomic_order(ya, yb, f"T={T}")


@pytest.mark.parametrize("form", sorted(SMALL_FORMS))
@pytest.mark.parametrize("T", [1, 32, 128])
def test_small_batch_forms_against_oracle(qwen, T, form):
    x = S.make_x(qwen.shape, 400 + T, tokens=T)
    _in_mode(SMALL_FORMS[form], lambda: qwen.check(x, f"{form} routing T={T}"))


@pytest.mark.parametrize("form", sorted(SMALL_FORMS))
@pytest.mark.parametrize("T", [1, 7, 48, 300])
def test_sigmoid_routing_forms_agree(T, form):
    from flashmlx_b200 import ops
    shape = S.MoEShape("sig", 512, 256, 32, 4, T, True, 256)
    layer = S.make_sigmoid_layer(shape, 25)
    x = ops.bf16_from_numpy(S.make_x(shape, 25), "cuda")
    blk = ops.MoEBlockVariant.sigmoid_from_numpy(shape, layer, "cuda", n_group=4, topk_group=2,
                                                 routed_scaling_factor=2.5)

    def run():
        y, r = blk(x, return_routing=True)
        torch.cuda.synchronize()
        return host_bf16(y), {k: v.cpu() for k, v in r.items()}
    ya, ra = _in_mode(_lib.FM_ROUTE_GRID, run)
    yb, rb = _in_mode(SMALL_FORMS[form], run)
    for k in ra:
        assert torch.equal(ra[k], rb[k]), f"T={T} {k}"
    _same_up_to_atomic_order(ya, yb, f"sigmoid T={T}")


@pytest.mark.parametrize("form", sorted(SMALL_FORMS))
@pytest.mark.parametrize("rows", [3, 64, 128, 160])
def test_given_indices_forms_agree(rows, form):
    """gather_qmm's given indices (one row per index, random experts): the same rows."""
    from flashmlx_b200 import ops
    rng = np.random.default_rng(rows)
    E, N, K = 8, 256, 512
    w, s, b = S.make_qmatrix(4, "gq", (E,), N, K, 64, 4, scale_std=0.05)
    x = S.f32_to_bf16(rng.standard_normal((rows, 1, K)).astype(np.float32))
    idx = rng.integers(0, E, rows).astype(np.uint32)
    args = (dev_bf16(x), dev_u32(w), dev_bf16(s), dev_bf16(b))

    def run():
        y = ops.gather_qmm(*args, rhs_indices=dev_u32(idx), group_size=64, bits=4)
        torch.cuda.synchronize()
        return host_bf16(y)
    np.testing.assert_array_equal(_in_mode(_lib.FM_ROUTE_GRID, run), _in_mode(SMALL_FORMS[form], run))


def test_unknown_route_mode_is_rejected():
    from flashmlx_b200 import ops
    with pytest.raises(ops.FlashMoEError):
        ops.default_handle().set_route_mode(7)
