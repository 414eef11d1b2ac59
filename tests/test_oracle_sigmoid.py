"""The CPU oracle's sigmoid-routed MoE variant (Nemotron-H / DeepSeek style,
server/src/nemotron_h.cpp:1010-1106) against the independent numpy restatement, and its
routing properties: group-limited selection, renormalisation, scaling."""
from __future__ import annotations

import numpy as np
import pytest

from flashmlx_b200 import synthetic as S
from oracle import oracle as O
from tests import numpy_ref as R
from tests._parity import metrics


def shape_of(tokens=6, E=16, k=4, H=128, I=128, shared=128, norm=True):
    return S.MoEShape("sig", H, I, E, k, tokens, norm, shared)


def clear_margin(sel, ids, k, eps=1e-5):
    """Tokens whose k-th and (k+1)-th selection scores differ by more than eps."""
    srt = np.sort(sel, axis=-1)[:, ::-1]
    return np.abs(srt[:, k - 1] - srt[:, k]) > eps


@pytest.mark.parametrize("n_group,topk_group", [(1, 1), (4, 2), (8, 3)])
@pytest.mark.parametrize("norm", [False, True])
def test_route_vs_numpy(n_group, topk_group, norm):
    shape = shape_of(tokens=64, E=32, k=4, norm=norm)
    layer = S.make_sigmoid_layer(shape, 3)
    x = S.make_x(shape, 3)
    routing = {"n_group": n_group, "topk_group": topk_group, "routed_scaling_factor": 2.5}
    ids, sc = O.SigmoidLayer(shape, layer, routing).route(x)
    rid, rsc, sel = R.sigmoid_route(x, layer["router_w"], layer["correction_bias"], shape.top_k, n_group,
                                    topk_group, norm, 2.5)
    ok = clear_margin(sel, rid, shape.top_k)
    assert ok.mean() > 0.8
    np.testing.assert_array_equal(ids[ok], rid[ok])  # same picks in the same (selection) order
    np.testing.assert_allclose(sc[ok], rsc[ok], rtol=1e-5, atol=1e-7)


def test_groups_limit_the_picks():
    shape = shape_of(tokens=128, E=32, k=6)
    layer = S.make_sigmoid_layer(shape, 4)
    x = S.make_x(shape, 4)
    ids, _ = O.SigmoidLayer(shape, layer, {"n_group": 8, "topk_group": 2}).route(x)
    groups = ids // (32 // 8)
    assert max(len(set(row)) for row in groups.tolist()) <= 2


def test_renormalised_scores_sum_to_the_scaling_factor():
    shape = shape_of(tokens=32, k=4, norm=True)
    layer = S.make_sigmoid_layer(shape, 5)
    _, sc = O.SigmoidLayer(shape, layer, {"routed_scaling_factor": 1.75}).route(S.make_x(shape, 5))
    np.testing.assert_allclose(sc.sum(-1), 1.75, rtol=1e-5)
    assert (sc > 0).all()


def test_unnormalised_scores_are_scaled_sigmoids():
    shape = shape_of(tokens=16, k=2, norm=False)
    layer = S.make_sigmoid_layer(shape, 6, correction_bias=False)
    _, sc = O.SigmoidLayer(shape, layer, {"routed_scaling_factor": 3.0}).route(S.make_x(shape, 6))
    assert ((sc > 0) & (sc < 3.0)).all()


@pytest.mark.parametrize("shared", [0, 128])
def test_moe_block_vs_numpy(shared):
    shape = shape_of(tokens=6, shared=shared)
    layer = S.make_sigmoid_layer(shape, 7)
    x = S.make_x(shape, 7)
    L = O.SigmoidLayer(shape, layer, {"n_group": 4, "topk_group": 2, "routed_scaling_factor": 2.5})
    y, ids, sc = L.moe_block(x)
    yr = R.sigmoid_moe_block(layer, shape, x, ids, sc)
    m = metrics(y, yr)
    assert m["max_rel"] < 2e-2 and m["mae_rel"] < 5e-3, m


def test_forced_routing_reproduces_own_routing():
    shape = shape_of(tokens=5)
    layer = S.make_sigmoid_layer(shape, 8)
    x = S.make_x(shape, 8)
    L = O.SigmoidLayer(shape, layer, {"routed_scaling_factor": 2.0})
    y, ids, sc = L.moe_block(x)
    y2, _, _ = L.moe_block(x, forced_ids=ids, forced_scores=sc)
    np.testing.assert_array_equal(y, y2)


def test_rejects_bad_grouping():
    shape = shape_of(tokens=2, E=16)
    layer = S.make_sigmoid_layer(shape, 9)
    with pytest.raises(ValueError):
        O.SigmoidLayer(shape, layer, {"n_group": 3, "topk_group": 1}).route(S.make_x(shape, 9))  # 16 % 3
    with pytest.raises(ValueError):
        O.SigmoidLayer(shape, layer, {"n_group": 4, "topk_group": 5}).route(S.make_x(shape, 9))
