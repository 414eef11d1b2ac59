"""CPU tests: the oracle against the known-answer fixtures, against an independent
numpy restatement, and its structural properties (sort stability, sorted vs
unsorted switch_mlp paths, token independence)."""
from __future__ import annotations

import os

import numpy as np
import pytest

from flashmlx_b200 import synthetic as S
from oracle import oracle as O
from tests import numpy_ref as R
from tests._parity import metrics, same_sets

KAT = np.load(os.path.join(os.path.dirname(__file__), "golden", "kat.npz"))


def small_shape(tokens=8, shared=256, E=6, k=2, norm=False, H=128, I=128, zipf=0.0):
    return S.MoEShape("small", H, I, E, k, tokens, norm, shared, zipf)


# ------------------------------------------------------------------ known answers
def test_kat_nibble_order():
    y = O.quantized_matmul(KAT["nibble_order_x"], KAT["nibble_order_w"], KAT["nibble_order_s"],
                           KAT["nibble_order_b"])
    np.testing.assert_array_equal(y, KAT["nibble_order_y"])


def test_kat_group_bias():
    y = O.quantized_matmul(KAT["group_bias_x"], KAT["group_bias_w"], KAT["group_bias_s"], KAT["group_bias_b"])
    np.testing.assert_array_equal(y, KAT["group_bias_y"])


def test_kat_gather_broadcast_and_lhs():
    x, w, s, b, rhs, lhs = (KAT[k] for k in ("gather_x", "gather_w", "gather_s", "gather_b", "gather_rhs",
                                             "gather_lhs"))
    y = O.gather_qmm(x, w, s, b, None, rhs)
    np.testing.assert_array_equal(y, KAT["gather_y_bcast"])
    y = O.gather_qmm(x, w, s, b, lhs, rhs)
    np.testing.assert_array_equal(y, KAT["gather_y_lhs"])


@pytest.mark.parametrize("k", [2, 4])
def test_kat_router_ties(k):
    ids, sc, lg, pr = O.route(KAT["router_ties_x"], KAT["router_ties_w"], k)
    np.testing.assert_array_equal(ids, KAT[f"router_ties_ids_k{k}"])


@pytest.mark.parametrize("k", [1, 2])
def test_kat_one_expert(k):
    ids, sc, _, _ = O.route(KAT["one_expert_x"], KAT["one_expert_w"], k)
    np.testing.assert_array_equal(ids, KAT[f"one_expert_ids_k{k}"])
    st, sf, off = O.sort_pairs(ids, 6)
    assert off[5 + 1] - off[5] == 70  # every token on expert 5


def test_single_expert_router_is_prob_one():
    x = S.f32_to_bf16(np.ones((3, 64), np.float32))
    w = S.f32_to_bf16(np.full((1, 64), 0.01, np.float32))
    ids, sc, _, pr = O.route(x, w, 1)
    assert (ids == 0).all() and (S.bf16_to_f32(sc) == 1.0).all()


# ------------------------------------------------------------------ vs numpy restatement
@pytest.mark.parametrize("M,K,N,gs", [(1, 128, 32, 64), (7, 256, 48, 64), (5, 256, 32, 32), (3, 256, 16, 128)])
def test_quantized_matmul_vs_numpy(M, K, N, gs):
    rng = np.random.default_rng(M * 1000 + K + N + gs)
    x = S.f32_to_bf16(rng.standard_normal((M, K), dtype=np.float32))
    w, s, b = S.make_qmatrix(7, f"qm{M}{K}{N}", (), N, K, gs)
    y = O.quantized_matmul(x, w, s, b, group_size=gs)
    yr = R.quantized_matmul(x, w, s, b, group_size=gs)
    m = metrics(y, yr)
    # fp32 (oracle) vs fp64 (numpy) accumulation: at most one bf16 rounding apart
    assert m["max_rel"] < 1e-2 and m["exact_frac"] > 0.97, m


def test_gather_qmm_vs_numpy():
    rng = np.random.default_rng(3)
    E, N, K = 5, 32, 128
    w, s, b = S.make_qmatrix(3, "g", (E,), N, K)
    x = S.f32_to_bf16(rng.standard_normal((6, 1, K), dtype=np.float32))
    rhs = rng.integers(0, E, size=(6, 3)).astype(np.uint32)
    y = O.gather_qmm(x, w, s, b, None, rhs.ravel())
    for i in range(18):
        e = rhs.ravel()[i]
        yr = R.quantized_matmul(x[i // 3], w[e], s[e], b[e])
        assert metrics(y[i], yr)["max_rel"] < 1e-2


@pytest.mark.parametrize("shared", [0, 256])
@pytest.mark.parametrize("norm", [False, True])
def test_moe_block_vs_numpy(shared, norm):
    shape = small_shape(tokens=6, shared=shared, norm=norm)
    layer = S.make_layer(shape, 11)
    x = S.make_x(shape, 11)
    L = O.Layer(shape, layer)
    y, ids, sc = L.moe_block(x)
    yr = R.moe_block(layer, shape, x, ids, sc)
    m = metrics(y, yr)
    assert m["max_rel"] < 2e-2 and m["mae_rel"] < 5e-3, m


# ------------------------------------------------------------------ structural properties
def test_sort_pairs_is_stable_argsort():
    rng = np.random.default_rng(5)
    ids = rng.integers(0, 9, size=(50, 3)).astype(np.int32)
    st, sf, off = O.sort_pairs(ids, 9)
    order = np.argsort(ids.ravel(), kind="stable")
    np.testing.assert_array_equal(sf, order)
    np.testing.assert_array_equal(st, order // 3)
    np.testing.assert_array_equal(off, np.concatenate([[0], np.cumsum(np.bincount(ids.ravel(), minlength=9))]))


def test_sorted_and_unsorted_paths_agree():
    # T*k = 60 takes the unsorted path, 64 the sorted one (model.cpp:683); tokens are
    # independent, so the first 15 rows must be identical bit for bit.
    shape = small_shape(tokens=16, shared=256, E=6, k=4)
    layer = S.make_layer(shape, 21)
    x = S.make_x(shape, 21)
    L = O.Layer(shape, layer)
    y16, ids16, _ = L.moe_block(x)
    y15, ids15, _ = L.moe_block(x[:15])
    np.testing.assert_array_equal(ids16[:15], ids15)
    np.testing.assert_array_equal(y16[:15], y15)


def test_forced_routing_reproduces_own_routing():
    shape = small_shape(tokens=9)
    layer = S.make_layer(shape, 4)
    x = S.make_x(shape, 4)
    L = O.Layer(shape, layer)
    y, ids, sc = L.moe_block(x)
    y2, ids2, _ = L.moe_block(x, forced_ids=ids, forced_scores=sc)
    np.testing.assert_array_equal(y, y2)


def test_norm_topk_scores_sum_to_one():
    shape = small_shape(tokens=20, E=16, k=4, norm=True, shared=0)
    layer = S.make_layer(shape, 8)
    x = S.make_x(shape, 8)
    ids, sc, _, pr = O.route(x, layer["router_w"], 4, norm_topk=True)
    s = S.bf16_to_f32(sc).sum(1)
    assert np.all(np.abs(s - 1.0) < 2e-2)


def test_topk_is_descending_and_matches_probs():
    shape = small_shape(tokens=30, E=60, k=4, shared=0)
    layer = S.make_layer(shape, 9)
    x = S.make_x(shape, 9)
    ids, sc, lg, pr = O.route(x, layer["router_w"], 4)
    p = S.bf16_to_f32(pr)
    top = np.argsort(-p, axis=1, kind="stable")[:, :4]
    assert same_sets(ids, top).all()
    np.testing.assert_array_equal(np.take_along_axis(pr, ids, 1), sc)


def test_router_bias_skews_load():
    shape = S.MoEShape("zipf", 256, 128, 8, 2, 256, True, 0, 1.2)
    layer = S.make_layer(shape, 2)
    x = S.make_x(shape, 2)
    ids, _, _, _ = O.route(x, layer["router_w"], 2, norm_topk=True, router_bias=layer["router_bias"])
    cnt = np.bincount(ids.ravel(), minlength=8)
    hot = int(np.argmax(S.bf16_to_f32(layer["router_bias"])))
    assert cnt[hot] == cnt.max() and cnt.max() > 2 * cnt.min()


# ------------------------------------------------------------------ synthetic generator
def test_synthetic_is_seeded_and_mlx_layout():
    shape = S.CONFIGS["qwen15_decode"]
    a = S.make_qmatrix(0, "gate", (2,), 16, 2048)
    b = S.make_qmatrix(0, "gate", (2,), 16, 2048)
    for u, v in zip(a, b):
        np.testing.assert_array_equal(u, v)
    w, s, bias = a
    assert w.shape == (2, 16, 256) and w.dtype == np.uint32 and s.shape == (2, 16, 32)
    np.testing.assert_array_equal(S.bf16_to_f32(bias), -8 * S.bf16_to_f32(s))
    assert S.layer_weight_bytes(shape)["expert"] == 4866048
    assert S.layer_weight_bytes(shape)["shared"] == 19464192
