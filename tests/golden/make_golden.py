"""Writes tests/golden/kat.npz: known-answer cases for the MoE-block operators.

The reference ships no golden vectors for this path (its tests are end-to-end, dense
model only), so these cases are built from the layout and the arithmetic the
reference's MLX calls define, with outputs derived in closed form here (small
integers / dyadic values, exact in bf16) rather than computed by any implementation:

  nibble_order   quantized_matmul, one-hot x picks single dequantized elements:
                 MLX affine packing puts element j of a row at bits 4*(j%8) of word j/8
  group_bias     quantized_matmul across two quantization groups with distinct
                 scale / bias, w_hat = scale*q + bias (model.cpp:476-480)
  gather         gather_qmm with expert-constant weights, rhs / lhs indices
                 (model.cpp:703-721)
  router_ties    softmax top-k with exact logit ties: the lower expert id wins
                 (argpartition order is unspecified; ids compared as sets)
  one_expert     every token routed to the same expert (k=1 and k=2)

    python tests/golden/make_golden.py
"""
from __future__ import annotations

import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

from flashmlx_b200.synthetic import f32_to_bf16  # noqa: E402


def pack_rows(nibbles: np.ndarray) -> np.ndarray:
    """nibbles [N, K] in 0..15 -> [N, K/8] uint32 (element j at bits 4*(j%8))."""
    N, K = nibbles.shape
    q = nibbles.reshape(N, K // 8, 8).astype(np.uint32)
    return np.bitwise_or.reduce(q << (np.arange(8, dtype=np.uint32) * 4), axis=2).astype(np.uint32)


def bf(a):
    return f32_to_bf16(np.asarray(a, np.float32))


def main():
    out = {}
    # --- nibble_order: K=64, N=16; row n element k = (k%8 + n) % 8 (+8 for rows >= 8)
    K, N = 64, 16
    nib = np.zeros((N, K), np.int64)
    for n in range(N):
        for k in range(K):
            nib[n, k] = ((k % 8 + n) % 8) + (8 if n >= 8 else 0)
    x = np.zeros((8, K), np.float32)
    for m in range(8):
        x[m, m] = 1.0
    expect = np.array([[((m + n) % 8) + (8 if n >= 8 else 0) for n in range(N)] for m in range(8)], np.float32)
    out["nibble_order_x"] = bf(x)
    out["nibble_order_w"] = pack_rows(nib)
    out["nibble_order_s"] = bf(np.ones((N, 1)))
    out["nibble_order_b"] = bf(np.zeros((N, 1)))
    out["nibble_order_y"] = bf(expect)

    # --- group_bias: K=128 (two groups), N=16; q = 3 everywhere
    K, N = 128, 16
    nib = np.full((N, K), 3)
    s = np.zeros((N, 2), np.float32)
    b = np.zeros((N, 2), np.float32)
    for n in range(N):
        s[n] = [2.0, 0.5] if n % 2 == 0 else [1.0, -1.0]
        b[n] = [-1.0, 0.25] if n % 2 == 0 else [0.0, 8.0]
    x = np.zeros((2, K), np.float32)
    x[0, :] = 1.0
    x[1, :64] = 1.0
    w_hat = np.concatenate([np.repeat(s[:, :1] * 3 + b[:, :1], 64, 1), np.repeat(s[:, 1:] * 3 + b[:, 1:], 64, 1)], 1)
    expect = x.astype(np.float64) @ w_hat.T.astype(np.float64)   # 432 / 512 / 320 / 192: exact
    out["group_bias_x"] = bf(x)
    out["group_bias_w"] = pack_rows(nib)
    out["group_bias_s"] = bf(s)
    out["group_bias_b"] = bf(b)
    out["group_bias_y"] = bf(expect)

    # --- gather: E=3 experts, expert e has q = e+1, scale 1, bias 0; K=64, N=16
    E, K, N = 3, 64, 16
    w = np.stack([pack_rows(np.full((N, K), e + 1)) for e in range(E)])
    out["gather_w"] = w
    out["gather_s"] = bf(np.ones((E, N, 1)))
    out["gather_b"] = bf(np.zeros((E, N, 1)))
    xb = 4
    x = np.stack([np.full((1, K), float(bi + 1)) for bi in range(xb)]).astype(np.float32)  # [4, 1, 64]
    rhs = np.array([2, 0, 1, 1, 0, 2, 2, 1], np.uint32)  # B = 8 -> broadcast lhs(i) = i // 2
    lhs = np.array([3, 3, 0, 1, 2, 0, 1, 2], np.uint32)
    y_bcast = np.array([64.0 * (rhs[i] + 1) * (i // 2 + 1) for i in range(8)], np.float32)
    y_lhs = np.array([64.0 * (rhs[i] + 1) * (lhs[i] + 1) for i in range(8)], np.float32)
    out["gather_x"] = bf(x)
    out["gather_rhs"] = rhs
    out["gather_lhs"] = lhs
    out["gather_y_bcast"] = bf(np.repeat(y_bcast[:, None, None], N, 2))
    out["gather_y_lhs"] = bf(np.repeat(y_lhs[:, None, None], N, 2))

    # --- router_ties: E=8, H=64, x = ones; logits = c_e exactly (router rows c_e/64)
    c = np.array([1, 3, 3, 2, 3, 0, 1, 2], np.float32)
    out["router_ties_w"] = bf(np.repeat((c / 64.0)[:, None], 64, 1))
    out["router_ties_x"] = bf(np.ones((4, 64)))
    out["router_ties_ids_k2"] = np.tile(np.array([1, 2], np.int32), (4, 1))   # three 3s: lowest two ids
    out["router_ties_ids_k4"] = np.tile(np.array([1, 2, 4, 3], np.int32), (4, 1))  # then the lower of the 2s

    # --- one_expert: expert 5 of 6 gets logit 4, the others 0
    w1 = np.zeros((6, 64), np.float32)
    w1[5, :] = 1.0 / 16.0
    out["one_expert_w"] = bf(w1)
    out["one_expert_x"] = bf(np.ones((70, 64)))
    out["one_expert_ids_k1"] = np.full((70, 1), 5, np.int32)
    out["one_expert_ids_k2"] = np.tile(np.array([5, 0], np.int32), (70, 1))

    np.savez_compressed(os.path.join(HERE, "kat.npz"), **out)
    print("wrote", os.path.join(HERE, "kat.npz"), len(out), "arrays")


if __name__ == "__main__":
    main()
