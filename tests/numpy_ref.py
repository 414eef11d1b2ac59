"""A second, independent restatement of the MoE-block arithmetic in vectorised numpy
(float64 accumulation), used only to cross-check the C++ oracle on small cases."""
from __future__ import annotations

import numpy as np

from flashmlx_b200.synthetic import bf16_to_f32, f32_to_bf16


def rbf(a):
    return bf16_to_f32(f32_to_bf16(np.asarray(a, dtype=np.float32)))


def dequant(w, s, b, group_size=64, bits=4):
    """w [..., N, K*bits/32] u32 -> [..., N, K] float64 (exact)."""
    pf = 32 // bits
    shifts = (np.arange(pf, dtype=np.uint32) * bits)
    q = (w[..., None] >> shifts) & np.uint32((1 << bits) - 1)
    q = q.reshape(*w.shape[:-1], w.shape[-1] * pf).astype(np.float64)
    sf = np.repeat(bf16_to_f32(s).astype(np.float64), group_size, axis=-1)
    bf = np.repeat(bf16_to_f32(b).astype(np.float64), group_size, axis=-1) if b is not None else 0.0
    return sf * q + bf


def quantized_matmul(x, w, s, b, group_size=64, bits=4):
    W = dequant(w, s, b, group_size, bits)
    return f32_to_bf16((bf16_to_f32(x).astype(np.float64) @ W.T).astype(np.float32))


def swiglu(g, u):
    g = bf16_to_f32(g)
    u = bf16_to_f32(u)
    sg = rbf(1.0 / (1.0 + np.exp(-g.astype(np.float64))))
    return f32_to_bf16(rbf(g * sg) * u)


def moe_block(layer: dict, shape, x, ids, scores):
    """Expert part of moe_block for given routing (ids [T,k], scores bf16 [T,k])."""
    T = x.shape[0]
    k = shape.top_k
    H = shape.hidden
    xf = bf16_to_f32(x).astype(np.float64)
    y = np.zeros((T, H), np.float64)
    for t in range(T):
        acc = 0.0
        for j in range(k):
            e = int(ids[t, j])
            Wg = dequant(layer["gate"][0][e], layer["gate"][1][e], layer["gate"][2][e])
            Wu = dequant(layer["up"][0][e], layer["up"][1][e], layer["up"][2][e])
            Wd = dequant(layer["down"][0][e], layer["down"][1][e], layer["down"][2][e])
            g = f32_to_bf16((xf[t] @ Wg.T).astype(np.float32))
            u = f32_to_bf16((xf[t] @ Wu.T).astype(np.float32))
            a = bf16_to_f32(swiglu(g, u)).astype(np.float64)
            d = rbf((a @ Wd.T).astype(np.float32))
            acc = acc + rbf(d * bf16_to_f32(scores[t, j]))
        y[t] = rbf(acc)
    if shape.shared_inter:
        Wg = dequant(*layer["shared_gate"])
        Wu = dequant(*layer["shared_up"])
        Wd = dequant(*layer["shared_down"])
        g = f32_to_bf16((xf @ Wg.T).astype(np.float32))
        u = f32_to_bf16((xf @ Wu.T).astype(np.float32))
        a = bf16_to_f32(swiglu(g, u)).astype(np.float64)
        sh = rbf((a @ Wd.T).astype(np.float32))
        wg = bf16_to_f32(layer["shared_expert_gate_w"]).astype(np.float64)
        gl = rbf((xf @ wg.T).astype(np.float32))
        gs = rbf(1.0 / (1.0 + np.exp(-gl.astype(np.float64))))
        y = rbf(rbf(y) + rbf(gs * sh))
    return f32_to_bf16(y.astype(np.float32))
