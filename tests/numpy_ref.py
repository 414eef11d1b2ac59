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


def relu2(u):
    """bf16(max(u, 0)^2) of bf16 bits u (nemotron_h.cpp:53-58)."""
    r = np.maximum(bf16_to_f32(u), 0.0).astype(np.float32)
    return f32_to_bf16(r * r)


def sigmoid_route(x, router_w, bias, k, n_group=1, topk_group=1, norm=False, scale=1.0):
    """The sigmoid routing of nemotron_h.cpp:1018-1050 in float64: ids [T, k] (selection
    order), scores [T, k], and the selection scores [T, E] used to find near-ties."""
    xf = bf16_to_f32(x).astype(np.float64)
    logits = rbf((xf @ bf16_to_f32(router_w).astype(np.float64).T).astype(np.float32)).astype(np.float64)
    orig = 1.0 / (1.0 + np.exp(-logits))
    sel = orig + (np.asarray(bias, np.float64) if bias is not None else 0.0)
    T, E = sel.shape
    if n_group > 1:
        g = sel.reshape(T, n_group, E // n_group)
        gscore = np.sort(g, axis=-1)[..., -2:].sum(-1)
        sel = sel.copy()
        for t in range(T):
            low = sorted(range(n_group), key=lambda gi: (gscore[t, gi], -gi))[: n_group - topk_group]
            for gi in low:
                sel[t, gi * (E // n_group):(gi + 1) * (E // n_group)] = 0.0
    ids = np.argsort(-sel, axis=-1, kind="stable")[:, :k]
    sc = np.take_along_axis(orig, ids, -1)
    if norm and k > 1:
        sc = sc / (sc.sum(-1, keepdims=True) + 1e-20)
    return ids.astype(np.int32), sc * scale, sel


def sigmoid_moe_block(layer: dict, shape, x, ids, scores):
    """fc1 -> relu2 -> fc2 per routed pair, fp32-scaled sum, plus the ungated shared
    expert (nemotron_h.cpp:1052-1106), for given routing."""
    T, k, H = x.shape[0], shape.top_k, shape.hidden
    xf = bf16_to_f32(x).astype(np.float64)
    y = np.zeros((T, H), np.float64)
    for t in range(T):
        for j in range(k):
            e = int(ids[t, j])
            W1 = dequant(layer["fc1"][0][e], layer["fc1"][1][e], layer["fc1"][2][e])
            W2 = dequant(layer["fc2"][0][e], layer["fc2"][1][e], layer["fc2"][2][e])
            u = f32_to_bf16((xf[t] @ W1.T).astype(np.float32))
            a = bf16_to_f32(relu2(u)).astype(np.float64)
            d = rbf((a @ W2.T).astype(np.float32)).astype(np.float64)
            y[t] += d * float(scores[t, j])
    y = rbf(y.astype(np.float32))
    if shape.shared_inter:
        Wu = dequant(*layer["shared_up"])
        Wd = dequant(*layer["shared_down"])
        u = f32_to_bf16((xf @ Wu.T).astype(np.float32))
        a = bf16_to_f32(relu2(u)).astype(np.float64)
        sh = rbf((a @ Wd.T).astype(np.float32))
        y = rbf(y + sh)
    return f32_to_bf16(np.asarray(y, np.float32))
