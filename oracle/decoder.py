"""CPU restatement of the reference's full decoder forward (LlamaModel, Qwen1.5-MoE form),
the checker for the device decoder ops and the C++ decoder.

TEST INFRASTRUCTURE ONLY: imported by tests/ and the CPU leg of bench.py, never by the
product library.

PARITY UNPINNED: the reference runs these ops through MLX (mx::fast::rms_norm,
mx::fast::rope, mx::fast::scaled_dot_product_attention, mx::dequantize, mx::take,
mx::argmax), which is not available here and ships no golden vectors for them.  Each
function restates the op's documented arithmetic, rounding to bf16 at every MLX op
boundary as the reference's op sequence does:

  rms_norm       model.cpp:486-488 -> mx::fast::rms_norm: fp32 mean of squares,
                 n = 1 / sqrt(mean + eps), y = bf16(bf16(x * n) * w)
  add            model.cpp:824, 838 -> mx::add of two bf16 arrays: bf16(a + b)
  rope           model.cpp:588-589 -> mx::fast::rope(traditional=false, base=rope_theta,
                 scale=1, offset): pairs (i, i + d/2), inv_freq_i = base^(-2i/d) (computed
                 in float64, rounded to fp32), theta = fp32(pos) * inv_freq_i, rotation in fp32
  sdpa           model.cpp:630-635 -> mx::fast::scaled_dot_product_attention with scale
                 1/sqrt(d), causal for L > 1: fp32 scores, fp32 softmax, fp32 weighted sum
  attention      model.cpp:542-643: q/k/v quantized_matmul, bf16 bias adds, the optional
                 per-head RMSNorm of q and k (QK-norm, 573-581), rope,
                 slice_update of the bf16 cache at the batch's (uniform) offset, sdpa, o_proj
  block          model.cpp:813-839: x + attention(rms_norm(x)), then + moe_block / mlp
  mlp            model.cpp:645-656: down(swiglu(gate(x), up(x))), the swiglu of 14-25 with
                 bf16 rounding after every op
  embed          model.cpp:216-230, 490-496: the embedding table dequantized once to bf16
                 (bf16(fma(s, q, b))), rows taken by token id
  lm_head        model.cpp:499-520: quantized_matmul with lm_head.* (or the quantized
                 embedding when tie_word_embeddings)
  greedy         argmax of the bf16 logits, the first index among equal maxima
"""
from __future__ import annotations

import math

import numpy as np

from . import oracle as O


def bf16(a) -> np.ndarray:
    """fp32 -> bf16 bit patterns, round to nearest even (NaN stays NaN)."""
    u = np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)
    nan = (u & 0x7FFFFFFF) > 0x7F800000
    r = (u + (0x7FFF + ((u >> 16) & 1))) >> 16
    return np.where(nan, (u >> 16) | 0x40, r).astype(np.uint16)


def f32(b) -> np.ndarray:
    return (np.ascontiguousarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def add(a, b) -> np.ndarray:
    return bf16(f32(a) + f32(b))


def rms_norm(x, w, eps: float) -> np.ndarray:
    """x [..., H], w [H] bf16 bits -> bf16(bf16(x * n) * w), n = 1/sqrt(mean(x^2) + eps) in fp32."""
    xf = f32(x)
    ms = np.mean(xf * xf, axis=-1, keepdims=True, dtype=np.float32)
    n = np.float32(1.0) / np.sqrt(ms + np.float32(eps))
    return bf16(f32(bf16(xf * n)) * f32(w))


def inv_freq(head_dim: int, theta: float) -> np.ndarray:
    i = np.arange(head_dim // 2, dtype=np.float64)
    return np.exp2(-(2.0 * i / head_dim) * math.log2(theta)).astype(np.float32)


def rope(x, positions, n_heads: int, head_dim: int, theta: float) -> np.ndarray:
    """x [T, n_heads*head_dim] bf16 bits, positions [T] -> the rotated rows (bf16 bits)."""
    T = x.shape[0]
    half = head_dim // 2
    xf = f32(x).reshape(T, n_heads, head_dim)
    ang = np.asarray(positions, np.float32)[:, None] * inv_freq(head_dim, theta)[None, :]  # fp32
    c = np.cos(ang)[:, None, :]
    s = np.sin(ang)[:, None, :]
    x1, x2 = xf[..., :half], xf[..., half:]
    out = np.concatenate([x1 * c - x2 * s, x1 * s + x2 * c], axis=-1)
    return bf16(out.reshape(T, n_heads * head_dim))


def sdpa(q, cache_k, cache_v, B: int, L: int, offset: int, n_heads: int, n_kv_heads: int, head_dim: int,
         scale: float | None = None) -> np.ndarray:
    """q [B*L, n_heads*head_dim] (roped), caches [B, n_kv_heads, max_len, head_dim] holding
    positions [0, offset + L) -> out [B*L, n_heads*head_dim] bf16 bits.  The query at
    position offset + l attends keys 0 .. offset + l (causal; the single decode row attends
    the whole cache, which is the same set)."""
    scale = np.float32(1.0 / math.sqrt(head_dim) if scale is None else scale)
    group = n_heads // n_kv_heads
    total = offset + L
    qf = f32(q).reshape(B, L, n_heads, head_dim)
    kf = f32(cache_k[:, :, :total])
    vf = f32(cache_v[:, :, :total])
    out = np.empty((B, L, n_heads, head_dim), np.float32)
    for b in range(B):
        for h in range(n_heads):
            kh, vh = kf[b, h // group], vf[b, h // group]
            s = (qf[b, :, h] @ kh.T) * scale  # [L, total] fp32
            mask = np.arange(total)[None, :] > (offset + np.arange(L))[:, None]
            s = np.where(mask, -np.inf, s).astype(np.float32)
            p = np.exp(s - s.max(axis=-1, keepdims=True)).astype(np.float32)
            out[b, :, h] = (p @ vh) / p.sum(axis=-1, keepdims=True, dtype=np.float32)
    return bf16(out.reshape(B * L, n_heads * head_dim))


def dequantize(w, s, b, group_size: int = 64, bits: int = 4) -> np.ndarray:
    """[N, K*bits/32] codes + [N, K/gs] scales / biases -> [N, K] bf16(fma(s, q, b))."""
    pf = 32 // bits
    N = w.shape[0]
    shifts = (np.arange(pf, dtype=np.uint32) * bits)[None, None, :]
    q = ((np.asarray(w, np.uint32)[:, :, None] >> shifts) & ((1 << bits) - 1)).reshape(N, -1).astype(np.float32)
    K = q.shape[1]
    sf = np.repeat(f32(s), group_size, axis=1)[:, :K]
    bfv = np.repeat(f32(b), group_size, axis=1)[:, :K] if b is not None else np.zeros_like(sf)
    return bf16((sf.astype(np.float64) * q + bfv).astype(np.float32))  # one rounding of the exact s*q + b


def swiglu(g, u) -> np.ndarray:
    """silu(g) * u with bf16 rounding after every op (model.cpp:14-25): bf16(sigmoid(g)),
    bf16(g * that), bf16(that * u); sigmoid in fp32."""
    gf = f32(g)
    sg = f32(bf16(np.float32(1.0) / (np.float32(1.0) + np.exp(-gf))))
    return bf16(f32(bf16(gf * sg)) * f32(u))


def argmax(logits) -> np.ndarray:
    """First index of the maximum along the last axis (bf16 bits compared as values)."""
    return np.argmax(f32(logits), axis=-1).astype(np.int32)


class Decoder:
    """The forward pass over numpy weights (the layout of synthetic.make_decoder): per
    layer `in_norm`, `post_norm` [H] bf16, `q`, `k`, `v`, `o` (w, s, b), `q_bias`, `k_bias`,
    `v_bias` [n*d] bf16 (optional), and the MoE layer dict `moe`; the embedding `embed`
    (w, s, b), `norm` [H], `lm_head` (w, s, b) unless tied.  `cfg` has the fields of
    synthetic.DecoderShape (hidden, layers, n_heads, n_kv_heads, head_dim, vocab,
    rope_theta, rms_eps, moe, tie_word_embeddings, group_size, bits)."""

    def __init__(self, cfg, weights: dict, max_batch: int, max_len: int):
        self.cfg, self.w = cfg, weights
        self.moe = [O.Layer(cfg.moe, lw["moe"]) if "moe" in lw else None for lw in weights["layers"]]
        shape = (max_batch, cfg.n_kv_heads, max_len, cfg.head_dim)
        self.cache_k = [np.zeros(shape, np.uint16) for _ in range(cfg.layers)]
        self.cache_v = [np.zeros(shape, np.uint16) for _ in range(cfg.layers)]
        self.offset = 0

    def embed(self, ids) -> np.ndarray:
        """Rows of the dequantized embedding table for ids (only those rows are dequantized)."""
        ids = np.asarray(ids, np.int64).reshape(-1)
        w, s, b = self.w["embed"]
        uniq, inv = np.unique(ids, return_inverse=True)
        rows = dequantize(w[uniq], s[uniq], None if b is None else b[uniq], self.cfg.group_size, self.cfg.bits)
        return rows[inv]

    def _qmm(self, x, q):
        w, s, b = q
        return O.quantized_matmul(x, w, s, b, self.cfg.group_size, self.cfg.bits)

    def mlp(self, x, m):
        g, u = self._qmm(x, m["gate"]), self._qmm(x, m["up"])
        return self._qmm(swiglu(g, u), m["down"])

    def attention(self, x, li: int, B: int, L: int):
        c, lw = self.cfg, self.w["layers"][li]
        q, k, v = self._qmm(x, lw["q"]), self._qmm(x, lw["k"]), self._qmm(x, lw["v"])
        if lw.get("q_bias") is not None:
            q = add(q, lw["q_bias"][None, :])
        if lw.get("k_bias") is not None:
            k = add(k, lw["k_bias"][None, :])
        if lw.get("v_bias") is not None:
            v = add(v, lw["v_bias"][None, :])
        T = q.shape[0]
        if lw.get("q_norm") is not None:
            q = rms_norm(q.reshape(T, c.n_heads, c.head_dim), lw["q_norm"], c.rms_eps).reshape(T, -1)
        if lw.get("k_norm") is not None:
            k = rms_norm(k.reshape(T, c.n_kv_heads, c.head_dim), lw["k_norm"], c.rms_eps).reshape(T, -1)
        pos = self.offset + np.tile(np.arange(L), B)
        q = rope(q, pos, c.n_heads, c.head_dim, c.rope_theta)
        k = rope(k, pos, c.n_kv_heads, c.head_dim, c.rope_theta)
        ck, cv = self.cache_k[li], self.cache_v[li]
        ck[:B, :, self.offset:self.offset + L] = k.reshape(B, L, c.n_kv_heads, c.head_dim).transpose(0, 2, 1, 3)
        cv[:B, :, self.offset:self.offset + L] = v.reshape(B, L, c.n_kv_heads, c.head_dim).transpose(0, 2, 1, 3)
        a = sdpa(q, ck[:B], cv[:B], B, L, self.offset, c.n_heads, c.n_kv_heads, c.head_dim)
        return self._qmm(a, lw["o"])

    def forward(self, ids, trace: list | None = None):
        """ids [B, L] int -> logits of the last position [B, vocab] (bf16 bits); advances
        the cache offset by L.  `trace` (a list) collects each layer's output rows."""
        c = self.cfg
        ids = np.asarray(ids, np.int64)
        B, L = ids.shape
        if self.offset + L > self.cache_k[0].shape[2] or B > self.cache_k[0].shape[0]:
            raise ValueError("offset + L exceeds max_len, or B exceeds max_batch")
        x = self.embed(ids)
        for li, lw in enumerate(self.w["layers"]):
            h = add(x, self.attention(rms_norm(x, lw["in_norm"], c.rms_eps), li, B, L))
            n2 = rms_norm(h, lw["post_norm"], c.rms_eps)
            m = self.moe[li].moe_block(n2)[0] if self.moe[li] is not None else self.mlp(n2, lw["mlp"])
            x = add(h, m)
            if trace is not None:
                trace.append(x)
        self.offset += L
        last = x.reshape(B, L, c.hidden)[:, -1]
        n = rms_norm(last, self.w["norm"], c.rms_eps)
        head = self.w["embed"] if c.tie_word_embeddings else self.w["lm_head"]
        return self._qmm(n, head)

    def generate(self, prompt, steps: int) -> np.ndarray:
        """Greedy: prefill the prompt [B, L] (its argmax is token 1), then steps - 1
        single-token forwards -> [B, steps]."""
        prompt = np.asarray(prompt)
        if steps <= 0:
            return np.zeros((prompt.shape[0], 0), np.int32)
        out = [argmax(self.forward(prompt))]
        for _ in range(steps - 1):
            out.append(argmax(self.forward(out[-1][:, None])))
        return np.stack(out, axis=1)
