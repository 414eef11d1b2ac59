"""The CPU restatement of the full decoder (oracle/decoder.py) against independent forms of
its ops and against the properties the reference's forward has: the KV cache makes a
token-by-token pass equal to one pass over the whole sequence, causal attention does not
see later positions, RoPE at position 0 is the identity and preserves dot products under
a common shift, the dequantized embedding equals the oracle's bf16-weights product with
one-hot rows (model.cpp:216-230, 486-496, 542-643, 813-839)."""
from __future__ import annotations

import math

import numpy as np
import pytest

from flashmlx_b200 import synthetic as S
from oracle import decoder as D
from oracle import oracle as O

MOE = S.MoEShape("dec_moe", 256, 128, 4, 2, 0, False, 256)
SMALL = S.DecoderShape("dec_small", 256, 2, 4, 2, 64, 512, 1e6, 1e-6, MOE)


def _bf16(a):
    return D.bf16(np.asarray(a, np.float32))


def test_rms_norm_against_float64():
    rng = np.random.default_rng(0)
    x = _bf16(rng.standard_normal((16, 512)) * 3)
    w = _bf16(1 + 0.1 * rng.standard_normal(512))
    y = D.rms_norm(x, w, 1e-6)
    xf = D.f32(x).astype(np.float64)
    ref = xf / np.sqrt((xf * xf).mean(-1, keepdims=True) + 1e-6) * D.f32(w)
    np.testing.assert_allclose(D.f32(y), ref, rtol=2 ** -7, atol=1e-6)


def test_rope_identity_at_zero_and_shift_invariance():
    rng = np.random.default_rng(1)
    nh, d = 2, 64
    q = _bf16(rng.standard_normal((1, nh * d)))
    k = _bf16(rng.standard_normal((1, nh * d)))
    np.testing.assert_array_equal(D.rope(q, [0], nh, d, 1e6), q)  # cos 0 = 1, sin 0 = 0
    def dot(a, b):
        return (D.f32(a).reshape(nh, d) * D.f32(b).reshape(nh, d)).sum(-1)
    base = dot(D.rope(q, [37], nh, d, 1e4), D.rope(k, [5], nh, d, 1e4))
    shifted = dot(D.rope(q, [137], nh, d, 1e4), D.rope(k, [105], nh, d, 1e4))
    np.testing.assert_allclose(shifted, base, rtol=0.05, atol=0.1)  # bf16 rounding of the rotated rows


def test_rope_against_complex_rotation():
    rng = np.random.default_rng(2)
    nh, d, theta = 3, 128, 1e6
    x = _bf16(rng.standard_normal((5, nh * d)))
    pos = np.array([0, 1, 7, 300, 767])
    y = D.f32(D.rope(x, pos, nh, d, theta)).reshape(5, nh, d)
    xf = D.f32(x).reshape(5, nh, d).astype(np.float64)
    inv = theta ** (-2.0 * np.arange(d // 2) / d)
    z = (xf[..., : d // 2] + 1j * xf[..., d // 2:]) * np.exp(1j * pos[:, None, None] * inv[None, None, :])
    np.testing.assert_allclose(y, np.concatenate([z.real, z.imag], -1), rtol=2 ** -7, atol=2e-3)


def _cache(rng, B, nkv, max_len, d, total):
    ck = np.zeros((B, nkv, max_len, d), np.uint16)
    cv = np.zeros_like(ck)
    ck[:, :, :total] = _bf16(rng.standard_normal((B, nkv, total, d)))
    cv[:, :, :total] = _bf16(rng.standard_normal((B, nkv, total, d)))
    return ck, cv


def test_sdpa_against_float64_and_causality():
    rng = np.random.default_rng(3)
    B, L, off, nh, nkv, d = 2, 5, 3, 4, 2, 64
    ck, cv = _cache(rng, B, nkv, 16, d, off + L)
    q = _bf16(rng.standard_normal((B * L, nh * d)))
    out = D.f32(D.sdpa(q, ck, cv, B, L, off, nh, nkv, d)).reshape(B, L, nh, d)
    qf = D.f32(q).reshape(B, L, nh, d).astype(np.float64)
    for b in range(B):
        for h in range(nh):
            for l in range(L):
                kk = D.f32(ck[b, h // 2, : off + l + 1]).astype(np.float64)
                vv = D.f32(cv[b, h // 2, : off + l + 1]).astype(np.float64)
                s = kk @ qf[b, l, h] / math.sqrt(d)
                p = np.exp(s - s.max())
                np.testing.assert_allclose(out[b, l, h], p @ vv / p.sum(), rtol=2 ** -7, atol=1e-3)
    # a later position's cache entries do not change an earlier row
    ck2, cv2 = ck.copy(), cv.copy()
    ck2[:, :, off + L - 1] = _bf16(rng.standard_normal((B, nkv, d)))
    cv2[:, :, off + L - 1] = _bf16(rng.standard_normal((B, nkv, d)))
    out2 = D.f32(D.sdpa(q, ck2, cv2, B, L, off, nh, nkv, d)).reshape(B, L, nh, d)
    np.testing.assert_array_equal(out2[:, : L - 1], out[:, : L - 1])
    assert not np.array_equal(out2[:, L - 1], out[:, L - 1])


def test_dequantize_matches_bf16_weight_product():
    w, s, b = S.make_qmatrix(4, "deq", (), 96, 256, 64, 4, scale_std=0.1)
    table = D.dequantize(w, s, b)
    eye = _bf16(np.eye(256))
    with O.weight_rounding(O.BF16_WEIGHTS):
        t2 = O.quantized_matmul(eye, w, s, b)  # [K, N]: row j = dequantized column j
    np.testing.assert_array_equal(table, t2.T)


def test_argmax_first_of_ties():
    lg = _bf16(np.array([[1, 3, 3, 2], [5, 5, 5, 5], [-1, -2, -0.5, -0.5]]))
    np.testing.assert_array_equal(D.argmax(lg), [1, 0, 2])


def test_cache_pass_equals_full_pass():
    """Prefill L tokens then one decode step gives the logits of a prefill of L+1 tokens."""
    w = S.make_decoder(SMALL, 5)
    ids = np.random.default_rng(5).integers(0, SMALL.vocab, (2, 7))
    a = D.Decoder(SMALL, w, 2, 16)
    a.forward(ids[:, :6])
    step = a.forward(ids[:, 6:7])
    full = D.Decoder(SMALL, w, 2, 16).forward(ids)
    np.testing.assert_array_equal(step, full)


def test_generate_is_greedy_stepping():
    w = S.make_decoder(SMALL, 6)
    ids = np.random.default_rng(6).integers(0, SMALL.vocab, (2, 5))
    toks = D.Decoder(SMALL, w, 2, 16).generate(ids, 4)
    ref = D.Decoder(SMALL, w, 2, 16)
    t = D.argmax(ref.forward(ids))
    seq = [t]
    for _ in range(3):
        t = D.argmax(ref.forward(t[:, None]))
        seq.append(t)
    np.testing.assert_array_equal(toks, np.stack(seq, 1))
    assert toks.shape == (2, 4)


def test_tied_embeddings_use_the_quantized_embedding():
    sh = S.DecoderShape("tied", 256, 1, 4, 4, 64, 300, 1e4, 1e-5, MOE, tie_word_embeddings=True)
    w = S.make_decoder(sh, 7)
    assert "lm_head" not in w
    dec = D.Decoder(sh, w, 1, 8)
    lg = dec.forward(np.array([[3, 4]]))
    assert lg.shape == (1, 300)


@pytest.mark.parametrize("name", list(S.DECODER_CONFIGS))
def test_decoder_configs_are_consistent(name):
    sh = S.DECODER_CONFIGS[name]
    assert sh.n_heads % sh.n_kv_heads == 0 and sh.head_dim in (64, 128)
    assert sh.moe.hidden == sh.hidden


MIXED = S.DecoderShape("dec_mixed", 256, 3, 4, 2, 64, 320, 1e6, 1e-6, MOE, dense_layers=(0,), intermediate=384)


def test_dense_layer_mlp():
    """A dense layer's MLP: down(swiglu(gate(x), up(x))) with the compiled swiglu's bf16
    rounding after every op (model.cpp:14-25, 645-656), against a float64 restatement of
    the same rounding chain."""
    w = S.make_decoder(MIXED, 8)
    assert "mlp" in w["layers"][0] and "moe" in w["layers"][1]
    dec = D.Decoder(MIXED, w, 1, 8)
    x = _bf16(np.random.default_rng(8).standard_normal((5, 256)))
    m = w["layers"][0]["mlp"]
    g, u = O.quantized_matmul(x, *m["gate"]), O.quantized_matmul(x, *m["up"])
    gf = D.f32(g).astype(np.float64)
    sg = D.f32(_bf16(1.0 / (1.0 + np.exp(-gf))))
    act = _bf16(D.f32(_bf16(gf * sg)) * D.f32(u))
    np.testing.assert_array_equal(dec.mlp(x, m), O.quantized_matmul(act, *m["down"]))


def test_mixed_decoder_cache_pass_equals_full_pass():
    w = S.make_decoder(MIXED, 9)
    ids = np.random.default_rng(9).integers(0, MIXED.vocab, (2, 6))
    a = D.Decoder(MIXED, w, 2, 8)
    a.forward(ids[:, :5])
    np.testing.assert_array_equal(a.forward(ids[:, 5:6]), D.Decoder(MIXED, w, 2, 8).forward(ids))


QKN = S.DecoderShape("dec_qkn", 256, 2, 4, 2, 64, 320, 1e6, 1e-6, MOE, attn_bias=False, qk_norm=True)


def test_qk_norm_decoder():
    """Qwen3-style QK-norm (model.cpp:573-581): the per-head RMSNorm of q and k changes the
    logits, and the cached pass still equals the full pass."""
    w = S.make_decoder(QKN, 10)
    assert "q_norm" in w["layers"][0] and "q_bias" not in w["layers"][0]
    ids = np.random.default_rng(10).integers(0, QKN.vocab, (2, 6))
    a = D.Decoder(QKN, w, 2, 8)
    a.forward(ids[:, :5])
    step = a.forward(ids[:, 5:6])
    np.testing.assert_array_equal(step, D.Decoder(QKN, w, 2, 8).forward(ids))
    plain = {**w, "layers": [{k: v for k, v in lw.items() if k not in ("q_norm", "k_norm")} for lw in w["layers"]]}
    assert not np.array_equal(D.Decoder(QKN, plain, 2, 8).forward(ids), D.Decoder(QKN, w, 2, 8).forward(ids))


def test_query_width_differs_from_hidden():
    """Qwen3-style attention whose query width (heads x head_dim) is twice the hidden size,
    with GQA and QK-norm: the cached pass still equals the full pass."""
    sh = S.DecoderShape("dec_wide", 256, 2, 8, 2, 64, 320, 1e6, 1e-6, MOE, attn_bias=False, qk_norm=True)
    w = S.make_decoder(sh, 11)
    assert w["layers"][0]["q"][0].shape == (512, 256 // 8) and w["layers"][0]["o"][0].shape == (256, 512 // 8)
    ids = np.random.default_rng(11).integers(0, sh.vocab, (2, 5))
    a = D.Decoder(sh, w, 2, 8)
    a.forward(ids[:, :4])
    np.testing.assert_array_equal(a.forward(ids[:, 4:5]), D.Decoder(sh, w, 2, 8).forward(ids))


def test_fused_qkv_rows_equal_separate_projections():
    """The decoder's fused q|k|v matrix (the three matrices' rows, scales and biases
    concatenated) gives the three projections side by side, bit for bit: the rows of a
    quantized linear do not interact (model.cpp:476-480 per projection)."""
    rng = np.random.default_rng(12)
    H, QD, KVD = 256, 512, 128
    mats = [S.make_qmatrix(20 + i, f"p{i}", (), n, H, 64, 4, scale_std=0.05) for i, n in enumerate((QD, KVD, KVD))]
    fused = tuple(np.concatenate([m[j] for m in mats], axis=0) for j in range(3))
    x = _bf16(rng.standard_normal((7, H)))
    sep = np.concatenate([O.quantized_matmul(x, *m) for m in mats], axis=1)
    np.testing.assert_array_equal(O.quantized_matmul(x, *fused), sep)


def test_logits_form_gap():
    """The whole-decoder logits bound of the GPU tests (DECODER_LOGITS) is set from the
    gap between MLX's two valid arithmetic forms of the 4-bit products (exact weights, as
    qmv; bf16-rounded weights, as qmm) on the small test decoder: the gap must be real
    (larger than the per-op bound) and inside DECODER_LOGITS."""
    from tests._parity import DECODER_LOGITS, MAE_REL, metrics
    sm = S.DecoderShape("dec_small", 256, 2, 4, 2, 64, 320, 1e6, 1e-6, MOE)
    w = S.make_decoder(sm, 71)
    prompt = np.random.default_rng(71).integers(0, sm.vocab, (2, 9)).astype(np.int32)

    def run():
        d = D.Decoder(sm, w, 2, 16)
        outs = [d.forward(prompt)]
        for _ in range(3):
            outs.append(d.forward(D.argmax(outs[0])[:, None]))
        return outs

    exact = run()
    with O.weight_rounding(O.BF16_WEIGHTS):
        rounded = run()
    gaps = [metrics(a, b) for a, b in zip(exact, rounded)]
    worst = max(g["mae_rel"] for g in gaps)
    assert worst > 2 * MAE_REL, gaps
    assert all(g["max_rel"] <= DECODER_LOGITS["max_rel"] and g["mae_rel"] <= DECODER_LOGITS["mae_rel"]
               for g in gaps), gaps
