"""The decoder's device ops (fm_dequantize, fm_embed, fm_rms_norm, fm_attention,
fm_swiglu, fm_argmax) and the C++ Decoder (host/decoder.cpp, through fmh.h) against the
CPU restatement of the reference's forward (oracle/decoder.py: model.cpp:486-660,
813-839, sampling.cpp:5-7).

Integer and copy ops are bit-exact.  Floating-point ops are held to the north-star
tolerances (tests/_parity.py); attention rounds its softmax probabilities to bf16 for
the tensor-core product, so its outputs are compared normwise.  The whole-model logits
carry two layers of such differences plus the two 4-bit GEMM forms, and are compared
with DECODER_LOGITS, a bound set from the gap between the oracle's own two forms on
the same logits (tests/test_oracle_decoder.py::test_logits_form_gap pins it); greedy
tokens must agree wherever the oracle's top two logits are more than a few ulps apart."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from flashmlx_b200 import synthetic as S
from oracle import decoder as D
from tests._parity import DECODER_LOGITS, TIGHT, assert_close

pytestmark = pytest.mark.gpu


def _dev(a):
    from flashmlx_b200 import ops
    return ops.bf16_from_numpy(a, "cuda")


def _host(t):
    from flashmlx_b200 import ops
    torch.cuda.synchronize()
    return ops.bf16_to_numpy(t)


def _rnd(rng, shape, std=1.0):
    return D.bf16(rng.standard_normal(shape).astype(np.float32) * std)


def test_dequantize_bit_exact():
    from flashmlx_b200 import ops
    w, s, b = S.make_qmatrix(61, "deq", (), 320, 512, 64, 4, scale_std=0.1)
    got = ops.dequantize(ops.u32_from_numpy(w, "cuda"), _dev(s), _dev(b))
    np.testing.assert_array_equal(_host(got), D.dequantize(w, s, b))


def test_embed_rows_and_bad_ids():
    from flashmlx_b200 import _lib, ops
    rng = np.random.default_rng(62)
    table = _rnd(rng, (50, 256))
    ids = np.array([[0, 49, 7], [7, 3, 0]], np.int32)
    got = ops.embed(_dev(table), torch.from_numpy(ids).cuda())
    np.testing.assert_array_equal(_host(got), table[ids])
    h = ops.default_handle(torch.cuda.current_device())
    h.sync()
    bad = torch.tensor([1, 50], dtype=torch.int32, device="cuda")
    y = ops.embed(_dev(table), bad)
    with pytest.raises(_lib.FlashMoEError) as e:
        h.sync()  # the out-of-range id is a device-side bounds failure
    assert e.value.status == _lib.FM_EDEVICE
    np.testing.assert_array_equal(_host(y)[1], np.zeros(256, np.uint16))


@pytest.mark.parametrize("residual", [False, True])
@pytest.mark.parametrize("H", [256, 2048, 2056])
def test_rms_norm(residual, H):
    from flashmlx_b200 import ops
    rng = np.random.default_rng(63)
    x = _rnd(rng, (37, H), 2.0)
    r = _rnd(rng, (37, H)) if residual else None
    w = D.bf16(1 + 0.1 * rng.standard_normal(H).astype(np.float32))
    xt = _dev(x)
    h_out = xt if residual else None  # in place: x becomes x + r
    y = ops.rms_norm(xt, _dev(w), 1e-6, residual=_dev(r) if residual else None, h_out=h_out)
    h = D.add(x, r) if residual else x
    if residual:
        np.testing.assert_array_equal(_host(xt), h)
    assert_close(_host(y), D.rms_norm(h, w, 1e-6), f"rms_norm H={H} residual={residual}", **TIGHT)


@pytest.mark.parametrize("B,L,offset,nh,nkv,d", [
    (1, 1, 0, 4, 4, 128),      # the first decode position
    (2, 9, 0, 4, 2, 64),       # prefill, GQA
    (1, 70, 0, 2, 2, 128),     # two query tiles
    (3, 1, 77, 4, 4, 128),     # decode across a key-block boundary
    (2, 66, 60, 2, 1, 128),    # a prefill continuing a cache
])
def test_attention_against_oracle(B, L, offset, nh, nkv, d):
    from flashmlx_b200 import ops
    rng = np.random.default_rng(64 + L + offset)
    max_len = offset + L + 5
    theta = 1e6
    # caches hold positions [0, offset) from an earlier call (random), the rest is garbage
    ck = np.full((B, nkv, max_len, d), 0x7FC0, np.uint16)  # NaN: must never be read
    cv = ck.copy()
    ck[:, :, :offset] = _rnd(rng, (B, nkv, offset, d))
    cv[:, :, :offset] = _rnd(rng, (B, nkv, offset, d))
    q, k, v = _rnd(rng, (B * L, nh * d)), _rnd(rng, (B * L, nkv * d)), _rnd(rng, (B * L, nkv * d))
    bq, bk, bv = _rnd(rng, nh * d, 0.02), _rnd(rng, nkv * d, 0.02), _rnd(rng, nkv * d, 0.02)
    qt, ckt, cvt = _dev(q), _dev(ck), _dev(cv)
    out = ops.attention(qt, _dev(k), _dev(v), ckt, cvt, B, L, offset, theta, q_bias=_dev(bq), k_bias=_dev(bk),
                        v_bias=_dev(bv))
    pos = offset + np.tile(np.arange(L), B)
    q_ref = D.rope(D.add(q, bq[None]), pos, nh, d, theta)
    k_ref = D.rope(D.add(k, bk[None]), pos, nkv, d, theta)
    v_ref = D.add(v, bv[None])
    ck_ref, cv_ref = ck.copy(), cv.copy()
    ck_ref[:, :, offset:offset + L] = k_ref.reshape(B, L, nkv, d).transpose(0, 2, 1, 3)
    cv_ref[:, :, offset:offset + L] = v_ref.reshape(B, L, nkv, d).transpose(0, 2, 1, 3)
    # rotated q and the cache rows: RoPE's cos / sin may differ by an fp32 ulp from numpy's
    assert_close(_host(qt), q_ref, "rope q", max_rel=1e-2, mae_rel=1e-4)
    got_ck, got_cv = _host(ckt), _host(cvt)
    np.testing.assert_array_equal(got_cv[:, :, :offset + L], cv_ref[:, :, :offset + L])
    np.testing.assert_array_equal(got_ck[:, :, :offset], ck_ref[:, :, :offset])
    assert_close(got_ck[:, :, offset:offset + L], ck_ref[:, :, offset:offset + L], "rope k", max_rel=1e-2, mae_rel=1e-4)
    ref = D.sdpa(q_ref, ck_ref, cv_ref, B, L, offset, nh, nkv, d)
    assert_close(_host(out), ref, f"sdpa B={B} L={L} offset={offset}", max_rel=2e-2, mae_rel=5e-3)


@pytest.mark.parametrize("d", [64, 128])
def test_attention_on_fused_qkv_rows(d):
    """fm_attention with qkv_ld (q, k, v side by side in one [T, (nh + 2 n_kv) d] buffer,
    the fused projection's output) gives the separate-buffer call's output, rotated q and
    caches bit for bit."""
    from flashmlx_b200 import ops
    rng = np.random.default_rng(70 + d)
    B, L, offset, nh, nkv, max_len, theta = 2, 7, 3, 4, 2, 16, 1e6
    ck = np.zeros((B, nkv, max_len, d), np.uint16)
    ck[:, :, :offset] = _rnd(rng, (B, nkv, offset, d))
    cv = ck.copy()
    q, k, v = _rnd(rng, (B * L, nh * d)), _rnd(rng, (B * L, nkv * d)), _rnd(rng, (B * L, nkv * d))
    bq, bk, bv = _rnd(rng, nh * d, 0.02), _rnd(rng, nkv * d, 0.02), _rnd(rng, nkv * d, 0.02)
    qn, kn = _rnd(rng, d, 0.1), _rnd(rng, d, 0.1)
    extra = dict(q_bias=_dev(bq), k_bias=_dev(bk), v_bias=_dev(bv), q_norm=_dev(qn), k_norm=_dev(kn))
    qt, ck1, cv1 = _dev(q), _dev(ck), _dev(cv)
    out1 = ops.attention(qt, _dev(k), _dev(v), ck1, cv1, B, L, offset, theta, **extra)
    qkv = _dev(np.concatenate([q, k, v], axis=1))
    ck2, cv2 = _dev(ck), _dev(cv)
    out2 = ops.attention_qkv(qkv, ck2, cv2, B, L, offset, theta, **extra)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(_host(out2), _host(out1))
    np.testing.assert_array_equal(_host(qkv)[:, :nh * d], _host(qt))
    np.testing.assert_array_equal(_host(qkv)[:, nh * d:], np.concatenate([k, v], axis=1))  # k, v read only
    np.testing.assert_array_equal(_host(ck2), _host(ck1))
    np.testing.assert_array_equal(_host(cv2), _host(cv1))


@pytest.mark.parametrize("d", [64, 128])
def test_attention_with_qk_norm(d):
    """QK-norm inside fm_attention: each q / k head RMS-normalised (after the bias, before
    RoPE), against the oracle's rms_norm of the reshaped heads."""
    from flashmlx_b200 import ops
    rng = np.random.default_rng(68 + d)
    B, L, nh, nkv, max_len, theta, eps = 2, 5, 4, 2, 8, 1e6, 1e-6
    ck = np.zeros((B, nkv, max_len, d), np.uint16)
    cv = ck.copy()
    q, k, v = _rnd(rng, (B * L, nh * d), 3.0), _rnd(rng, (B * L, nkv * d), 3.0), _rnd(rng, (B * L, nkv * d))
    qn, kn = D.bf16(1 + 0.1 * rng.standard_normal(d).astype(np.float32)), D.bf16(
        1 + 0.1 * rng.standard_normal(d).astype(np.float32))
    qt, ckt, cvt = _dev(q), _dev(ck), _dev(cv)
    out = ops.attention(qt, _dev(k), _dev(v), ckt, cvt, B, L, 0, theta, q_norm=_dev(qn), k_norm=_dev(kn),
                        norm_eps=eps)
    T = B * L
    pos = np.tile(np.arange(L), B)
    q_ref = D.rope(D.rms_norm(q.reshape(T, nh, d), qn, eps).reshape(T, -1), pos, nh, d, theta)
    k_ref = D.rope(D.rms_norm(k.reshape(T, nkv, d), kn, eps).reshape(T, -1), pos, nkv, d, theta)
    assert_close(_host(qt), q_ref, "qk-norm q", max_rel=1e-2, mae_rel=1e-4)
    ck_ref = ck.copy()
    ck_ref[:, :, :L] = k_ref.reshape(B, L, nkv, d).transpose(0, 2, 1, 3)
    assert_close(_host(ckt), ck_ref, "qk-norm k cache", max_rel=1e-2, mae_rel=1e-4)
    cv_ref = cv.copy()
    cv_ref[:, :, :L] = v.reshape(B, L, nkv, d).transpose(0, 2, 1, 3)
    ref = D.sdpa(q_ref, ck_ref, cv_ref, B, L, 0, nh, nkv, d)
    assert_close(_host(out), ref, "qk-norm sdpa", max_rel=2e-2, mae_rel=5e-3)


@pytest.mark.parametrize("M,K,N", [(1, 2048, 2048), (32, 2048, 512), (100, 1408, 2048), (600, 2048, 1024),
                                   (3, 2112, 256)])
def test_linear_equals_quantized_matmul(M, K, N):
    """fm_linear (rows laid out by dense_prep_kernel) gives fm_quantized_matmul's output bit
    for bit: the same GEMM kernels on either expert path (GEMV for few rows, tcgen05 for
    many; K % 128 == 64 always tcgen05)."""
    from flashmlx_b200 import ops
    rng = np.random.default_rng(M + K + N)
    w, s, b = S.make_qmatrix(67, "lin", (), N, K, 64, 4)
    x = _rnd(rng, (M, K))
    wt, st, bt, xt = ops.u32_from_numpy(w, "cuda"), _dev(s), _dev(b), _dev(x)
    a = ops.linear(xt, wt, st, bt)
    ref = ops.quantized_matmul(xt, wt, st, bt)
    np.testing.assert_array_equal(_host(a), _host(ref))


def test_swiglu():
    from flashmlx_b200 import ops
    rng = np.random.default_rng(65)
    g, u = _rnd(rng, (7, 1408), 3.0), _rnd(rng, (7, 1408))
    gf, uf = D.f32(g), D.f32(u)
    ref = D.bf16(D.f32(D.bf16(gf * D.f32(D.bf16(1 / (1 + np.exp(-gf)))))) * uf)
    assert_close(_host(ops.swiglu(_dev(g), _dev(u))), ref, "swiglu", max_rel=1e-2, mae_rel=1e-4)


def test_argmax_first_of_ties():
    from flashmlx_b200 import ops
    rng = np.random.default_rng(66)
    lg = _rnd(rng, (6, 151936))
    lg[1, [5, 100000]] = D.bf16(np.float32(50.0))   # a tie: the lower index wins
    lg[2, :] = D.bf16(np.float32(-3.0))             # all equal
    lg[3, 151935] = D.bf16(np.float32(99.0))        # the last element
    got = ops.argmax(_dev(lg))
    torch.cuda.synchronize()
    np.testing.assert_array_equal(got.cpu().numpy(), D.argmax(lg))


# ---------------------------------------------------------------- the whole decoder
MOE = S.MoEShape("dec_moe", 256, 128, 4, 2, 0, False, 256)
SMALL = S.DecoderShape("dec_small", 256, 2, 4, 2, 64, 320, 1e6, 1e-6, MOE)


def _clear_tokens(logits_bits, ulps=4):
    """Rows whose top two logits are more than `ulps` bf16 ulps apart (at their scale)."""
    f = np.sort(D.f32(logits_bits), axis=-1)
    gap = f[:, -1] - f[:, -2]
    return gap > ulps * np.abs(f[:, -1]) * 2.0 ** -8


def test_decoder_against_oracle():
    from flashmlx_b200 import decoder as DEC
    w = S.make_decoder(SMALL, 71)
    B, L = 2, 9
    prompt = np.random.default_rng(71).integers(0, SMALL.vocab, (B, L)).astype(np.int32)
    dec = DEC.Decoder.from_weights(SMALL, DEC.upload_weights(w, "cuda"), "cuda", B, 16)
    ora = D.Decoder(SMALL, w, B, 16)
    nxt = dec.forward(torch.from_numpy(prompt).cuda())
    ref = ora.forward(prompt)
    assert_close(_host(dec.logits(B, SMALL.vocab, "cuda")), ref, "prefill logits", **DECODER_LOGITS)
    clear = _clear_tokens(ref)
    np.testing.assert_array_equal(nxt.cpu().numpy()[clear], D.argmax(ref)[clear])
    # teacher-forced decode steps: both sides take the oracle's tokens
    tok = D.argmax(ref)
    for step in range(3):
        dec.forward(torch.from_numpy(tok[:, None].copy()).cuda())
        ref = ora.forward(tok[:, None])
        assert_close(_host(dec.logits(B, SMALL.vocab, "cuda")), ref, f"decode step {step} logits", **DECODER_LOGITS)
        tok = D.argmax(ref)
    assert dec.offset == L + 3


def test_decoder_from_checkpoint_and_generate(tmp_path):
    """fmh_decoder_open over a written checkpoint equals the decoder over the same weights
    uploaded directly (same kernels, bit for bit); generate() equals manual stepping."""
    from flashmlx_b200 import decoder as DEC
    from tests.decoder_util import write_decoder_checkpoint
    w = S.make_decoder(SMALL, 72)
    write_decoder_checkpoint(str(tmp_path), SMALL, w)
    B, L, steps = 2, 6, 5
    prompt = np.random.default_rng(72).integers(0, SMALL.vocab, (B, L)).astype(np.int32)
    a = DEC.Decoder.open(str(tmp_path), "cuda", B, L + steps)
    b = DEC.Decoder.from_weights(SMALL, DEC.upload_weights(w, "cuda"), "cuda", B, L + steps)
    ta = a.generate(prompt, steps)
    tb = b.generate(prompt, steps)
    np.testing.assert_array_equal(ta, tb)
    b.reset()
    seq = [b.forward(torch.from_numpy(prompt).cuda())]
    for _ in range(steps - 1):
        seq.append(b.forward(seq[-1][:, None].contiguous()))
    np.testing.assert_array_equal(torch.stack(seq, 1).cpu().numpy(), tb)


def test_mixed_decoder_with_a_dense_layer():
    """A dense SwiGLU layer (fm_linear, fm_swiglu, fm_linear) followed by MoE layers."""
    from flashmlx_b200 import decoder as DEC
    mixed = S.DecoderShape("dec_mixed", 256, 3, 4, 2, 64, 320, 1e6, 1e-6, MOE, dense_layers=(0,), intermediate=384)
    w = S.make_decoder(mixed, 73)
    B, L = 2, 7
    prompt = np.random.default_rng(73).integers(0, mixed.vocab, (B, L)).astype(np.int32)
    dec = DEC.Decoder.from_weights(mixed, DEC.upload_weights(w, "cuda"), "cuda", B, 12)
    dec.forward(torch.from_numpy(prompt).cuda())
    ref = D.Decoder(mixed, w, B, 12).forward(prompt)
    assert_close(_host(dec.logits(B, mixed.vocab, "cuda")), ref, "mixed decoder logits", **DECODER_LOGITS)


def test_qk_norm_decoder_against_oracle():
    from flashmlx_b200 import decoder as DEC
    qkn = S.DecoderShape("dec_qkn", 256, 2, 4, 2, 64, 320, 1e6, 1e-6, MOE, attn_bias=False, qk_norm=True)
    w = S.make_decoder(qkn, 74)
    B, L = 2, 7
    prompt = np.random.default_rng(74).integers(0, qkn.vocab, (B, L)).astype(np.int32)
    dec = DEC.Decoder.from_weights(qkn, DEC.upload_weights(w, "cuda"), "cuda", B, 12)
    dec.forward(torch.from_numpy(prompt).cuda())
    ref = D.Decoder(qkn, w, B, 12).forward(prompt)
    assert_close(_host(dec.logits(B, qkn.vocab, "cuda")), ref, "qk-norm decoder logits", **DECODER_LOGITS)


def test_wide_query_gqa_decoder_against_oracle():
    """Query width twice the hidden size (8 heads of 64 over hidden 256), 2 KV heads, QK-norm:
    the Qwen3-30B-A3B layout in small."""
    from flashmlx_b200 import decoder as DEC
    sh = S.DecoderShape("dec_wide", 256, 2, 8, 2, 64, 320, 1e6, 1e-6, MOE, attn_bias=False, qk_norm=True)
    w = S.make_decoder(sh, 75)
    B, L = 2, 6
    prompt = np.random.default_rng(75).integers(0, sh.vocab, (B, L)).astype(np.int32)
    dec = DEC.Decoder.from_weights(sh, DEC.upload_weights(w, "cuda"), "cuda", B, 10)
    dec.forward(torch.from_numpy(prompt).cuda())
    ref = D.Decoder(sh, w, B, 10).forward(prompt)
    assert_close(_host(dec.logits(B, sh.vocab, "cuda")), ref, "wide-query decoder logits", **DECODER_LOGITS)
