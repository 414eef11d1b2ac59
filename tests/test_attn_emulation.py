"""CPU emulation of decoder.cu's attention kernels (qkv_rope_kernel, attn_kernel<D>),
lane by lane, from the PTX fragment layouts of mma.sync.m16n8k16 (bf16 A / B, fp32 C)
and ldmatrix.x4.trans, with every shared- and global-memory index the kernels compute;
run against the oracle's RoPE and SDPA (model.cpp:560-635).  It checks the kernels'
index arithmetic -- row strides (packed q / k / v, or the fused projection's rows
qkv_ld apart), the cp.async tile fill and its zero fill past offset + L, the causal
masks, the GQA head map, the online softmax across key tiles -- without a GPU.  Global
reads are bounds-checked; cache rows past offset + L and the shared tiles' padding
columns hold NaN, so a read of either shows up in the output."""
from __future__ import annotations

import math

import numpy as np
import pytest

from oracle import decoder as D
from tests._parity import assert_close

ROWS = KEYS = 64  # kAttnRows, kAttnKeys
NAN16 = 0x7FC0


def f32(u):
    return D.f32(np.asarray(u, np.uint16))


def bf(x):
    return D.bf16(np.asarray(x, np.float32))


class Mem:
    """A flat bf16 buffer with bounds-checked element reads and writes."""

    def __init__(self, a):
        self.a = np.array(a, np.uint16).reshape(-1)

    def get(self, idx):
        idx = np.asarray(idx, np.int64)
        assert (idx >= 0).all() and (idx < self.a.size).all(), "out-of-bounds read"
        return self.a[idx]

    def put(self, idx, v):
        idx = np.asarray(idx, np.int64)
        assert (idx >= 0).all() and (idx < self.a.size).all(), "out-of-bounds write"
        self.a[idx] = v


def _fma(a, b, c):
    return (np.float64(a) * np.float64(b) + np.float64(c)).astype(np.float32)


def _head_norm(x1, x2, w, d, eps):
    """The QK-norm of one head in qkv_rope_kernel: lane l's fp32 sum of squares over its
    pairs i = l, l + 32 (fmaf chain, zeros past d/2), the xor-butterfly warp sum, then
    bf16(bf16(x * n) * w)."""
    half = d // 2
    X1, X2 = np.zeros(64, np.float32), np.zeros(64, np.float32)
    X1[:half], X2[:half] = x1, x2
    lane = np.arange(32)
    ss = np.zeros(32, np.float32)
    for j in range(2):
        ss = _fma(X1[lane + 32 * j], X1[lane + 32 * j], _fma(X2[lane + 32 * j], X2[lane + 32 * j], ss))
    for off in (16, 8, 4, 2, 1):
        ss = (ss + ss[lane ^ off]).astype(np.float32)
    assert (ss == ss[0]).all()
    n = np.float32(1) / np.sqrt(np.float32(ss[0] / np.float32(d) + np.float32(eps)))
    i = np.arange(half)
    return (f32(bf(f32(bf(x1 * n)) * f32(w[i]))), f32(bf(f32(bf(x2 * n)) * f32(w[i + half]))))


def qkv_rope(q, k, v, bias, cache_k, cache_v, B, L, offset, nh, nkv, d, max_len, q_ld, kv_ld, theta,
             norms=(None, None), eps=1e-6):
    """qkv_rope_kernel: one warp per (token, head slot), lane l holding pairs (i, i + d/2)
    for i = l, l + 32; bias, then the optional QK-norm (norms = (q_norm, k_norm)), then RoPE."""
    half = d // 2
    log2_theta = math.log2(theta)
    for t in range(B * L):
        b, l = divmod(t, L)
        pos = offset + l
        for slot in range(nh + 2 * nkv):
            if slot < nh:
                src, dst, bias_v, rot = (q, t * q_ld + slot * d), (q, t * q_ld + slot * d), bias[0][slot * d:], True
            elif slot < nh + nkv:
                kh = slot - nh
                src, bias_v, rot = (k, t * kv_ld + kh * d), bias[1][kh * d:], True
                dst = (cache_k, ((b * nkv + kh) * max_len + pos) * d)
            else:
                vh = slot - nh - nkv
                src, bias_v, rot = (v, t * kv_ld + vh * d), bias[2][vh * d:], False
                dst = (cache_v, ((b * nkv + vh) * max_len + pos) * d)
            i = np.array([lane + 32 * j for j in range(2) for lane in range(32)])
            i = i[i < half]
            x1 = f32(src[0].get(src[1] + i))
            x2 = f32(src[0].get(src[1] + i + half))
            x1 = f32(bf(x1 + f32(bias_v[i])))
            x2 = f32(bf(x2 + f32(bias_v[i + half])))
            norm = norms[0] if slot < nh else (norms[1] if slot < nh + nkv else None)
            if norm is not None:
                x1, x2 = _head_norm(x1, x2, norm, d, eps)
            if rot:
                inv = np.exp2(-(2.0 * i / d) * log2_theta).astype(np.float32)
                ang = np.float32(pos) * inv
                cs, sn = np.cos(ang).astype(np.float32), np.sin(ang).astype(np.float32)
                x1, x2 = x1 * cs - x2 * sn, x1 * sn + x2 * cs
            dst[0].put(dst[1] + i, bf(x1))
            dst[0].put(dst[1] + i + half, bf(x2))


def _a_matrix(regs, g, c):
    """The 16 x 16 A operand of m16n8k16 from the four registers of every lane:
    r0 (row g, k 2c..2c+1), r1 (row g+8), r2 (row g, k + 8), r3 (row g+8, k + 8)."""
    A = np.full((16, 16), np.nan, np.float32)
    for r, (dr, dk) in enumerate(((0, 0), (8, 0), (0, 8), (8, 8))):
        for e in range(2):
            A[g + dr, 2 * c + dk + e] = regs[r][:, e]
    assert not np.isnan(A).any()
    return A


def _b_matrix(regs, g, c):
    """The 16 x 8 B operand from r0 (k 2c..2c+1, n g) and r1 (k 2c+8.., n g)."""
    Bm = np.full((16, 8), np.nan, np.float32)
    for r, dk in enumerate((0, 8)):
        for e in range(2):
            Bm[2 * c + dk + e, g] = regs[r][:, e]
    assert not np.isnan(Bm).any()
    return Bm


def attn(q, cache_k, cache_v, out, B, L, offset, nh, nkv, Dh, max_len, q_ld, out_ld, scale):
    """attn_kernel<D> over its whole grid (query tiles x heads x batch), 4 warps per CTA."""
    DS, KS, NT = Dh + 8, Dh // 16, Dh // 8
    lane = np.arange(32)
    g, c = lane >> 2, lane & 3
    total = offset + L
    for b in range(B):
        for h in range(nh):
            kvh = h // (nh // nkv)
            kbase = (b * nkv + kvh) * max_len * Dh
            for qt in range((L + ROWS - 1) // ROWS):
                q0 = qt * ROWS
                last_row = min(q0 + ROWS, L) - 1
                nkb = (offset + last_row) // KEYS + 1
                tiles = []
                for kb in range(nkb):  # load_tile: 16-byte chunks, zero past offset + L
                    sK = np.full(KEYS * DS, 0xFFFF, np.uint16)  # padding columns: NaN
                    sV = sK.copy()
                    for r in range(KEYS):
                        key = kb * KEYS + r
                        for ch in range(0, Dh, 8):
                            dstv = r * DS + ch + np.arange(8)
                            if key < total:
                                sK[dstv] = cache_k.get(kbase + key * Dh + ch + np.arange(8))
                                sV[dstv] = cache_v.get(kbase + key * Dh + ch + np.arange(8))
                            else:
                                sK[dstv] = 0
                                sV[dstv] = 0
                    tiles.append((sK, sV))
                for warp in range(4):
                    row_g = q0 + warp * 16 + g
                    row_g8 = row_g + 8
                    pos_g, pos_g8 = offset + row_g, offset + row_g8
                    qg = (b * L + np.minimum(row_g, L - 1)) * q_ld + h * Dh
                    qg8 = (b * L + np.minimum(row_g8, L - 1)) * q_ld + h * Dh

                    def pair(mem, off):
                        return f32(mem.get(np.stack([off, off + 1], -1)))
                    QA = [_a_matrix([pair(q, qg + 16 * ks + 2 * c), pair(q, qg8 + 16 * ks + 2 * c),
                                     pair(q, qg + 16 * ks + 2 * c + 8), pair(q, qg8 + 16 * ks + 2 * c + 8)], g, c)
                          for ks in range(KS)]
                    o = np.zeros((NT, 32, 4), np.float32)
                    m_g = np.full(32, -np.inf, np.float32)
                    m_g8 = m_g.copy()
                    l_g = np.zeros(32, np.float32)
                    l_g8 = l_g.copy()
                    for kb in range(nkb):
                        sK, sV = tiles[kb]
                        s = np.zeros((8, 32, 4), np.float32)
                        for ks in range(KS):
                            for j in range(8):
                                kr = (8 * j + g) * DS + 16 * ks + 2 * c
                                Bm = _b_matrix([f32(sK[np.stack([kr, kr + 1], -1)]),
                                                f32(sK[np.stack([kr + 8, kr + 9], -1)])], g, c)
                                C = QA[ks] @ Bm  # fp32 accumulate
                                s[j, :, 0] += C[g, 2 * c]
                                s[j, :, 1] += C[g, 2 * c + 1]
                                s[j, :, 2] += C[g + 8, 2 * c]
                                s[j, :, 3] += C[g + 8, 2 * c + 1]
                        for j in range(8):
                            for e in range(2):
                                key = kb * KEYS + 8 * j + 2 * c + e
                                s[j, :, e] = np.where(key <= pos_g, s[j, :, e] * np.float32(scale), -np.inf)
                                s[j, :, 2 + e] = np.where(key <= pos_g8, s[j, :, 2 + e] * np.float32(scale), -np.inf)
                        mx_g = s[:, :, 0:2].max(axis=(0, 2))
                        mx_g8 = s[:, :, 2:4].max(axis=(0, 2))
                        mx_g = mx_g.reshape(8, 4).max(1).repeat(4)  # xor-shuffle max over the lane quad
                        mx_g8 = mx_g8.reshape(8, 4).max(1).repeat(4)
                        mn_g, mn_g8 = np.maximum(m_g, mx_g), np.maximum(m_g8, mx_g8)
                        al_g, al_g8 = np.exp(m_g - mn_g).astype(np.float32), np.exp(m_g8 - mn_g8).astype(np.float32)
                        m_g, m_g8 = mn_g, mn_g8
                        l_g, l_g8 = l_g * al_g, l_g8 * al_g8
                        o[:, :, 0:2] *= al_g[None, :, None]
                        o[:, :, 2:4] *= al_g8[None, :, None]
                        p = np.empty_like(s)
                        p[:, :, 0:2] = np.exp(s[:, :, 0:2] - mn_g[None, :, None])
                        p[:, :, 2:4] = np.exp(s[:, :, 2:4] - mn_g8[None, :, None])
                        for j in range(8):
                            l_g = l_g + (p[j, :, 0] + p[j, :, 1])
                            l_g8 = l_g8 + (p[j, :, 2] + p[j, :, 3])
                        pa = f32(bf(p))  # P rounded to bf16 as the A operand
                        for kk in range(4):
                            PA = _a_matrix([pa[2 * kk][:, 0:2], pa[2 * kk][:, 2:4], pa[2 * kk + 1][:, 0:2],
                                            pa[2 * kk + 1][:, 2:4]], g, c)
                            mi, rr = lane >> 3, lane & 7
                            vrow = (16 * kk + (mi & 1) * 8 + rr) * DS + (mi >> 1) * 8
                            for n in range(0, NT, 2):
                                addr = vrow + 8 * n
                                # ldmatrix.x4.trans: matrix m's row r is 8 values at lane 8m + r's
                                # address; lane t receives (M[2(t%4)][t/4], M[2(t%4)+1][t/4])
                                regs = []
                                for mtx in range(4):
                                    M = np.stack([sV[addr[8 * mtx + r] + np.arange(8)] for r in range(8)])
                                    regs.append(f32(np.stack([M[2 * c, g], M[2 * c + 1, g]], -1)))
                                for nn, (b0, b1) in ((n, (regs[0], regs[1])), (n + 1, (regs[2], regs[3]))):
                                    C = PA @ _b_matrix([b0, b1], g, c)
                                    o[nn, :, 0] += C[g, 2 * c]
                                    o[nn, :, 1] += C[g, 2 * c + 1]
                                    o[nn, :, 2] += C[g + 8, 2 * c]
                                    o[nn, :, 3] += C[g + 8, 2 * c + 1]
                    for off in (1, 2):  # quad sums, xor butterfly
                        l_g = l_g + l_g[lane ^ off]
                        l_g8 = l_g8 + l_g8[lane ^ off]
                    inv_g, inv_g8 = np.float32(1) / l_g, np.float32(1) / l_g8
                    for n in range(NT):
                        for e in range(2):
                            ok = row_g < L
                            out.put(((b * L + row_g) * out_ld + h * Dh + 8 * n + 2 * c + e)[ok],
                                    bf(o[n, :, e] * inv_g)[ok])
                            ok8 = row_g8 < L
                            out.put(((b * L + row_g8) * out_ld + h * Dh + 8 * n + 2 * c + e)[ok8],
                                    bf(o[n, :, 2 + e] * inv_g8)[ok8])


@pytest.mark.parametrize("B,L,offset,nh,nkv,d", [(2, 5, 0, 4, 2, 64), (1, 1, 70, 2, 1, 128), (1, 70, 3, 2, 2, 64),
                                                 (2, 3, 62, 4, 1, 64)])
@pytest.mark.parametrize("fused", [False, True])
def test_attention_kernels_against_oracle(B, L, offset, nh, nkv, d, fused):
    rng = np.random.default_rng(B * 1000 + L * 10 + offset)
    theta, max_len = 1e6, offset + L + 3
    T, QD, KVD = B * L, nh * d, nkv * d
    qn = bf(rng.standard_normal((T, QD)))
    kn, vn = bf(rng.standard_normal((T, KVD))), bf(rng.standard_normal((T, KVD)))
    bias = [bf(0.02 * rng.standard_normal(n)) for n in (QD, KVD, KVD)]
    ck = np.full((B, nkv, max_len, d), NAN16, np.uint16)  # rows past offset + L: never read
    ck[:, :, :offset] = bf(rng.standard_normal((B, nkv, offset, d)))
    cv = ck.copy()
    cv[:, :, :offset] = bf(rng.standard_normal((B, nkv, offset, d)))
    if fused:  # one [T, QD + 2 KVD] buffer, rows qkv_ld apart (fm_attn_config.qkv_ld)
        W = QD + 2 * KVD
        buf = Mem(np.concatenate([qn, kn, vn], axis=1))
        q = k = v = buf
        qo, ko, vo, q_ld, kv_ld = 0, QD, QD + KVD, W, W
    else:
        q, k, v = Mem(qn), Mem(kn), Mem(vn)
        qo = ko = vo = 0
        q_ld, kv_ld = QD, KVD

    class At:  # a view of a buffer from an element offset (the kernels' base pointers)
        def __init__(self, mem, base):
            self.mem, self.base = mem, base

        def get(self, idx):
            return self.mem.get(np.asarray(idx) + self.base)

        def put(self, idx, val):
            self.mem.put(np.asarray(idx) + self.base, val)
    cache_k, cache_v = Mem(ck), Mem(cv)
    qkv_rope(At(q, qo), At(k, ko), At(v, vo), bias, cache_k, cache_v, B, L, offset, nh, nkv, d, max_len, q_ld,
             kv_ld, theta)
    out = Mem(np.zeros((T, QD), np.uint16))
    attn(At(q, qo), cache_k, cache_v, out, B, L, offset, nh, nkv, d, max_len, q_ld, QD, 1.0 / math.sqrt(d))

    pos = offset + np.tile(np.arange(L), B)
    q_ref = D.rope(D.add(qn, bias[0][None]), pos, nh, d, theta)
    k_ref = D.rope(D.add(kn, bias[1][None]), pos, nkv, d, theta)
    v_ref = D.add(vn, bias[2][None])
    ck_ref, cv_ref = ck.copy(), cv.copy()
    ck_ref[:, :, offset:offset + L] = k_ref.reshape(B, L, nkv, d).transpose(0, 2, 1, 3)
    cv_ref[:, :, offset:offset + L] = v_ref.reshape(B, L, nkv, d).transpose(0, 2, 1, 3)
    q_got = q.a.reshape(T, -1)[:, :QD]
    assert_close(q_got, q_ref, "rope q", max_rel=1e-2, mae_rel=1e-4)
    got_ck, got_cv = cache_k.a.reshape(ck.shape), cache_v.a.reshape(cv.shape)
    np.testing.assert_array_equal(got_cv[:, :, :offset + L], cv_ref[:, :, :offset + L])
    np.testing.assert_array_equal(got_ck[:, :, :offset], ck_ref[:, :, :offset])
    assert (got_ck[:, :, offset + L:] == NAN16).all() and (got_cv[:, :, offset + L:] == NAN16).all()
    assert_close(got_ck[:, :, offset:offset + L], ck_ref[:, :, offset:offset + L], "rope k", max_rel=1e-2,
                 mae_rel=1e-4)
    if fused:  # k and v columns of the fused rows are only read
        np.testing.assert_array_equal(q.a.reshape(T, -1)[:, QD:], np.concatenate([kn, vn], axis=1))
    ref = D.sdpa(q_ref, ck_ref, cv_ref, B, L, offset, nh, nkv, d)
    assert_close(out.a.reshape(T, QD), ref, f"sdpa B={B} L={L} offset={offset}", max_rel=2e-2, mae_rel=5e-3)


@pytest.mark.parametrize("d", [64, 128])
@pytest.mark.parametrize("fused", [False, True])
def test_qk_norm_lanes_against_oracle(d, fused):
    """Qwen3's QK-norm inside qkv_rope_kernel (model.cpp:573-581), lane by lane, against
    the oracle's rms_norm of each q / k head followed by RoPE."""
    rng = np.random.default_rng(90 + d)
    B, L, offset, nh, nkv, theta, eps = 2, 3, 4, 4, 2, 1e6, 1e-6
    max_len, T, QD, KVD = offset + L, B * L, nh * d, nkv * d
    qn = bf(3 * rng.standard_normal((T, QD)))
    kn, vn = bf(3 * rng.standard_normal((T, KVD))), bf(rng.standard_normal((T, KVD)))
    wq, wk = bf(1 + 0.1 * rng.standard_normal(d)), bf(1 + 0.1 * rng.standard_normal(d))
    zero = [np.zeros(n, np.uint16) for n in (QD, KVD, KVD)]
    ck = np.zeros((B, nkv, max_len, d), np.uint16)
    cv = ck.copy()
    if fused:
        buf = Mem(np.concatenate([qn, kn, vn], axis=1))
        views, q_ld, kv_ld = ((buf, 0), (buf, QD), (buf, QD + KVD)), QD + 2 * KVD, QD + 2 * KVD
    else:
        views, q_ld, kv_ld = ((Mem(qn), 0), (Mem(kn), 0), (Mem(vn), 0)), QD, KVD

    class At:
        def __init__(self, mem, base):
            self.mem, self.base = mem, base

        def get(self, idx):
            return self.mem.get(np.asarray(idx) + self.base)

        def put(self, idx, val):
            self.mem.put(np.asarray(idx) + self.base, val)
    cache_k, cache_v = Mem(ck), Mem(cv)
    qv = At(*views[0])
    qkv_rope(qv, At(*views[1]), At(*views[2]), zero, cache_k, cache_v, B, L, offset, nh, nkv, d, max_len, q_ld,
             kv_ld, theta, norms=(wq, wk), eps=eps)
    pos = offset + np.tile(np.arange(L), B)
    q_ref = D.rope(D.rms_norm(qn.reshape(T, nh, d), wq, eps).reshape(T, -1), pos, nh, d, theta)
    k_ref = D.rope(D.rms_norm(kn.reshape(T, nkv, d), wk, eps).reshape(T, -1), pos, nkv, d, theta)
    q_got = views[0][0].a.reshape(T, -1)[:, :QD]
    assert_close(q_got, q_ref, "qk-norm q", max_rel=1e-2, mae_rel=1e-4)
    got_k = cache_k.a.reshape(ck.shape)[:, :, offset:].transpose(0, 2, 1, 3).reshape(T, KVD)
    assert_close(got_k, k_ref, "qk-norm k", max_rel=1e-2, mae_rel=1e-4)
    got_v = cache_v.a.reshape(cv.shape)[:, :, offset:].transpose(0, 2, 1, 3).reshape(T, KVD)
    np.testing.assert_array_equal(got_v, vn)  # v: no norm, no rotation
