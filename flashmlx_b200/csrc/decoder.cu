// decoder.cu -- the non-MoE ops of the reference's decoder forward (LlamaModel, Qwen form),
// so a whole decoder layer runs on libflashmoe: embedding lookup, residual add + RMSNorm,
// q/k/v bias + RoPE + KV-cache write, causal flash attention over the bf16 cache, SwiGLU
// for dense MLP layers, greedy argmax.
//
// Reference ops (server/src/model.cpp) and the arithmetic kept from them:
//   dequantize_kernel   mx::dequantize of the embedding at load (216-230): bf16(fma(s, q, b))
//   embed_kernel        mx::take(table, ids, 0) (490-496): row copies
//   add_rms_norm_kernel mx::add (824, 838) + mx::fast::rms_norm (486-488): h = bf16(x + r),
//                       n = 1 / sqrt(mean_fp32(h^2) + eps), y = bf16(bf16(h * n) * w)
//   qkv_rope_kernel     bias adds (560-566), the optional QK-norm (mx::fast::rms_norm of each
//                       q / k head, 573-581), mx::fast::rope(traditional=false, base, scale 1,
//                       offset) (588-589), mx::slice_update of the cache (608-617): pairs
//                       (i, i + d/2) rotated in fp32 by theta = fp32(pos) * inv_freq_i,
//                       inv_freq_i = base^(-2i/d) evaluated in fp64 and rounded once
//   attn_kernel         mx::fast::scaled_dot_product_attention (622-635), causal for L > 1:
//                       fp32 scores x scale, online fp32 softmax, probabilities rounded to
//                       bf16 for the P.V tensor-core product, fp32 sums, bf16 out
//   swiglu_kernel       the compiled swiglu (14-25): bf16 rounding after every op
//   argmax_kernel       greedy sampling: the first index of the largest bf16 logit
//
// Layouts: activations token-major [T, n * d] (T = B * L, token t = b * L + l); the KV
// cache [B, n_kv, max_len, d] bf16 as the reference allocates it.  Attention runs on the
// legacy mma.sync bf16 path (m16n8k16) with cp.async-staged, double-buffered K / V tiles:
// at these sizes (d = 128, <= 768 positions) it is a small share of the layer next to
// the MoE block.
#include <algorithm>

#include "fm_internal.cuh"

namespace fm {

namespace {

FM_DEV uint32_t lds32(const uint16_t* p) { return *reinterpret_cast<const uint32_t*>(p); }

FM_DEV void ldsm_x4_trans(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

FM_DEV float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

}  // namespace

// ------------------------------------------------------------------ dequantize / embed
// out [N, K] = bf16(fma(s, q, b)); one thread per packed word (8 codes -> 16 bytes out).
__global__ void dequant_kernel(const uint32_t* __restrict__ w, const uint16_t* __restrict__ s,
                               const uint16_t* __restrict__ b, int64_t N, int K, int gs, uint16_t* __restrict__ out) {
  const int kw = K / 8, gpr = K / gs;
  const int64_t total = N * kw;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t n = i / kw;
    const int j = static_cast<int>(i - n * kw);
    const uint32_t word = w[i];
    const int64_t gi = n * gpr + (8 * j) / gs;
    const float sc = bf2f(s[gi]), bi = b ? bf2f(b[gi]) : 0.f;
    float v[8];
#pragma unroll
    for (int p = 0; p < 8; ++p) v[p] = fmaf(sc, static_cast<float>((word >> (4 * p)) & 15u), bi);
    uint4 o;
    o.x = pack_bf16x2(v[0], v[1]);
    o.y = pack_bf16x2(v[2], v[3]);
    o.z = pack_bf16x2(v[4], v[5]);
    o.w = pack_bf16x2(v[6], v[7]);
    *reinterpret_cast<uint4*>(out + n * K + 8 * j) = o;
  }
}

// y[t] = table[ids[t]] (16-byte copies); an id outside [0, V) gives a zero row and sets
// DEVERR_BOUNDS
__global__ void embed_kernel(const uint16_t* __restrict__ table, int64_t V, int H, const int32_t* __restrict__ ids,
                             int64_t T, uint16_t* __restrict__ y, uint32_t* err) {
  const int segs = H / 8;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < T * segs;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t t = i / segs;
    const int col = static_cast<int>(i - t * segs) * 8;
    const int64_t id = ids[t];
    uint4 v = make_uint4(0, 0, 0, 0);
    if (id >= 0 && id < V) {
      v = *reinterpret_cast<const uint4*>(table + id * H + col);
    } else if (col == 0) {
      report(err, DEVERR_BOUNDS);
    }
    *reinterpret_cast<uint4*>(y + t * H + col) = v;
  }
}

// ------------------------------------------------------------------ add + rms_norm
// One CTA per row.  Pass 1: h = bf16(x + r) (or x), written to h_out when given, and the
// fp32 sum of h^2; pass 2 re-reads h (h_out, or x / x + r again) chunk by chunk in the
// same thread order, so h_out may alias x.
constexpr int kNormThreads = 256;

__global__ void __launch_bounds__(kNormThreads) add_rms_norm_kernel(const uint16_t* x, const uint16_t* r,
                                                                   const uint16_t* __restrict__ w, int H, float eps,
                                                                   uint16_t* h_out, uint16_t* __restrict__ y) {
  const int64_t row = blockIdx.x;
  const uint16_t* xr = x + row * H;
  const uint16_t* rr = r ? r + row * H : nullptr;
  uint16_t* hr = h_out ? h_out + row * H : nullptr;
  float ss = 0.f;
  for (int c = threadIdx.x * 8; c < H; c += kNormThreads * 8) {
    uint4 xv = *reinterpret_cast<const uint4*>(xr + c);
    uint32_t hv[4] = {xv.x, xv.y, xv.z, xv.w};
    if (rr) {
      const uint4 rv = *reinterpret_cast<const uint4*>(rr + c);
      const uint32_t ra[4] = {rv.x, rv.y, rv.z, rv.w};
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float lo = bf2f(static_cast<uint16_t>(hv[q] & 0xffffu)) + bf2f(static_cast<uint16_t>(ra[q] & 0xffffu));
        const float hi = bf2f(static_cast<uint16_t>(hv[q] >> 16)) + bf2f(static_cast<uint16_t>(ra[q] >> 16));
        hv[q] = pack_bf16x2(lo, hi);
      }
      if (hr) *reinterpret_cast<uint4*>(hr + c) = make_uint4(hv[0], hv[1], hv[2], hv[3]);
    } else if (hr && hr != xr) {
      *reinterpret_cast<uint4*>(hr + c) = xv;
    }
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const float lo = bf2f(static_cast<uint16_t>(hv[q] & 0xffffu)), hi = bf2f(static_cast<uint16_t>(hv[q] >> 16));
      ss = fmaf(lo, lo, ss);
      ss = fmaf(hi, hi, ss);
    }
  }
  __shared__ float red[kNormThreads / 32];
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  float tot = 0.f;
#pragma unroll
  for (int i = 0; i < kNormThreads / 32; ++i) tot += red[i];
  const float n = 1.0f / sqrtf(tot / static_cast<float>(H) + eps);
  for (int c = threadIdx.x * 8; c < H; c += kNormThreads * 8) {
    uint32_t hv[4];
    if (hr) {
      const uint4 v = *reinterpret_cast<const uint4*>(hr + c);
      hv[0] = v.x; hv[1] = v.y; hv[2] = v.z; hv[3] = v.w;
    } else {
      const uint4 v = *reinterpret_cast<const uint4*>(xr + c);
      hv[0] = v.x; hv[1] = v.y; hv[2] = v.z; hv[3] = v.w;
      if (rr) {
        const uint4 rv = *reinterpret_cast<const uint4*>(rr + c);
        const uint32_t ra[4] = {rv.x, rv.y, rv.z, rv.w};
#pragma unroll
        for (int q = 0; q < 4; ++q)
          hv[q] = pack_bf16x2(bf2f(static_cast<uint16_t>(hv[q] & 0xffffu)) + bf2f(static_cast<uint16_t>(ra[q] & 0xffffu)),
                              bf2f(static_cast<uint16_t>(hv[q] >> 16)) + bf2f(static_cast<uint16_t>(ra[q] >> 16)));
      }
    }
    const uint4 wv = *reinterpret_cast<const uint4*>(w + c);
    const uint32_t wa[4] = {wv.x, wv.y, wv.z, wv.w};
    uint32_t o[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const float lo = rbf(bf2f(static_cast<uint16_t>(hv[q] & 0xffffu)) * n) * bf2f(static_cast<uint16_t>(wa[q] & 0xffffu));
      const float hi = rbf(bf2f(static_cast<uint16_t>(hv[q] >> 16)) * n) * bf2f(static_cast<uint16_t>(wa[q] >> 16));
      o[q] = pack_bf16x2(lo, hi);
    }
    *reinterpret_cast<uint4*>(y + row * H + c) = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

// ------------------------------------------------------------------ q/k/v bias + rope + cache
// One warp per (token, head slot): slots [0, nh) rotate q in place, [nh, nh + nkv) rotate
// k into cache_k, [nh + nkv, nh + 2 nkv) copy v into cache_v; the bias is added first
// (bf16 add, model.cpp:560-566), then the head's RMSNorm when a QK-norm weight is given
// (fp32 sum of squares over the head, bf16(bf16(x * n) * w)).  Lane l holds the pairs
// (i, i + d/2) for i = l and l + 32 (d <= 128).
__global__ void qkv_rope_kernel(const AttnArgs a) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int slots = a.nh + 2 * a.nkv;
  const int64_t item = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + warp;
  if (item >= static_cast<int64_t>(a.B) * a.L * slots) return;
  const int64_t t = item / slots;
  const int slot = static_cast<int>(item - t * slots);
  const int b = static_cast<int>(t / a.L), l = static_cast<int>(t - static_cast<int64_t>(b) * a.L);
  const int pos = a.offset + l;
  const int d = a.head_dim, half = d / 2;
  const uint16_t* src;
  const uint16_t* bias;
  const uint16_t* norm = nullptr;
  uint16_t* dst;
  bool rot = true;
  if (slot < a.nh) {
    src = a.q + t * a.q_ld + slot * d;
    bias = a.q_bias ? a.q_bias + slot * d : nullptr;
    norm = a.q_norm;
    dst = a.q + t * a.q_ld + slot * d;
  } else if (slot < a.nh + a.nkv) {
    const int kh = slot - a.nh;
    src = a.k + t * a.kv_ld + kh * d;
    bias = a.k_bias ? a.k_bias + kh * d : nullptr;
    norm = a.k_norm;
    dst = a.cache_k + ((static_cast<int64_t>(b) * a.nkv + kh) * a.max_len + pos) * d;
  } else {
    const int vh = slot - a.nh - a.nkv;
    src = a.v + t * a.kv_ld + vh * d;
    bias = a.v_bias ? a.v_bias + vh * d : nullptr;
    dst = a.cache_v + ((static_cast<int64_t>(b) * a.nkv + vh) * a.max_len + pos) * d;
    rot = false;
  }
  // the lane's pairs (i, i + d/2), i = lane + 32 j < d/2, bias added
  float x1[2] = {0.f, 0.f}, x2[2] = {0.f, 0.f};
#pragma unroll
  for (int j = 0; j < 2; ++j) {
    const int i = lane + 32 * j;
    if (i < half) {
      x1[j] = bf2f(src[i]);
      x2[j] = bf2f(src[i + half]);
      if (bias) {
        x1[j] = rbf(x1[j] + bf2f(bias[i]));
        x2[j] = rbf(x2[j] + bf2f(bias[i + half]));
      }
    }
  }
  if (norm) {  // QK-norm over the head's d values (lanes past d/2 hold zeros); norm is warp-uniform
    float ss = 0.f;
#pragma unroll
    for (int j = 0; j < 2; ++j) ss = fmaf(x1[j], x1[j], fmaf(x2[j], x2[j], ss));
    ss = warp_sum(ss);
    const float n = 1.0f / sqrtf(ss / static_cast<float>(d) + a.norm_eps);
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const int i = lane + 32 * j;
      if (i < half) {
        x1[j] = rbf(rbf(x1[j] * n) * bf2f(norm[i]));
        x2[j] = rbf(rbf(x2[j] * n) * bf2f(norm[i + half]));
      }
    }
  }
#pragma unroll
  for (int j = 0; j < 2; ++j) {
    const int i = lane + 32 * j;
    if (i >= half) continue;
    float o1 = x1[j], o2 = x2[j];
    if (rot) {
      const float inv = static_cast<float>(exp2(-(2.0 * i / d) * a.log2_theta));
      const float ang = static_cast<float>(pos) * inv;
      const float cs = cosf(ang), sn = sinf(ang);
      o1 = x1[j] * cs - x2[j] * sn;
      o2 = x1[j] * sn + x2[j] * cs;
    }
    dst[i] = f2bf(o1);
    dst[i + half] = f2bf(o2);
  }
}

// ------------------------------------------------------------------ causal flash attention
// CTA = 4 warps = 64 query rows of one (batch, head); warp w owns rows 16 w .. 16 w + 15.
// K / V tiles of 64 positions x D are staged by cp.async into a double buffer (row stride
// D + 8 bf16: conflict-free 4-byte reads of K and ldmatrix.trans of V); positions at or
// past offset + L are zero-filled and masked.  S = Q K^T on m16n8k16 (Q fragments held in
// registers), online softmax in fp32 (rows' max and sum reduced over the lane quad), P
// rounded to bf16 as the A operand of O += P V.
constexpr int kAttnRows = 64;
constexpr int kAttnKeys = 64;

template <int D>
constexpr int attn_smem_bytes() {
  return 2 * 2 * kAttnKeys * (D + 8) * 2;
}

template <int D>
__global__ void __launch_bounds__(128) attn_kernel(const AttnArgs a) {
  constexpr int DS = D + 8;        // smem row stride (bf16)
  constexpr int KS = D / 16;       // k-steps of S = Q K^T
  constexpr int NT = D / 8;        // n-tiles of O
  extern __shared__ __align__(16) uint16_t smem[];
  uint16_t* sK = smem;                          // [2][64][DS]
  uint16_t* sV = smem + 2 * kAttnKeys * DS;     // [2][64][DS]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, c = lane & 3;
  const int qt = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int kvh = h / (a.nh / a.nkv);
  const int total = a.offset + a.L;
  const int q0 = qt * kAttnRows;
  const int row_g = q0 + warp * 16 + g, row_g8 = row_g + 8;  // query rows (may pass L)
  const int pos_g = a.offset + row_g, pos_g8 = a.offset + row_g8;
  const int last_row = min(q0 + kAttnRows, a.L) - 1;
  const int nkb = (a.offset + last_row) / kAttnKeys + 1;  // key blocks any row of the tile sees
  const uint16_t* kbase = a.cache_k + (static_cast<int64_t>(b) * a.nkv + kvh) * a.max_len * D;
  const uint16_t* vbase = a.cache_v + (static_cast<int64_t>(b) * a.nkv + kvh) * a.max_len * D;

  auto load_tile = [&](int kb, int buf) {
    uint16_t* dk = sK + buf * kAttnKeys * DS;
    uint16_t* dv = sV + buf * kAttnKeys * DS;
    constexpr int CPR = D / 8;  // 16-byte chunks per row
    for (int i = threadIdx.x; i < kAttnKeys * CPR; i += blockDim.x) {
      const int r = i / CPR, ch = (i - r * CPR) * 8;
      const int key = kb * kAttnKeys + r;
      if (key < total) {
        cp_async16(smem_u32(dk + r * DS + ch), kbase + static_cast<int64_t>(key) * D + ch);
        cp_async16(smem_u32(dv + r * DS + ch), vbase + static_cast<int64_t>(key) * D + ch);
      } else {
        *reinterpret_cast<uint4*>(dk + r * DS + ch) = make_uint4(0, 0, 0, 0);
        *reinterpret_cast<uint4*>(dv + r * DS + ch) = make_uint4(0, 0, 0, 0);
      }
    }
    cp_async_commit();
  };
  load_tile(0, 0);

  // Q fragments: rows g, g + 8 of the warp's 16, clamped to the last valid row
  uint32_t qa[KS][4];
  {
    const int64_t tg = static_cast<int64_t>(b) * a.L + min(row_g, a.L - 1);
    const int64_t tg8 = static_cast<int64_t>(b) * a.L + min(row_g8, a.L - 1);
    const uint16_t* qg = a.q + tg * a.q_ld + h * D;
    const uint16_t* qg8 = a.q + tg8 * a.q_ld + h * D;
#pragma unroll
    for (int ks = 0; ks < KS; ++ks) {
      qa[ks][0] = *reinterpret_cast<const uint32_t*>(qg + 16 * ks + 2 * c);
      qa[ks][1] = *reinterpret_cast<const uint32_t*>(qg8 + 16 * ks + 2 * c);
      qa[ks][2] = *reinterpret_cast<const uint32_t*>(qg + 16 * ks + 2 * c + 8);
      qa[ks][3] = *reinterpret_cast<const uint32_t*>(qg8 + 16 * ks + 2 * c + 8);
    }
  }
  float o[NT][4];
#pragma unroll
  for (int n = 0; n < NT; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
  float m_g = -INFINITY, m_g8 = -INFINITY, l_g = 0.f, l_g8 = 0.f;

  for (int kb = 0; kb < nkb; ++kb) {
    if (kb + 1 < nkb) {
      load_tile(kb + 1, (kb + 1) & 1);
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    const uint16_t* tk = sK + (kb & 1) * kAttnKeys * DS;
    const uint16_t* tv = sV + (kb & 1) * kAttnKeys * DS;
    float s[8][4];
#pragma unroll
    for (int j = 0; j < 8; ++j) s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.f;
#pragma unroll
    for (int ks = 0; ks < KS; ++ks)
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const uint16_t* kr = tk + (8 * j + g) * DS + 16 * ks + 2 * c;
        mma_bf16_16816(s[j], qa[ks][0], qa[ks][1], qa[ks][2], qa[ks][3], lds32(kr), lds32(kr + 8));
      }
    // scale, causal mask (key > query position), tile max per row
    float mx_g = -INFINITY, mx_g8 = -INFINITY;
#pragma unroll
    for (int j = 0; j < 8; ++j)
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int key = kb * kAttnKeys + 8 * j + 2 * c + e;
        s[j][e] = key <= pos_g ? s[j][e] * a.scale : -INFINITY;
        s[j][2 + e] = key <= pos_g8 ? s[j][2 + e] * a.scale : -INFINITY;
        mx_g = fmaxf(mx_g, s[j][e]);
        mx_g8 = fmaxf(mx_g8, s[j][2 + e]);
      }
#pragma unroll
    for (int off = 1; off < 4; off <<= 1) {
      mx_g = fmaxf(mx_g, __shfl_xor_sync(0xffffffffu, mx_g, off));
      mx_g8 = fmaxf(mx_g8, __shfl_xor_sync(0xffffffffu, mx_g8, off));
    }
    const float mn_g = fmaxf(m_g, mx_g), mn_g8 = fmaxf(m_g8, mx_g8);
    // block 0 holds key 0 <= every row's position, so mn_* is finite from the first block on
    const float al_g = expf(m_g - mn_g), al_g8 = expf(m_g8 - mn_g8);  // exp(-inf) = 0 on the first block
    m_g = mn_g;
    m_g8 = mn_g8;
    l_g *= al_g;
    l_g8 *= al_g8;
#pragma unroll
    for (int n = 0; n < NT; ++n) {
      o[n][0] *= al_g;
      o[n][1] *= al_g;
      o[n][2] *= al_g8;
      o[n][3] *= al_g8;
    }
    uint32_t pa[8][2];  // P of n-tile j as bf16 pairs: [j][0] row g, [j][1] row g + 8
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float p0 = expf(s[j][0] - mn_g), p1 = expf(s[j][1] - mn_g);
      const float p2 = expf(s[j][2] - mn_g8), p3 = expf(s[j][3] - mn_g8);
      l_g += p0 + p1;
      l_g8 += p2 + p3;
      pa[j][0] = pack_bf16x2(p0, p1);
      pa[j][1] = pack_bf16x2(p2, p3);
    }
    // O += P V: k-step kk covers keys 16 kk .. 16 kk + 15 (n-tiles 2 kk, 2 kk + 1 of S)
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      const int mi = lane >> 3, rr = lane & 7;
      const uint16_t* vrow = tv + (16 * kk + (mi & 1) * 8 + rr) * DS + (mi >> 1) * 8;
#pragma unroll
      for (int n = 0; n < NT; n += 2) {
        uint32_t b0, b1, b2, b3;
        ldsm_x4_trans(smem_u32(vrow + 8 * n), b0, b1, b2, b3);
        mma_bf16_16816(o[n], pa[2 * kk][0], pa[2 * kk][1], pa[2 * kk + 1][0], pa[2 * kk + 1][1], b0, b1);
        mma_bf16_16816(o[n + 1], pa[2 * kk][0], pa[2 * kk][1], pa[2 * kk + 1][0], pa[2 * kk + 1][1], b2, b3);
      }
    }
    __syncthreads();  // the next iteration's prefetch overwrites this buffer
  }
#pragma unroll
  for (int off = 1; off < 4; off <<= 1) {
    l_g += __shfl_xor_sync(0xffffffffu, l_g, off);
    l_g8 += __shfl_xor_sync(0xffffffffu, l_g8, off);
  }
  const float inv_g = 1.0f / l_g, inv_g8 = 1.0f / l_g8;
  if (row_g < a.L) {
    uint16_t* og = a.out + (static_cast<int64_t>(b) * a.L + row_g) * a.out_ld + h * D;
#pragma unroll
    for (int n = 0; n < NT; ++n)
      *reinterpret_cast<uint32_t*>(og + 8 * n + 2 * c) = pack_bf16x2(o[n][0] * inv_g, o[n][1] * inv_g);
  }
  if (row_g8 < a.L) {
    uint16_t* og = a.out + (static_cast<int64_t>(b) * a.L + row_g8) * a.out_ld + h * D;
#pragma unroll
    for (int n = 0; n < NT; ++n)
      *reinterpret_cast<uint32_t*>(og + 8 * n + 2 * c) = pack_bf16x2(o[n][2] * inv_g8, o[n][3] * inv_g8);
  }
}

// ------------------------------------------------------------------ swiglu / argmax
// out may alias gate or up (each element is read before it is written, by one thread)
__global__ void swiglu_kernel(const uint16_t* gate, const uint16_t* up, int64_t n, uint16_t* out) {
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const float g = bf2f(gate[i]), u = bf2f(up[i]);
    const float gs = rbf(sigmoid_f(g));
    out[i] = f2bf(rbf(g * gs) * u);
  }
}

constexpr int kArgmaxThreads = 512;

// one CTA per row; ties go to the lower index (strict > keeps the first seen in each
// thread's ascending scan, and the reduction prefers the lower index on equal values)
__global__ void __launch_bounds__(kArgmaxThreads) argmax_kernel(const uint16_t* __restrict__ logits, int64_t V,
                                                               int32_t* __restrict__ ids) {
  const uint16_t* row = logits + static_cast<int64_t>(blockIdx.x) * V;
  float best = -INFINITY;
  int64_t bi = V;  // "none yet" sorts after every real index
  for (int64_t i = threadIdx.x; i < V; i += kArgmaxThreads) {
    const float v = bf2f(row[i]);
    if (v > best || (bi == V && v == best)) {
      best = v;
      bi = i;
    }
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, best, off);
    const int64_t oi = __shfl_xor_sync(0xffffffffu, bi, off);
    if (ov > best || (ov == best && oi < bi)) {
      best = ov;
      bi = oi;
    }
  }
  __shared__ float sv[kArgmaxThreads / 32];
  __shared__ int64_t si[kArgmaxThreads / 32];
  if ((threadIdx.x & 31) == 0) {
    sv[threadIdx.x >> 5] = best;
    si[threadIdx.x >> 5] = bi;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < kArgmaxThreads / 32; ++w)
      if (sv[w] > best || (sv[w] == best && si[w] < bi)) {
        best = sv[w];
        bi = si[w];
      }
    ids[blockIdx.x] = bi < V ? static_cast<int32_t>(bi) : 0;  // a row of NaNs picks 0
  }
}

// ------------------------------------------------------------------ launchers
cudaError_t launch_dequant(const uint32_t* w, const uint16_t* s, const uint16_t* b, int64_t N, int K, int gs,
                           uint16_t* out, int num_sms, cudaStream_t st) {
  const int64_t total = N * (K / 8);
  const int grid = static_cast<int>(std::min<int64_t>((total + 255) / 256, static_cast<int64_t>(num_sms) * 16));
  dequant_kernel<<<std::max(grid, 1), 256, 0, st>>>(w, s, b, N, K, gs, out);
  return cudaGetLastError();
}

cudaError_t launch_embed(const uint16_t* table, int64_t V, int H, const int32_t* ids, int64_t T, uint16_t* y,
                         uint32_t* err, int num_sms, cudaStream_t st) {
  const int64_t total = T * (H / 8);
  const int grid = static_cast<int>(std::min<int64_t>((total + 255) / 256, static_cast<int64_t>(num_sms) * 8));
  embed_kernel<<<std::max(grid, 1), 256, 0, st>>>(table, V, H, ids, T, y, err);
  return cudaGetLastError();
}

cudaError_t launch_rms_norm(const uint16_t* x, const uint16_t* r, const uint16_t* w, int64_t T, int H, float eps,
                            uint16_t* h_out, uint16_t* y, cudaStream_t st) {
  add_rms_norm_kernel<<<static_cast<unsigned>(T), kNormThreads, 0, st>>>(x, r, w, H, eps, h_out, y);
  return cudaGetLastError();
}

cudaError_t attn_init() {
  cudaError_t e = cudaFuncSetAttribute(attn_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       attn_smem_bytes<128>());
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(attn_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize, attn_smem_bytes<64>());
  return e;
}

cudaError_t launch_attention(const AttnArgs& a, cudaStream_t st) {
  const int64_t items = static_cast<int64_t>(a.B) * a.L * (a.nh + 2 * a.nkv);
  qkv_rope_kernel<<<static_cast<unsigned>((items + 3) / 4), 128, 0, st>>>(a);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  const dim3 grid((a.L + kAttnRows - 1) / kAttnRows, a.nh, a.B);
  if (a.head_dim == 128)
    attn_kernel<128><<<grid, 128, attn_smem_bytes<128>(), st>>>(a);
  else
    attn_kernel<64><<<grid, 128, attn_smem_bytes<64>(), st>>>(a);
  return cudaGetLastError();
}

cudaError_t launch_swiglu(const uint16_t* gate, const uint16_t* up, int64_t n, uint16_t* out, int num_sms,
                          cudaStream_t st) {
  const int grid = static_cast<int>(std::min<int64_t>((n + 255) / 256, static_cast<int64_t>(num_sms) * 8));
  swiglu_kernel<<<std::max(grid, 1), 256, 0, st>>>(gate, up, n, out);
  return cudaGetLastError();
}

cudaError_t launch_argmax(const uint16_t* logits, int64_t T, int64_t V, int32_t* ids, cudaStream_t st) {
  argmax_kernel<<<static_cast<unsigned>(T), kArgmaxThreads, 0, st>>>(logits, V, ids);
  return cudaGetLastError();
}

}  // namespace fm
