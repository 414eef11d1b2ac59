// route.cu -- router, top-k, token/expert sort and tile planning in one cooperative kernel.
//
// Replaces the MLX op chain of LlamaModel::moe_block / switch_mlp up to the first
// gather_qmm (model.cpp:757-775 and 682-700):
//   matmul(x, Wr^T) -> softmax(precise) -> argpartition top-k -> take_along_axis
//   -> argsort(flat ids) (stable) -> take(x, order / k)
// and, in "given" mode, the index bookkeeping of a bare gather_qmm / quantized_matmul.
//
// Phases (grid barriers between them, every wait bounded):
//   1  router partial logits (mma.sync over 16-token x 8-expert tiles, K split across
//      warps), the pair-permuted copy x_perm of x, zeroing of the fp32 accumulators
//   2  per token: bf16 logits, softmax, top-k (ties -> lower id), renorm, shared gate;
//      per 16-token chunk: expert bitmasks -> chunk counts and stable in-chunk ranks
//   3  per expert: exclusive scan of the chunk counts (stable order across chunks)
//   4  expert offsets, tile tables for the expert-product kernels, scatter of the
//      pairs into expert-major order
#include "fm_ep.cuh"

namespace fm {

namespace {

// within-8 pair permutation of one 16-byte chunk: [e0..e7] -> [e0,e4,e1,e5,e2,e6,e3,e7]
FM_DEV uint4 perm_chunk(uint4 v) {
  uint4 o;
  o.x = __byte_perm(v.x, v.z, 0x5410);
  o.y = __byte_perm(v.x, v.z, 0x7632);
  o.z = __byte_perm(v.y, v.w, 0x5410);
  o.w = __byte_perm(v.y, v.w, 0x7632);
  return o;
}

FM_DEV uint4 ldg_v4(const void* p) { return __ldg(reinterpret_cast<const uint4*>(p)); }

FM_DEV float warp_sum_bfly(float v) {
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
  return v;
}

FM_DEV float warp_max(float v) {
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, off));
  return v;
}

// exclusive scan of n ints in shared memory by the whole block; returns the total
__device__ int block_exclusive_scan(int* a, int n, int* s_tmp /* >= 33 ints */) {
  const int tid = threadIdx.x, nt = blockDim.x;
  const int per = (n + nt - 1) / nt;
  const int lo = min(n, tid * per), hi = min(n, lo + per);
  int local = 0;
  for (int i = lo; i < hi; ++i) local += a[i];
  // inclusive warp scan
  const int lane = tid & 31, warp = tid >> 5;
  int v = local;
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    int u = __shfl_up_sync(0xffffffffu, v, off);
    if (lane >= off) v += u;
  }
  if (lane == 31) s_tmp[warp] = v;
  __syncthreads();
  if (warp == 0) {
    const int nw = nt >> 5;
    int w = (lane < nw) ? s_tmp[lane] : 0;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      int u = __shfl_up_sync(0xffffffffu, w, off);
      if (lane >= off) w += u;
    }
    if (lane < nw) s_tmp[lane] = w;  // inclusive per warp
    if (lane == nw - 1) s_tmp[32] = w;
  }
  __syncthreads();
  int run = v - local + (warp > 0 ? s_tmp[warp - 1] : 0);
  for (int i = lo; i < hi; ++i) {
    const int x = a[i];
    a[i] = run;
    run += x;
  }
  const int total = s_tmp[32];
  __syncthreads();
  return total;
}

struct RouteSmem {
  uint32_t mask[kMaxExperts];  // token bitmask of the current chunk, per expert
  int ids[kRouteChunk * 16];   // expert ids of the current chunk's pairs (-1: dropped)
  int offs[kMaxExperts + 1];
  int cnt_a[kMaxGroups + 1];
  int cnt_b[kMaxGroups + 1];
  int tmp[40];
  int flag;
};

// ------------------------------------------------------------------ phase 1
// J: 8-logit MMA tiles per pass over K; TT: 16-token tiles per item (each router-weight
// fragment a warp loads from L2 feeds TT tiles: the weights are re-read once per item,
// which bounds phase 1 for long batches).  J = 8, TT = 1 (one pass for <= 64 logits) in
// the one-cluster / last-block forms and the grid form; J = 4, TT = 2 in the grid form's
// wide instance, which keeps the kernel at <= 128 registers (two CTAs per SM, twice the
// warps to hide the latency of phase 2's loads; the activations of a token tile are read
// once per pass, from L2 after the first).
template <int J, int TT>
__device__ void phase_router(const RouteArgs& a) {
  const int lane = threadIdx.x & 31;
  const int g = lane >> 2, c = lane & 3;
  const int gw = blockIdx.x * (kRouteThreads / 32) + (threadIdx.x >> 5);
  const int nw = gridDim.x * (kRouteThreads / 32);
  const int64_t T = a.T;
  const int H = a.H;
  const int ntt = static_cast<int>((T + 15) / 16);
  const int nti = (ntt + TT - 1) / TT;  // items of TT token tiles
  const int kblocks = H / 32;
  const int items = nti * a.ksplit;
  const int Etot = a.E + (a.shared_gate_w ? 1 : 0);  // logits: the experts and the shared gate
  const int ngroups = (Etot + 8 * J - 1) / (8 * J);  // logit groups (columns past Etot are never read)
  for (int item = gw; item < items; item += nw) {
    const int ti = item / a.ksplit, ks = item % a.ksplit;
    const int kb0 = kblocks * ks / a.ksplit, kb1 = kblocks * (ks + 1) / a.ksplit;
    int64_t ta[TT], tb[TT];
    const uint16_t* xa[TT];
    const uint16_t* xb[TT];
#pragma unroll
    for (int u = 0; u < TT; ++u) {
      const int64_t t0 = static_cast<int64_t>(ti * TT + u) * 16;
      ta[u] = t0 + g;
      tb[u] = t0 + g + 8;
      xa[u] = (ta[u] < T) ? a.x + ta[u] * H : nullptr;
      xb[u] = (tb[u] < T) ? a.x + tb[u] * H : nullptr;
    }
    for (int eg = 0; eg < ngroups; ++eg) {
      float acc[TT][J][4];
#pragma unroll
      for (int u = 0; u < TT; ++u)
#pragma unroll
        for (int j = 0; j < J; ++j) acc[u][j][0] = acc[u][j][1] = acc[u][j][2] = acc[u][j][3] = 0.f;
      const uint16_t* wr[J];
#pragma unroll
      for (int j = 0; j < J; ++j) {
        const int e = eg * 8 * J + 8 * j + g;
        wr[j] = (e < a.E) ? a.router_w + static_cast<int64_t>(e) * H : (e == a.E ? a.shared_gate_w : nullptr);
      }
      // the loads of k-block kb + 1 are issued before the MMAs of kb (double-buffered
      // registers), so an item pays the load latency about once, not once per k-block
      const uint4 z = make_uint4(0, 0, 0, 0);
      uint4 va[TT], vb[TT], w[J];
      auto load_kb = [&](int kb, uint4 (&xa_v)[TT], uint4 (&xb_v)[TT], uint4 (&wv)[J]) {
        const int koff = kb * 32 + 8 * c;
#pragma unroll
        for (int u = 0; u < TT; ++u) {
          xa_v[u] = xa[u] ? ldg_v4(xa[u] + koff) : z;
          xb_v[u] = xb[u] ? ldg_v4(xb[u] + koff) : z;
        }
#pragma unroll
        for (int j = 0; j < J; ++j) wv[j] = wr[j] ? ldg_v4(wr[j] + koff) : z;
      };
      if (kb0 < kb1) load_kb(kb0, va, vb, w);
      for (int kb = kb0; kb < kb1; ++kb) {
        uint4 na[TT], nb[TT], nw[J];
#pragma unroll
        for (int u = 0; u < TT; ++u) na[u] = nb[u] = z;
#pragma unroll
        for (int j = 0; j < J; ++j) nw[j] = z;
        if (kb + 1 < kb1) load_kb(kb + 1, na, nb, nw);
        const int koff = kb * 32 + 8 * c;
        if (eg == 0) {
#pragma unroll
          for (int u = 0; u < TT; ++u) {
            if (xa[u]) *reinterpret_cast<uint4*>(a.x_perm + ta[u] * H + koff) = perm_chunk(va[u]);
            if (xb[u]) *reinterpret_cast<uint4*>(a.x_perm + tb[u] * H + koff) = perm_chunk(vb[u]);
          }
        }
#pragma unroll
        for (int j = 0; j < J; ++j)
#pragma unroll
          for (int u = 0; u < TT; ++u) {
            mma_bf16_16816(acc[u][j], va[u].x, vb[u].x, va[u].y, vb[u].y, w[j].x, w[j].y);
            mma_bf16_16816(acc[u][j], va[u].z, vb[u].z, va[u].w, vb[u].w, w[j].z, w[j].w);
          }
#pragma unroll
        for (int u = 0; u < TT; ++u) {
          va[u] = na[u];
          vb[u] = nb[u];
        }
#pragma unroll
        for (int j = 0; j < J; ++j) w[j] = nw[j];
      }
      float* part = a.partial + static_cast<int64_t>(ks) * T * a.epad;
#pragma unroll
      for (int j = 0; j < J; ++j) {
        const int e = eg * 8 * J + 8 * j + 2 * c;
        if (e < a.epad) {
#pragma unroll
          for (int u = 0; u < TT; ++u) {
            if (ta[u] < T) *reinterpret_cast<float2*>(part + ta[u] * a.epad + e) = make_float2(acc[u][j][0], acc[u][j][1]);
            if (tb[u] < T) *reinterpret_cast<float2*>(part + tb[u] * a.epad + e) = make_float2(acc[u][j][2], acc[u][j][3]);
          }
        }
      }
    }
  }
}

__device__ void phase_permute_x(const RouteArgs& a) {
  const int64_t chunks_per_row = a.H / 8;
  const int64_t n = a.x_rows * chunks_per_row;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const uint4 v = ldg_v4(a.x + i * 8);
    *reinterpret_cast<uint4*>(a.x_perm + i * 8) = perm_chunk(v);
  }
}

__device__ void phase_zero(float* p, int64_t n) {
  if (!p) return;
  const int64_t n4 = n / 4;
  float4* p4 = reinterpret_cast<float4*>(p);
  const float4 z = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n4;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x)
    p4[i] = z;
  for (int64_t i = n4 * 4 + static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x)
    p[i] = 0.f;
}

// ------------------------------------------------------------------ phase 2
static_assert(kRouteChunk <= 32, "one bitmask word per expert and chunk");

// the raw (fp32) logits of token t held by this lane: logit lane + 32 i, for the experts
// and the shared gate (slot E), each the fixed-order sum (ks = 0, 1, ...) of its K-split
// router partials.  The loads of KB slices of all the lane's logits are issued before
// any is added, so a token waits for ceil(ksplit / KB) L2 round trips, not one per
// logit and slice group.
template <int PER>
FM_DEV void load_logits(const RouteArgs& a, int64_t t, float (&raw)[PER]) {
  constexpr int KB = PER >= 32 ? 1 : 32 / PER;  // <= 32 loads in flight per lane
  const int lane = threadIdx.x & 31;
  const float* p = a.partial + t * a.epad + lane;
  const int64_t stride = a.T * a.epad;
  bool valid[PER];
#pragma unroll
  for (int i = 0; i < PER; ++i) {
    const int e = lane + 32 * i;
    valid[i] = e < a.E || (e == a.E && a.shared_gate_w);
    raw[i] = 0.f;
  }
  for (int ks0 = 0; ks0 < a.ksplit; ks0 += KB) {
    float v[KB][PER];
#pragma unroll
    for (int u = 0; u < KB; ++u)
#pragma unroll
      for (int i = 0; i < PER; ++i)
        v[u][i] = (valid[i] && ks0 + u < a.ksplit) ? p[(ks0 + u) * stride + 32 * i] : 0.f;
#pragma unroll
    for (int u = 0; u < KB; ++u)
#pragma unroll
      for (int i = 0; i < PER; ++i)
        if (ks0 + u < a.ksplit) raw[i] += v[u][i];
  }
}

template <int PER>
__device__ void route_token(const RouteArgs& a, int64_t t, RouteSmem* sm, int tl, const float (&raw)[PER]) {
  const int lane = threadIdx.x & 31;
  const int E = a.E, k = a.k;
  float p[PER];
  // bf16 logits: fixed-order sum of the K-split partials, then the optional bias
  float mx = -INFINITY;
#pragma unroll
  for (int i = 0; i < PER; ++i) {
    const int e = lane + 32 * i;
    p[i] = -INFINITY;
    if (e < E) {
      float l = rbf(raw[i]);
      if (a.router_bias) l = rbf(l + bf2f(a.router_bias[e]));
      p[i] = l;
      mx = fmaxf(mx, l);
    } else if (e == E && a.shared_gate_w) {
      a.gate_sig[t] = rbf(sigmoid_f(rbf(raw[i])));
    }
  }
  if (a.shared_ungated && lane == 0) a.gate_sig[t] = 1.0f;
  mx = warp_max(mx);
  // softmax(precise): fp32 exp; sum = lane-strided partial sums then xor butterfly
  float part = 0.f;
#pragma unroll
  for (int i = 0; i < PER; ++i) {
    const int e = lane + 32 * i;
    if (e < E) {
      p[i] = expf(p[i] - mx);
      part += p[i];
    }
  }
  const float sum = warp_sum_bfly(part);
#pragma unroll
  for (int i = 0; i < PER; ++i) {
    const int e = lane + 32 * i;
    p[i] = (e < E) ? rbf(p[i] / sum) : -INFINITY;
  }
  // top-k: k rounds of one warp max over 32-bit keys (bf16 probability bits << 16 |
  // 0xFFFF - expert).  The probabilities are bf16 values >= 0, so their bits order like
  // the values; equal probabilities go to the lower expert id.  NaN (bad input) ranks
  // lowest, and every round still returns a distinct valid id.
  uint32_t key[PER];
#pragma unroll
  for (int i = 0; i < PER; ++i) {
    const int e = lane + 32 * i;
    const uint32_t pb = isnan(p[i]) ? 0u : static_cast<uint32_t>(f2bf(p[i]));
    key[i] = (e < E) ? ((pb << 16) | static_cast<uint32_t>(0xFFFF - e)) : 0u;
  }
  // lane j keeps the pick of round j; the renormalisation sum runs in round order
  float sp = 0.f, ssum = 0.f;
  int se = 0;
  for (int j = 0; j < k; ++j) {
    uint32_t best = 0u;
#pragma unroll
    for (int i = 0; i < PER; ++i) best = max(best, key[i]);
    best = __reduce_max_sync(0xffffffffu, best);
    const int be = 0xFFFF - static_cast<int>(best & 0xFFFFu);
    const float bp = bf2f(static_cast<uint16_t>(best >> 16));
    if (lane == j) {
      sp = bp;
      se = be;
    }
    ssum += bp;
#pragma unroll
    for (int i = 0; i < PER; ++i)
      if (lane + 32 * i == be) key[i] = 0u;  // taken (a valid key is never 0: 0xFFFF - e > 0)
  }
  const float denom = a.norm_topk ? rbf(ssum) : 1.f;
  if (lane < k) {
    const float sc = a.norm_topk ? rbf(sp / denom) : sp;
    a.topk_ids[t * k + lane] = se;
    a.topk_score[t * k + lane] = sc;
    if (a.out_topk_ids) a.out_topk_ids[t * k + lane] = se;
    if (a.out_topk_scores) a.out_topk_scores[t * k + lane] = f2bf(sc);
    if (a.out_scores_f32) a.out_scores_f32[t * k + lane] = sc;
    if (sm) {
      sm->ids[tl * k + lane] = se;
      atomicOr(&sm->mask[se], 1u << tl);
    }
  }
}

// fp32 -> 32-bit key with the same order (NaN lowest)
FM_DEV uint32_t ordered_key(float f) {
  if (isnan(f)) return 0u;
  const uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// Sigmoid routing of one token by one warp (the Nemotron-H / DeepSeek-style block,
// nemotron_h.cpp:1018-1050): orig = sigmoid(fp32(bf16 logit)); sel = orig + correction
// bias; with n_group > 1 each group scores the sum of its two best sel and the
// n_group - topk_group lowest groups (equal scores: the higher group id first) get
// sel = 0; top-k of sel (equal: lower expert id) in k rounds of a 64-bit warp max; the
// scores are the picks' orig, divided by (their sum in pick order + 1e-20) when
// norm_topk and k > 1, times routed_scale, all fp32.
template <int PER>
__device__ void route_token_sigmoid(const RouteArgs& a, int64_t t, RouteSmem* sm, int tl, const float (&raw)[PER]) {
  const int lane = threadIdx.x & 31;
  const int E = a.E, k = a.k;
  float orig[PER];
  unsigned long long key[PER];
#pragma unroll
  for (int i = 0; i < PER; ++i) {
    const int e = lane + 32 * i;
    orig[i] = 0.f;
    key[i] = 0ull;
    if (e < E) {
      const float l = rbf(raw[i]);
      orig[i] = 1.0f / (1.0f + expf(-l));
    } else if (e == E && a.shared_gate_w) {
      a.gate_sig[t] = rbf(sigmoid_f(rbf(raw[i])));
    }
  }
  if (a.shared_ungated && lane == 0) a.gate_sig[t] = 1.0f;
  float sel[PER];
#pragma unroll
  for (int i = 0; i < PER; ++i) {
    const int e = lane + 32 * i;
    sel[i] = (e < E) ? (a.corr_bias ? orig[i] + a.corr_bias[e] : orig[i]) : -INFINITY;
  }
  if (a.n_group > 1) {  // n_group <= 32 (host-checked): lane gi holds group gi's score
    const int gsz = E / a.n_group;
    float gmine = 0.f;
    for (int gi = 0; gi < a.n_group; ++gi) {
      float m1 = -INFINITY, m2 = -INFINITY;
#pragma unroll
      for (int i = 0; i < PER; ++i) {
        const int e = lane + 32 * i;
        if (e < E && e / gsz == gi) {
          const float v = sel[i];
          if (v > m1) {
            m2 = m1;
            m1 = v;
          } else if (v > m2) {
            m2 = v;
          }
        }
      }
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) {  // top two of the warp
        const float b1 = __shfl_xor_sync(0xffffffffu, m1, off);
        const float b2 = __shfl_xor_sync(0xffffffffu, m2, off);
        const float n2 = fmaxf(fminf(m1, b1), fmaxf(m2, b2));
        m1 = fmaxf(m1, b1);
        m2 = n2;
      }
      if (lane == gi) gmine = m1 + m2;
    }
    int rank = 0;  // groups zeroed before this lane's group
    for (int gj = 0; gj < a.n_group; ++gj) {
      const float v = __shfl_sync(0xffffffffu, gmine, gj);
      if (lane < a.n_group && (v < gmine || (v == gmine && gj > lane))) ++rank;
    }
    const uint32_t zmask = __ballot_sync(0xffffffffu, lane < a.n_group && rank < a.n_group - a.topk_group);
#pragma unroll
    for (int i = 0; i < PER; ++i) {
      const int e = lane + 32 * i;
      if (e < E && ((zmask >> (e / gsz)) & 1u)) sel[i] = 0.f;
    }
  }
#pragma unroll
  for (int i = 0; i < PER; ++i) {
    const int e = lane + 32 * i;
    if (e < E)  // a valid key is never 0: its low half is 0xFFFF - e > 0
      key[i] = (static_cast<unsigned long long>(ordered_key(sel[i])) << 32) | static_cast<uint32_t>(0xFFFF - e);
  }
  float sp = 0.f, ssum = 0.f;
  int se = 0;
  for (int j = 0; j < k; ++j) {
    unsigned long long best = 0ull;
#pragma unroll
    for (int i = 0; i < PER; ++i) best = key[i] > best ? key[i] : best;
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
      const unsigned long long o = __shfl_xor_sync(0xffffffffu, best, off);
      best = o > best ? o : best;
    }
    const int be = 0xFFFF - static_cast<int>(best & 0xFFFFu);
    float mine = 0.f;  // the pick's orig, from the lane that holds it
#pragma unroll
    for (int i = 0; i < PER; ++i)
      if (i == (be >> 5)) mine = orig[i];
    const float bo = __shfl_sync(0xffffffffu, mine, be & 31);
    if (lane == j) {
      sp = bo;
      se = be;
    }
    ssum += bo;
#pragma unroll
    for (int i = 0; i < PER; ++i)
      if (lane + 32 * i == be) key[i] = 0ull;
  }
  const bool renorm = a.norm_topk && k > 1;
  const float denom = renorm ? ssum + 1e-20f : 1.f;
  if (lane < k) {
    const float sc = (renorm ? sp / denom : sp) * a.routed_scale;
    a.topk_ids[t * k + lane] = se;
    a.topk_score[t * k + lane] = sc;
    if (a.out_topk_ids) a.out_topk_ids[t * k + lane] = se;
    if (a.out_topk_scores) a.out_topk_scores[t * k + lane] = f2bf(sc);
    if (a.out_scores_f32) a.out_scores_f32[t * k + lane] = sc;
    if (sm) {
      sm->ids[tl * k + lane] = se;
      atomicOr(&sm->mask[se], 1u << tl);
    }
  }
}

__device__ void given_row(const RouteArgs& a, int64_t r, RouteSmem* sm, int tl) {
  if ((threadIdx.x & 31) != 0) return;
  const int64_t b = r / a.M, m = r % a.M;
  uint32_t e = a.given_ids ? a.given_ids[b] : 0u;
  int64_t xb = a.given_lhs ? static_cast<int64_t>(a.given_lhs[b]) : b * a.x_batches / a.batches;
  if (e >= static_cast<uint32_t>(a.E) || xb < 0 || xb >= a.x_batches) {
    report(a.err, DEVERR_BOUNDS);
    a.topk_ids[r] = -1;
    if (sm) sm->ids[tl] = -1;
    return;
  }
  a.topk_ids[r] = static_cast<int32_t>(e);
  a.topk_score[r] = 1.f;
  a.row_src[r] = static_cast<int32_t>(xb * a.M + m);
  if (sm) {
    sm->ids[tl] = static_cast<int>(e);
    atomicOr(&sm->mask[e], 1u << tl);
  }
}

// one token (or given row) t, routed by the calling warp
template <bool SIGMOID, int PER>
__device__ void route_one_per(const RouteArgs& a, int64_t t, RouteSmem* sm, int tl) {
  float raw[PER];
  load_logits<PER>(a, t, raw);
  if (SIGMOID) route_token_sigmoid<PER>(a, t, sm, tl, raw); else route_token<PER>(a, t, sm, tl, raw);
}

template <bool SIGMOID>
__device__ void route_one(const RouteArgs& a, int64_t t, RouteSmem* sm, int tl) {
  // lanes cover the logit slots: the E routed experts and, when the block has one, the
  // shared-expert gate at slot E (128 experts without a gate: four slots a lane)
  const int slots = a.E + (a.shared_gate_w ? 1 : 0);
  if (!a.do_router) given_row(a, t, sm, tl);
  else if (slots <= 64) route_one_per<SIGMOID, 2>(a, t, sm, tl);
  else if (slots <= 128) route_one_per<SIGMOID, 4>(a, t, sm, tl);
  else if (slots <= 256) route_one_per<SIGMOID, 8>(a, t, sm, tl);
  else route_one_per<SIGMOID, 17>(a, t, sm, tl);  // up to kMaxExperts = 512 experts and the gate
}

// the chunk's counts and stable in-chunk ranks from its bitmasks (sm.mask, sm.ids)
__device__ void count_chunk(const RouteArgs& a, RouteSmem& sm, int ch, int k) {
  for (int e = threadIdx.x; e < a.E; e += blockDim.x)
    a.chunk_counts[static_cast<int64_t>(ch) * a.E + e] = __popc(sm.mask[e]);
  const int64_t t0 = static_cast<int64_t>(ch) * kRouteChunk;
  const int ntok = static_cast<int>(a.T - t0 < kRouteChunk ? a.T - t0 : kRouteChunk);
  for (int i = threadIdx.x; i < ntok * k; i += blockDim.x) {
    const int tl = i / k;
    const int e = sm.ids[i];
    if (e < 0) continue;
    a.pair_rank[(t0 + tl) * k + (i % k)] = __popc(sm.mask[e] & ((1u << tl) - 1u));
  }
}

// bid / nb: this block's place among the blocks that share the phase (the whole grid in
// the cooperative kernel, block 0 of 1 in the last-block tail)
template <bool SIGMOID>
__device__ void phase_topk_count(const RouteArgs& a, RouteSmem& sm, int bid, int nb) {
  const int warp = threadIdx.x >> 5;
  const int nchunks = static_cast<int>((a.T + kRouteChunk - 1) / kRouteChunk);
  const int k = a.do_router ? a.k : 1;
  for (int ch = bid; ch < nchunks; ch += nb) {
    for (int e = threadIdx.x; e < a.E; e += blockDim.x) sm.mask[e] = 0u;
    __syncthreads();
    for (int i = 0; i < kRouteChunk / 8; ++i) {
      const int tl = warp * (kRouteChunk / 8) + i;
      const int64_t t = static_cast<int64_t>(ch) * kRouteChunk + tl;
      if (t >= a.T) break;
      route_one<SIGMOID>(a, t, &sm, tl);
    }
    __syncthreads();
    count_chunk(a, sm, ch, k);
    __syncthreads();
  }
}

// Phase 2 split in two for batches with few chunks (at most half the blocks'): every
// warp of the grid routes tokens (ids and scores to global memory), then, after a grid
// barrier, a block per chunk rebuilds the chunk's bitmasks from the ids and counts it --
// instead of 8 warps per chunk routing 2 tokens each while most blocks idle.  The same
// route_one and count_chunk, so the same ids, scores, counts and ranks.
template <bool SIGMOID>
__device__ void phase_topk_spread(const RouteArgs& a) {
  const int nw = gridDim.x * (kRouteThreads / 32);
  const int gw = blockIdx.x * (kRouteThreads / 32) + (threadIdx.x >> 5);
  for (int64_t tk = gw; tk < a.T; tk += nw) route_one<SIGMOID>(a, tk, nullptr, 0);
}

__device__ void phase_count_from_ids(const RouteArgs& a, RouteSmem& sm, int bid, int nb) {
  const int k = a.do_router ? a.k : 1;
  const int nchunks = static_cast<int>((a.T + kRouteChunk - 1) / kRouteChunk);
  for (int ch = bid; ch < nchunks; ch += nb) {
    for (int e = threadIdx.x; e < a.E; e += blockDim.x) sm.mask[e] = 0u;
    __syncthreads();
    const int64_t t0 = static_cast<int64_t>(ch) * kRouteChunk;
    const int ntok = static_cast<int>(a.T - t0 < kRouteChunk ? a.T - t0 : kRouteChunk);
    for (int i = threadIdx.x; i < ntok * k; i += blockDim.x) {
      const int e = a.topk_ids[t0 * k + i];
      sm.ids[i] = e;
      if (e >= 0) atomicOr(&sm.mask[e], 1u << (i / k));
    }
    __syncthreads();
    count_chunk(a, sm, ch, k);
    __syncthreads();
  }
}

// ------------------------------------------------------------------ phase 3
__device__ void phase_column_scan(const RouteArgs& a, RouteSmem& sm) {
  const int nchunks = static_cast<int>((a.T + kRouteChunk - 1) / kRouteChunk);
  int* buf = sm.cnt_a;  // reuse as scratch (kMaxGroups+1 >= 513 ints per pass)
  const int cap = kMaxGroups;
  for (int e = blockIdx.x; e < a.E; e += gridDim.x) {
    int carry = 0;
    for (int c0 = 0; c0 < nchunks; c0 += cap) {
      const int n = min(cap, nchunks - c0);
      for (int i = threadIdx.x; i < n; i += blockDim.x)
        buf[i] = a.chunk_counts[static_cast<int64_t>(c0 + i) * a.E + e];
      __syncthreads();
      const int tot = block_exclusive_scan(buf, n, sm.tmp);
      for (int i = threadIdx.x; i < n; i += blockDim.x)
        a.chunk_counts[static_cast<int64_t>(c0 + i) * a.E + e] = buf[i] + carry;
      carry += tot;
      __syncthreads();
    }
    if (threadIdx.x == 0) a.totals[e] = carry;
  }
}

// Phase 3 for one block and at most kRouteLastMaxChunks chunks: each thread scans its
// experts' chunk counts in registers (same exclusive scan and totals as above).
__device__ void phase_column_scan_one_block(const RouteArgs& a) {
  const int nchunks = static_cast<int>((a.T + kRouteChunk - 1) / kRouteChunk);
  for (int e = threadIdx.x; e < a.E; e += blockDim.x) {
    int c[kRouteLastMaxChunks];
#pragma unroll
    for (int i = 0; i < kRouteLastMaxChunks; ++i)
      c[i] = i < nchunks ? a.chunk_counts[static_cast<int64_t>(i) * a.E + e] : 0;
    int run = 0;
#pragma unroll
    for (int i = 0; i < kRouteLastMaxChunks; ++i) {
      if (i < nchunks) a.chunk_counts[static_cast<int64_t>(i) * a.E + e] = run;
      run += c[i];
    }
    a.totals[e] = run;
  }
}

// ------------------------------------------------------------------ phase 4
// Group G's tiling: weight blocks of rows_per_block output rows, chunks of at most
// chunk_max activation rows (balanced, rounded up to chunk_align), K splits.
__device__ void plan_one(TileGroup& G, int n_out, int rows_per_block, int chunk_max, int chunk_align) {
  G.nblocks = (n_out + rows_per_block - 1) / rows_per_block;
  if (G.rows > 0) {
    const int c0 = (G.rows + chunk_max - 1) / chunk_max;
    int cr = (G.rows + c0 - 1) / c0;
    cr = (cr + chunk_align - 1) / chunk_align * chunk_align;
    G.chunk_rows = cr;
    G.chunks = (G.rows + cr - 1) / cr;
  } else {
    G.chunk_rows = chunk_align;
    G.chunks = 0;
  }
}

// tile_begin of every group (exclusive scan of the tile counts) and the totals; cnt
// holds each group's tile count on entry (one CTA)
__device__ void finish_table(TileTable* tab, int ng, int* cnt, int* s_tmp) {
  __syncthreads();
  const int total = block_exclusive_scan(cnt, ng, s_tmp);
  for (int gi = threadIdx.x; gi < ng; gi += blockDim.x) tab->g[gi].tile_begin = cnt[gi];
  if (threadIdx.x == 0) {
    tab->num_groups = ng;
    tab->num_tiles = total;
  }
}

// One block plans a table: a group per thread, the tile counts' exclusive scan over the
// block (the grid form, whose blocks 0 and 1 have nothing else to do meanwhile).
__device__ void plan_groups(const RouteArgs& a, RouteSmem& sm, TileTable* tab, int rows_per_block, int n_routed,
                            int n_shared, int ksplit_shared, int* cnt) {
  const int has_sh = (n_shared > 0) ? 1 : 0;
  const int ng = a.E + has_sh;
  for (int gi = threadIdx.x; gi < ng; gi += blockDim.x) {
    TileGroup G;
    const bool sh = has_sh && gi == 0;
    const int e = sh ? -1 : gi - has_sh;
    G.expert = e;
    G.row_begin = sh ? 0 : sm.offs[e];
    G.rows = sh ? static_cast<int>(a.T) : (sm.offs[e + 1] - sm.offs[e]);
    G.ksplit = sh ? ksplit_shared : 1;
    plan_one(G, sh ? n_shared : n_routed, rows_per_block, a.chunk_max, a.chunk_align);
    tab->g[gi] = G;
    cnt[gi] = G.nblocks * G.chunks * G.ksplit;
  }
  finish_table(tab, ng, cnt, sm.tmp);
}

// One warp plans a whole table (the one-CTA tails of the small-batch forms): 32 groups at a time, the tile counts' exclusive scan by
// shuffles (group order, as the block scan gives), no block barrier -- so the tables and
// the scatter run on different warps at once.
__device__ void plan_groups_warp(const RouteArgs& a, const int* offs, TileTable* tab, int rows_per_block,
                                 int n_routed, int n_shared, int ksplit_shared) {
  const int lane = threadIdx.x & 31;
  const int has_sh = (n_shared > 0) ? 1 : 0;
  const int ng = a.E + has_sh;
  int running = 0;  // tiles of the groups before this batch of 32
  for (int base = 0; base < ng; base += 32) {
    const int gi = base + lane;
    TileGroup G;
    int cnt = 0;
    if (gi < ng) {
      const bool sh = has_sh && gi == 0;
      const int e = sh ? -1 : gi - has_sh;
      G.expert = e;
      G.row_begin = sh ? 0 : offs[e];
      G.rows = sh ? static_cast<int>(a.T) : (offs[e + 1] - offs[e]);
      G.ksplit = sh ? ksplit_shared : 1;
      plan_one(G, sh ? n_shared : n_routed, rows_per_block, a.chunk_max, a.chunk_align);
      cnt = G.nblocks * G.chunks * G.ksplit;
    }
    int incl = cnt;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const int u = __shfl_up_sync(0xffffffffu, incl, off);
      if (lane >= off) incl += u;
    }
    if (gi < ng) {
      G.tile_begin = running + incl - cnt;
      tab->g[gi] = G;
    }
    running += __shfl_sync(0xffffffffu, incl, 31);
  }
  if (lane == 0) {
    tab->num_groups = ng;
    tab->num_tiles = running;
  }
}

// The offsets (block 0) and the two tile tables, once sm.offs[0..E] holds the experts'
// exclusive row starts: table a in block 0 and table b in block 1 -- each planned by the
// whole block -- in the grid form; a block alone (the small-batch forms) has its warp 0
// plan table a and its warp 1 table b while the other warps go on to the scatter.
__device__ void emit_offsets_tables(const RouteArgs& a, RouteSmem& sm, int bid, int nb) {
  const int warp = threadIdx.x >> 5;
  if (bid == 0) {
    for (int e = threadIdx.x; e <= a.E; e += blockDim.x) {
      a.offsets[e] = sm.offs[e];
      if (a.out_offsets) a.out_offsets[e] = sm.offs[e];
    }
  }
  if (nb > 1) {
    if (bid == 0 && a.tab_a)
      plan_groups(a, sm, a.tab_a, a.a_rows_per_block, a.a_n, a.has_shared ? a.a_n_shared : 0, 1, sm.cnt_a);
    if (bid == 1 && a.tab_b)
      plan_groups(a, sm, a.tab_b, a.b_rows_per_block, a.b_n, a.has_shared ? a.b_n : 0, a.b_ksplit_shared, sm.cnt_b);
  } else {
    if (warp == 0 && a.tab_a)
      plan_groups_warp(a, sm.offs, a.tab_a, a.a_rows_per_block, a.a_n, a.has_shared ? a.a_n_shared : 0, 1);
    if (warp == 1 && a.tab_b)
      plan_groups_warp(a, sm.offs, a.tab_b, a.b_rows_per_block, a.b_n, a.has_shared ? a.b_n : 0, a.b_ksplit_shared);
  }
}

// the outputs of pair `flat` (expert e) placed at sorted position pos
__device__ __forceinline__ void emit_pair(const RouteArgs& a, int64_t flat, int k, int pos) {
  if (a.pair_pos) a.pair_pos[flat] = pos;
  const int64_t t = flat / k;
  a.sorted_token[pos] = a.do_router ? static_cast<int32_t>(t) : a.row_src[t];
  a.sorted_score[pos] = a.topk_score[flat];
  a.sorted_flat[pos] = static_cast<int32_t>(flat);
  if (a.out_sorted_token) a.out_sorted_token[pos] = static_cast<int32_t>(t);
}

__device__ void phase_scatter(const RouteArgs& a, RouteSmem& sm, int bid, int nb) {
  for (int e = threadIdx.x; e < a.E; e += blockDim.x) sm.offs[e] = a.totals[e];
  __syncthreads();
  const int P = block_exclusive_scan(sm.offs, a.E, sm.tmp);
  if (threadIdx.x == 0) sm.offs[a.E] = P;
  __syncthreads();
  emit_offsets_tables(a, sm, bid, nb);
  const int k = a.do_router ? a.k : 1;
  const int nchunks = static_cast<int>((a.T + kRouteChunk - 1) / kRouteChunk);
  for (int ch = bid; ch < nchunks; ch += nb) {
    const int64_t t0 = static_cast<int64_t>(ch) * kRouteChunk;
    const int ntok = static_cast<int>(a.T - t0 < kRouteChunk ? a.T - t0 : kRouteChunk);
    for (int i = threadIdx.x; i < ntok * k; i += blockDim.x) {
      const int64_t flat = t0 * k + i;
      const int e = a.topk_ids[flat];
      if (e < 0) {
        if (a.pair_pos) a.pair_pos[flat] = -1;
        continue;
      }
      emit_pair(a, flat, k, sm.offs[e] + a.chunk_counts[static_cast<int64_t>(ch) * a.E + e] + a.pair_rank[flat]);
    }
  }
}

// Phases 2b-4 of a small batch (T <= kTailTokens) in one block, in shared memory: the
// ids once from global memory, a token bitmask per expert (atomicOr), the experts'
// counts and exclusive starts, the tables, and each pair's position = its expert's start
// + the expert's tokens before it (popc of the mask below the token).  The same stable
// (expert, token) order as the chunked count / scan / scatter, without their round trips
// through global memory.
constexpr int kTailTokens = kRouteLastMaxChunks * kRouteChunk;
constexpr int kTailWords = kTailTokens / 32;
struct TailSmem {
  uint32_t tmask[kMaxExperts * kTailWords];  // [expert][token / 32]
  int ids[kTailTokens * 16];                 // the pairs' expert ids (k <= 16)
};

__device__ void tail_fused(const RouteArgs& a, RouteSmem& sm, TailSmem& ts, int k) {
  const int T = static_cast<int>(a.T), E = a.E, np = T * k;
  for (int i = threadIdx.x; i < E * kTailWords; i += blockDim.x) ts.tmask[i] = 0u;
  __syncthreads();
  for (int i = threadIdx.x; i < np; i += blockDim.x) {
    const int e = a.topk_ids[i];
    ts.ids[i] = e;
    if (e >= 0) {
      const int t = i / k;
      atomicOr(&ts.tmask[e * kTailWords + (t >> 5)], 1u << (t & 31));
    }
  }
  __syncthreads();
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    int c = 0;
#pragma unroll
    for (int w = 0; w < kTailWords; ++w) c += __popc(ts.tmask[e * kTailWords + w]);
    sm.offs[e] = c;
  }
  __syncthreads();
  const int P = block_exclusive_scan(sm.offs, E, sm.tmp);
  if (threadIdx.x == 0) sm.offs[E] = P;
  __syncthreads();
  emit_offsets_tables(a, sm, 0, 1);
  for (int i = threadIdx.x; i < np; i += blockDim.x) {
    const int e = ts.ids[i];
    if (e < 0) {
      if (a.pair_pos) a.pair_pos[i] = -1;
      continue;
    }
    const int t = i / k, wt = t >> 5;
    const uint32_t* m = ts.tmask + e * kTailWords;
    int rank = __popc(m[wt] & ((1u << (t & 31)) - 1u));
#pragma unroll
    for (int w = 0; w < kTailWords; ++w)
      if (w < wt) rank += __popc(m[w]);
    emit_pair(a, i, k, sm.offs[e] + rank);
  }
}

}  // namespace

// Dense rows in order (fm_linear: one matrix, no indices): the pair-permuted copy of x,
// identity row maps and a one-group tile table -- what the routing kernel's given-ids path
// writes in that case -- from one plain launch, without its grid barriers.
__global__ void __launch_bounds__(256) dense_prep_kernel(const RouteArgs a) {
  phase_permute_x(a);
  const int64_t T = a.T;
  for (int64_t r = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; r < T;
       r += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    a.sorted_token[r] = static_cast<int32_t>(r);
    a.sorted_flat[r] = static_cast<int32_t>(r);
    a.sorted_score[r] = 1.f;
  }
  if (blockIdx.x == 0 && threadIdx.x == 0) {
    TileGroup G;
    G.expert = 0;
    G.row_begin = 0;
    G.rows = static_cast<int32_t>(T);
    G.ksplit = 1;
    plan_one(G, a.a_n, a.a_rows_per_block, a.chunk_max, a.chunk_align);
    G.tile_begin = 0;
    a.tab_a->g[0] = G;
    a.tab_a->num_groups = 1;
    a.tab_a->num_tiles = G.nblocks * G.chunks;
    a.offsets[0] = 0;
    a.offsets[1] = static_cast<int32_t>(T);
  }
}

FM_DEV unsigned long long global_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

// thread 0 of the block that reports (block 0; the last block in the last-block form)
// accumulates the wall time of each phase as that block saw it
FM_DEV void phase_mark(const RouteArgs& a, int phase, unsigned long long& t, bool reporter) {
  if (reporter && threadIdx.x == 0 && a.phase_ns) {
    const unsigned long long now = global_ns();
    atomicAdd(a.phase_ns + phase, now - t);
    t = now;
  }
}

// Expert-parallel plan (one CTA): the rows a rank received sit in source-rank order,
// each source's rows in expert-major order, so every (source, local expert) segment is
// one tile group over contiguous rows; the rank's own tokens form the shared-expert
// group.  Also writes the identity row map and unit scores the expert kernels read
// for the received rows (the owner returns bf16(d); the token's rank scales it).
__device__ void ep_plan_body(const EpPlanArgs& a) {
  __shared__ int cnt_a[kMaxGroups + 1];
  __shared__ int cnt_b[kMaxGroups + 1];
  __shared__ int rbeg[kMaxGroups + 1];
  __shared__ int s_tmp[40];
  const int has_sh = a.T_shared > 0 ? 1 : 0;
  const int nseg = a.world * a.E_local;
  const int ng = nseg + has_sh;
  if (ng > kMaxGroups) {
    if (threadIdx.x == 0) report(a.err, DEVERR_CONFIG);
    return;
  }
  for (int i = threadIdx.x; i < nseg; i += blockDim.x) rbeg[i] = a.recv_counts[i];
  __syncthreads();
  const int R = block_exclusive_scan(rbeg, nseg, s_tmp);
  for (int gi = threadIdx.x; gi < ng; gi += blockDim.x) {
    const bool sh = has_sh && gi == 0;
    // routed groups in source order src_rot, src_rot + 1, ...: when every owner starts
    // from a different source, the down GEMMs' stores of d rows into the sources' memory
    // spread over all links instead of all owners writing to one source at a time
    const int k = sh ? 0 : gi - has_sh;
    const int src = (k / a.E_local + a.src_rot) % a.world;
    const int sg = src * a.E_local + k % a.E_local;
    TileGroup G;
    G.expert = sh ? -1 : sg % a.E_local;
    G.row_begin = sh ? 0 : rbeg[sg];
    G.rows = sh ? a.T_shared : a.recv_counts[sg];
    G.ksplit = 1;
    plan_one(G, sh ? a.a_n_shared : a.a_n, a.a_rows_per_block, a.chunk_max, a.chunk_align);
    a.tab_a->g[gi] = G;
    cnt_a[gi] = G.nblocks * G.chunks;
    G.ksplit = sh ? a.b_ksplit_shared : 1;
    plan_one(G, a.b_n, a.b_rows_per_block, a.chunk_max, a.chunk_align);
    a.tab_b->g[gi] = G;
    cnt_b[gi] = G.nblocks * G.chunks * G.ksplit;
  }
  finish_table(a.tab_a, ng, cnt_a, s_tmp);
  finish_table(a.tab_b, ng, cnt_b, s_tmp);
  for (int p = threadIdx.x; p < R; p += blockDim.x) {
    a.row_map[p] = p;
    a.unit_score[p] = 1.0f;
  }
  if (threadIdx.x == 0) *a.recv_total = R;
}

__global__ void __launch_bounds__(kRouteThreads) ep_plan_kernel(const EpPlanArgs a) { ep_plan_body(a); }

// Peer-memory variant (ep.cu): wait for every source's rows, copy the (source, local
// expert) counts of this owner from its board into the plan's count array, point each
// received row at its d row's destination (its source rank's ret buffer, at the row's
// position in that rank's send order), then plan.
__global__ void __launch_bounds__(kRouteThreads) ep_p2p_plan_kernel(const EpP2PArgs a, EpPlanArgs pa) {
  __shared__ int64_t s_off[kEpMaxWorld + 1], s_start[kEpMaxWorld];
  if (ep_block_error(a)) return;
  if (!ep_wait_all(a, 1)) return;
  const int W = a.world, E = a.E, me = a.rank;
  int first, count;
  ep_owner_range(E, me, W, first, count);
  const int32_t* cnt = ep_board(a, me);
  int32_t* rc = const_cast<int32_t*>(pa.recv_counts);
  for (int i = threadIdx.x; i < W * count; i += blockDim.x) {
    const int s = i / count, e = i % count;
    rc[i] = cnt[static_cast<int64_t>(s) * E + first + e];
  }
  if (threadIdx.x < W) {
    int64_t start = 0;
    for (int e = 0; e < first; ++e) start += cnt[static_cast<int64_t>(threadIdx.x) * E + e];
    s_start[threadIdx.x] = start;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    int64_t off = 0;
    for (int s = 0; s < W; ++s) {
      s_off[s] = off;
      for (int e = 0; e < count; ++e) off += rc[s * count + e];
    }
    s_off[W] = off;
    if (off > a.cap_recv) report(a.err, DEVERR_BOUNDS);
  }
  __syncthreads();
  const int64_t R = s_off[W] < a.cap_recv ? s_off[W] : a.cap_recv;
  for (int64_t p = threadIdx.x; p < R; p += blockDim.x) {
    int s = 0;
    while (s + 1 < W && p >= s_off[s + 1]) ++s;
    const int64_t pos = s_start[s] + (p - s_off[s]);
    if (pos >= a.cap_ret) {
      report(a.err, DEVERR_BOUNDS);
      a.row_dst[p] = nullptr;
      continue;
    }
    a.row_dst[p] = ep_rows(a, s, a.off_ret) + pos * a.H;
  }
  if (ep_block_error(a)) return;  // a barrier: the count array is complete before planning reads it
  ep_plan_body(pa);
}

template <bool SIGMOID, int J>
__device__ __forceinline__ void route_body(const RouteArgs& a, RouteSmem& sm) {
  const unsigned nb = gridDim.x;
  unsigned long long t = (blockIdx.x == 0 && threadIdx.x == 0) ? global_ns() : 0ull;
  // phase 1
  if (a.do_router) phase_router<J, (J == 4 ? 2 : 1)>(a);
  else phase_permute_x(a);
  phase_zero(a.zero0, a.zero0_n);
  phase_zero(a.zero1, a.zero1_n);
  if (!grid_sync(a.gsync, nb, a.err, &sm.flag)) return;
  phase_mark(a, 0, t, blockIdx.x == 0);
  // phase 2 (split for few chunks, in the one-CTA-per-SM instance that medium batches
  // take; the branch is uniform over the grid)
  const int nchunks = static_cast<int>((a.T + kRouteChunk - 1) / kRouteChunk);
  if (J == 8 && 2 * nchunks <= static_cast<int>(nb)) {
    phase_topk_spread<SIGMOID>(a);
    if (!grid_sync(a.gsync, nb, a.err, &sm.flag)) return;
    phase_count_from_ids(a, sm, blockIdx.x, nb);
  } else {
    phase_topk_count<SIGMOID>(a, sm, blockIdx.x, nb);
  }
  if (!grid_sync(a.gsync, nb, a.err, &sm.flag)) return;
  phase_mark(a, 1, t, blockIdx.x == 0);
  // phase 3
  phase_column_scan(a, sm);
  if (!grid_sync(a.gsync, nb, a.err, &sm.flag)) return;
  phase_mark(a, 2, t, blockIdx.x == 0);
  // phase 4
  phase_scatter(a, sm, blockIdx.x, nb);
  phase_mark(a, 3, t, blockIdx.x == 0);
}

// Small batches (at most kRouteLastMaxChunks chunks): phase 1 over the whole grid, then
// the block that arrives last runs phases 2-4 alone with block barriers.  There is no
// grid barrier and nothing waits: each block makes its phase-1 stores visible
// (__threadfence) before it counts itself in, the last arrival fences again before it
// reads them, and atomicInc wraps the counter back to 0 on that arrival.
template <bool SIGMOID>
__device__ __forceinline__ void route_last_body(const RouteArgs& a, RouteSmem& sm) {
  unsigned long long t = threadIdx.x == 0 ? global_ns() : 0ull;
  if (a.do_router) phase_router<8, 1>(a);
  else phase_permute_x(a);
  phase_zero(a.zero0, a.zero0_n);
  phase_zero(a.zero1, a.zero1_n);
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    const unsigned int arrived = atomicInc(a.arrive, gridDim.x - 1);
    __threadfence();
    sm.flag = arrived == gridDim.x - 1;
  }
  __syncthreads();
  if (!sm.flag) return;
  phase_mark(a, 0, t, true);  // phase 1 as the last block to finish it saw it
  phase_topk_count<SIGMOID>(a, sm, 0, 1);
  phase_mark(a, 1, t, true);
  phase_column_scan_one_block(a);
  __syncthreads();
  phase_mark(a, 2, t, true);
  phase_scatter(a, sm, 0, 1);
  phase_mark(a, 3, t, true);
}

// Cluster form for small batches (at most kRouteLastMaxChunks chunks): one cluster of
// kRouteClusterCtas CTAs.  Phase 1 over the cluster; a cluster barrier; every warp of
// the cluster routes its share of the tokens (softmax / sigmoid, top-k, scores) into
// global memory; a second cluster barrier; then CTA 0 alone counts, scans, plans and
// scatters in shared memory (tail_fused).  The cluster barriers are hardware barriers
// (no counter in memory, no spin); the stable (expert, token) order is the one the grid
// form's chunked count / scan / scatter gives, so the ids, scores and permutation are
// identical.
FM_DEV void cluster_barrier() {
  __threadfence();  // this thread's global stores are visible device-wide before it arrives
  asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
  asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}

template <bool SIGMOID>
__device__ __forceinline__ void route_cluster_body(const RouteArgs& a, RouteSmem& sm, TailSmem& ts) {
  unsigned long long t = (blockIdx.x == 0 && threadIdx.x == 0) ? global_ns() : 0ull;
  const bool rep0 = blockIdx.x == 0;
  if (a.do_router) phase_router<8, 1>(a);
  else phase_permute_x(a);
  phase_zero(a.zero0, a.zero0_n);
  phase_zero(a.zero1, a.zero1_n);
  cluster_barrier();
  phase_mark(a, 0, t, rep0);
  const int nw = gridDim.x * (kRouteThreads / 32);
  const int gw = blockIdx.x * (kRouteThreads / 32) + (threadIdx.x >> 5);
  for (int64_t tk = gw; tk < a.T; tk += nw) route_one<SIGMOID>(a, tk, nullptr, 0);
  cluster_barrier();
  phase_mark(a, 1, t, rep0);
  if (blockIdx.x != 0) return;  // no other CTA touches this CTA's shared memory
  tail_fused(a, sm, ts, a.do_router ? a.k : 1);
  phase_mark(a, 2, t, rep0);
}

__global__ void __cluster_dims__(kRouteClusterCtas, 1, 1) __launch_bounds__(kRouteThreads)
    route_cluster_kernel(const RouteArgs a) {
  __shared__ RouteSmem sm;
  __shared__ TailSmem ts;
  route_cluster_body<false>(a, sm, ts);
}
__global__ void __cluster_dims__(kRouteClusterCtas, 1, 1) __launch_bounds__(kRouteThreads)
    route_cluster_kernel_sigmoid(const RouteArgs a) {
  __shared__ RouteSmem sm;
  __shared__ TailSmem ts;
  route_cluster_body<true>(a, sm, ts);
}

__global__ void __launch_bounds__(kRouteThreads) route_last_kernel(const RouteArgs a) {
  __shared__ RouteSmem sm;
  route_last_body<false>(a, sm);
}
__global__ void __launch_bounds__(kRouteThreads) route_last_kernel_sigmoid(const RouteArgs a) {
  __shared__ RouteSmem sm;
  route_last_body<true>(a, sm);
}

// softmax routing (the reference's LlamaModel block) and sigmoid routing (the
// Nemotron-H / DeepSeek-style block) as separate kernels, so the default one keeps its
// registers and occupancy
__global__ void __launch_bounds__(kRouteThreads) route_kernel(const RouteArgs a) {
  __shared__ RouteSmem sm;
  route_body<false, 8>(a, sm);
}
__global__ void __launch_bounds__(kRouteThreads) route_kernel_sigmoid(const RouteArgs a) {
  __shared__ RouteSmem sm;
  route_body<true, 8>(a, sm);
}
// the same with four MMA tiles per router pass, at <= 128 registers: two CTAs per SM, for
// batches whose grid the one-CTA-per-SM form would cap
__global__ void __launch_bounds__(kRouteThreads, 2) route_kernel_wide(const RouteArgs a) {
  __shared__ RouteSmem sm;
  route_body<false, 4>(a, sm);
}
__global__ void __launch_bounds__(kRouteThreads, 2) route_kernel_sigmoid_wide(const RouteArgs a) {
  __shared__ RouteSmem sm;
  route_body<true, 4>(a, sm);
}

}  // namespace fm
