// oracle.cpp -- CPU restatement of FlashMLX's MoE block hot path.
//
// TEST INFRASTRUCTURE ONLY.  Nothing in the product (libflashmoe) links or calls
// this file; only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg
// load it, and only as the checker / the timed CPU baseline.
//
// PARITY UNPINNED.  The reference path's arithmetic lives in the third-party MLX
// library (pyproject.toml:7 pins only `mlx>=0.22.0`), which is neither vendored under
// the reference tree nor installed here, and the reference's own tests
// (server/tests/test_engine.py, server/tests/test_heterogeneous_attention.cpp) hold no
// MoE golden vectors.  This file therefore restates MLX's documented semantics as the
// reference calls them, op by op, and rounds to bf16 at every MLX op boundary:
//
//   quantized_matmul(x, w, s, b, transpose=true, gs, bits)   model.cpp:476-480, 741-747
//       w_hat[n, j] = fma(s[n, j/gs], q[n, j], b[n, j/gs])      (MLX "affine" mode)
//       q[n, j]     = (w[n, j / (32/bits)] >> (bits * (j % (32/bits)))) & (2^bits - 1)
//       out[m, n]   = bf16( sum_j x[m, j] * w_hat[n, j] )        fp32 accumulation
//   gather_qmm(x, w, s, b, lhs=None, rhs, ...)                 model.cpp:703-721
//       out[b] = x[lhs(b)] @ w_hat[rhs[b]]^T                    same arithmetic per pair
//   router: matmul(x, Wr^T) -> bf16 logits                      model.cpp:757-763
//   softmax(precise=true): fp32 exp/sum, bf16 out               model.cpp:764
//       (sum order: lane-strided partials + xor butterfly, see orc_route)
//   argpartition top-k + take_along_axis                        model.cpp:767-775
//       ties broken toward the lower expert id (MLX leaves the order unspecified;
//       tests compare id *sets* and exclude near-ties)
//   norm_topk_prob: s / bf16(sum s)                             nemotron_h.cpp:1045-1048
//       (parsed at model.cpp:138 but not applied by LlamaModel::moe_block; the
//        Qwen3/Mixtral-shaped configs of the benchmark ask for it)
//   switch_mlp: sort iff T*k >= 64 (stable argsort of flat ids), take, 3x gather_qmm,
//       compiled swiglu silu(g)*u, unsort                      model.cpp:673-734, 14-25
//   combine: y = bf16( sum_k bf16(d * score) )                  model.cpp:780-784
//   shared expert + sigmoid gate + add                          model.cpp:736-748, 786-804
//
// Every fp32 sum runs in a fixed order (8 interleaved partial sums, combined
// pairwise), so the oracle is deterministic for a given input.
#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <numeric>
#include <thread>
#include <vector>

namespace {

inline float bf2f(uint16_t b) {
  uint32_t u = static_cast<uint32_t>(b) << 16;
  float f;
  std::memcpy(&f, &u, 4);
  return f;
}

inline uint16_t f2bf(float f) {  // round to nearest even, NaN kept quiet
  uint32_t u;
  std::memcpy(&u, &f, 4);
  if ((u & 0x7fffffffu) > 0x7f800000u) return static_cast<uint16_t>((u >> 16) | 0x40);
  u += 0x7fffu + ((u >> 16) & 1u);
  return static_cast<uint16_t>(u >> 16);
}

inline float rbf(float f) { return bf2f(f2bf(f)); }

inline float sigmoidf(float v) { return 1.0f / (1.0f + std::exp(-v)); }

template <class F>
void parallel_for(int64_t n, int nthreads, F&& fn) {
  if (n <= 0) return;
  if (nthreads <= 1 || n == 1) {
    fn(int64_t(0), n);
    return;
  }
  int64_t nt = std::min<int64_t>(nthreads, n);
  std::vector<std::thread> th;
  th.reserve(nt);
  for (int64_t i = 0; i < nt; ++i) {
    int64_t lo = n * i / nt, hi = n * (i + 1) / nt;
    th.emplace_back([&fn, lo, hi] { fn(lo, hi); });
  }
  for (auto& t : th) t.join();
}

// fixed-order fp32 dot product: 8 interleaved partial sums, pairwise combine
inline float dot(const float* a, const float* b, int K) {
  float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  int j = 0;
  for (; j + 8 <= K; j += 8)
    for (int l = 0; l < 8; ++l) acc[l] += a[j + l] * b[j + l];
  for (; j < K; ++j) acc[j & 7] += a[j] * b[j];
  float s0 = acc[0] + acc[4], s1 = acc[1] + acc[5], s2 = acc[2] + acc[6], s3 = acc[3] + acc[7];
  return (s0 + s2) + (s1 + s3);
}

// Weight rounding mode: 0 = exact fp32 dequantization (MLX's documented arithmetic),
// 1 = dequantized weights rounded once to bf16, as a bf16 tensor-core path must
// (MLX's Metal qmm likewise dequantizes into bf16 threadgroup tiles).
int g_weight_rounding = 0;

// One row of an MLX affine-quantized matrix, dequantized in fp32 (fma(s, q, b)).
void dequant_row(const uint32_t* wrow, const uint16_t* srow, const uint16_t* brow, int K,
                 int gs, int bits, float* out) {
  const int pf = 32 / bits;
  const uint32_t mask = (bits == 32) ? 0xffffffffu : ((1u << bits) - 1u);
  const bool round_w = g_weight_rounding == 1;
  for (int g = 0; g < K / gs; ++g) {
    const float s = bf2f(srow[g]);
    const float b = brow ? bf2f(brow[g]) : 0.0f;
    for (int j = g * gs; j < (g + 1) * gs; ++j) {
      uint32_t q = (wrow[j / pf] >> ((j % pf) * bits)) & mask;
      const float w = std::fma(s, static_cast<float>(q), b);
      out[j] = round_w ? rbf(w) : w;
    }
  }
}

void to_float(const uint16_t* src, int64_t n, float* dst) {
  for (int64_t i = 0; i < n; ++i) dst[i] = bf2f(src[i]);
}

bool valid_quant(int K, int gs, int bits) {
  if (!(bits == 2 || bits == 4 || bits == 8)) return false;
  if (!(gs == 32 || gs == 64 || gs == 128)) return false;
  return K > 0 && K % gs == 0;
}

struct QMat {  // one (possibly stacked) affine-quantized matrix [E, N, K]
  const uint32_t* w;
  const uint16_t* s;
  const uint16_t* b;
  int N, K, gs, bits;
  const uint32_t* wrow(int e, int n) const {
    return w + (static_cast<int64_t>(e) * N + n) * (K / (32 / bits));
  }
  const uint16_t* srow(int e, int n) const { return s + (static_cast<int64_t>(e) * N + n) * (K / gs); }
  const uint16_t* brow(int e, int n) const {
    return b ? b + (static_cast<int64_t>(e) * N + n) * (K / gs) : nullptr;
  }
};

// out[r, n] = bf16(xrows[r] . w_hat[e, n]) for the listed rows, all with expert e.
// xf: fp32 copies of the input rows [R, K]; out: fp32 holding bf16 values [R, N].
void grouped_rows(const QMat& m, int e, const float* xf, int R, float* out, int n_lo, int n_hi) {
  std::vector<float> wrow(m.K);
  for (int n = n_lo; n < n_hi; ++n) {
    dequant_row(m.wrow(e, n), m.srow(e, n), m.brow(e, n), m.K, m.gs, m.bits, wrow.data());
    for (int r = 0; r < R; ++r) out[static_cast<int64_t>(r) * m.N + n] = rbf(dot(xf + static_cast<int64_t>(r) * m.K, wrow.data(), m.K));
  }
}

}  // namespace

extern "C" {

// Layout mirrors of the product's config / weight structs, declared independently.
struct orc_qweight {
  const uint32_t* w;
  const uint16_t* s;
  const uint16_t* b;
};

struct orc_moe_config {
  int hidden;                 // H
  int inter;                  // I (moe_intermediate_size)
  int num_experts;            // E
  int top_k;                  // k
  int group_size;             // 64
  int bits;                   // 4
  int norm_topk_prob;         // renormalise the top-k scores
  int shared_inter;           // Is, 0 = no shared expert
  int router_quantized;       // router weight is affine-quantized
  int shared_gate_quantized;  // shared_expert_gate weight is affine-quantized
};

struct orc_moe_weights {
  const void* router_w;  // [E, H] bf16, or [E, H/pf] u32 when quantized
  const uint16_t* router_s;
  const uint16_t* router_b;
  orc_qweight gate, up, down;                       // stacked [E, I, H], [E, I, H], [E, H, I]
  orc_qweight shared_gate, shared_up, shared_down;  // [Is, H], [Is, H], [H, Is]
  const void* shared_expert_gate_w;                 // [1, H] bf16 (or packed)
  const uint16_t* shared_expert_gate_s;
  const uint16_t* shared_expert_gate_b;
  const uint16_t* router_bias;  // [E] bf16 additive logit bias (benchmark load skew), nullable
};

int orc_version() { return 2; }

// 0: exact dequantization (default); 1: dequantized weights rounded to bf16.
int orc_set_weight_rounding(int mode) {
  if (mode != 0 && mode != 1) return 1;
  g_weight_rounding = mode;
  return 0;
}

// mx::quantized_matmul(x, w, s, b, transpose=true, gs, bits), x [M, K] -> out [M, N]
int orc_quantized_matmul(const uint16_t* x, int64_t M, int K, const uint32_t* w, const uint16_t* s,
                         const uint16_t* b, int N, int gs, int bits, uint16_t* out, int nthreads) {
  if (!valid_quant(K, gs, bits) || M < 0 || N <= 0) return 1;
  std::vector<float> xf(static_cast<size_t>(M) * K);
  to_float(x, M * K, xf.data());
  std::vector<float> of(static_cast<size_t>(M) * N);
  QMat m{w, s, b, N, K, gs, bits};
  parallel_for(N, nthreads, [&](int64_t lo, int64_t hi) {
    grouped_rows(m, 0, xf.data(), static_cast<int>(M), of.data(), static_cast<int>(lo), static_cast<int>(hi));
  });
  for (int64_t i = 0; i < M * N; ++i) out[i] = f2bf(of[i]);
  return 0;
}

// mx::gather_qmm(x, w, s, b, lhs, rhs, transpose=true, gs, bits):
// x [xb, M, K]; w [E, N, K/pf]; out [B, M, N]; out[i] = x[lhs(i)] @ w_hat[rhs[i]]^T.
// lhs == NULL means the x batch broadcasts against rhs: lhs(i) = i * xb / B.
int orc_gather_qmm(const uint16_t* x, int64_t xb, int M, int K, const uint32_t* w, const uint16_t* s,
                   const uint16_t* b, int E, int N, const uint32_t* lhs, const uint32_t* rhs, int64_t B,
                   int gs, int bits, uint16_t* out, int nthreads) {
  if (!valid_quant(K, gs, bits) || B < 0 || xb <= 0 || M <= 0 || E <= 0) return 1;
  if (!lhs && B % xb != 0) return 1;
  std::vector<std::vector<int64_t>> by_e(E);
  for (int64_t i = 0; i < B; ++i) {
    if (rhs[i] >= static_cast<uint32_t>(E)) return 1;
    int64_t xi = lhs ? lhs[i] : i * xb / B;
    if (xi < 0 || xi >= xb) return 1;
    by_e[rhs[i]].push_back(i);
  }
  QMat m{w, s, b, N, K, gs, bits};
  parallel_for(E, nthreads, [&](int64_t lo, int64_t hi) {
    for (int64_t e = lo; e < hi; ++e) {
      const auto& lst = by_e[e];
      if (lst.empty()) continue;
      const int R = static_cast<int>(lst.size()) * M;
      std::vector<float> xf(static_cast<size_t>(R) * K), of(static_cast<size_t>(R) * N);
      for (size_t r = 0; r < lst.size(); ++r) {
        int64_t xi = lhs ? lhs[lst[r]] : lst[r] * xb / B;
        to_float(x + xi * M * K, static_cast<int64_t>(M) * K, xf.data() + r * M * K);
      }
      grouped_rows(m, static_cast<int>(e), xf.data(), R, of.data(), 0, N);
      for (size_t r = 0; r < lst.size(); ++r)
        for (int64_t i = 0; i < static_cast<int64_t>(M) * N; ++i)
          out[lst[r] * M * N + i] = f2bf(of[r * M * N + i]);
    }
  });
  return 0;
}

// Router: logits (bf16), softmax(precise) probs (bf16), top-k ids / scores.
// ids are ordered by descending probability, ties toward the lower expert id.
// router_bias (nullable, bf16 [E]) is added to the bf16 logits and rounded again; it is
// not part of the reference's router and only skews the load for the Mixtral-shaped
// benchmark configuration.
int orc_route(const uint16_t* x, int64_t T, int H, const void* router_w, const uint16_t* router_s,
              const uint16_t* router_b, int router_quantized, const uint16_t* router_bias, int E, int k,
              int norm_topk, int gs, int bits, int32_t* ids, uint16_t* scores, uint16_t* logits_out,
              uint16_t* probs_out, int nthreads) {
  if (T < 0 || E <= 0 || k <= 0 || k > E) return 1;
  std::vector<uint16_t> logits(static_cast<size_t>(T) * E);
  if (router_quantized) {
    int rc = orc_quantized_matmul(x, T, H, static_cast<const uint32_t*>(router_w), router_s, router_b,
                                  E, gs, bits, logits.data(), nthreads);
    if (rc) return rc;
  } else {
    std::vector<float> wf(static_cast<size_t>(E) * H);
    to_float(static_cast<const uint16_t*>(router_w), static_cast<int64_t>(E) * H, wf.data());
    parallel_for(T, nthreads, [&](int64_t lo, int64_t hi) {
      std::vector<float> xf(H);
      for (int64_t t = lo; t < hi; ++t) {
        to_float(x + t * H, H, xf.data());
        for (int e = 0; e < E; ++e) logits[t * E + e] = f2bf(dot(xf.data(), wf.data() + static_cast<int64_t>(e) * H, H));
      }
    });
  }
  if (router_bias)
    for (int64_t t = 0; t < T; ++t)
      for (int e = 0; e < E; ++e) logits[t * E + e] = f2bf(bf2f(logits[t * E + e]) + bf2f(router_bias[e]));
  parallel_for(T, nthreads, [&](int64_t lo, int64_t hi) {
    std::vector<float> p(E);
    std::vector<int> order(E);
    for (int64_t t = lo; t < hi; ++t) {
      const uint16_t* l = logits.data() + t * E;
      float mx = -INFINITY;
      for (int e = 0; e < E; ++e) mx = std::max(mx, bf2f(l[e]));
      // softmax sum order: 32 lane-strided partial sums (e = l, l+32, ...), then an xor
      // butterfly over the partials (16, 8, 4, 2, 1).  MLX leaves the order unspecified;
      // this one is the device kernel's warp reduction, so both round identically.
      float lane_sum[32] = {0};
      for (int e = 0; e < E; ++e) {
        p[e] = std::exp(bf2f(l[e]) - mx);
        lane_sum[e & 31] += p[e];
      }
      for (int off = 16; off > 0; off >>= 1) {
        float nxt[32];
        for (int q = 0; q < 32; ++q) nxt[q] = lane_sum[q] + lane_sum[q ^ off];
        std::memcpy(lane_sum, nxt, sizeof(lane_sum));
      }
      const float sum = lane_sum[0];
      for (int e = 0; e < E; ++e) p[e] = rbf(p[e] / sum);
      if (logits_out) std::memcpy(logits_out + t * E, l, E * sizeof(uint16_t));
      if (probs_out)
        for (int e = 0; e < E; ++e) probs_out[t * E + e] = f2bf(p[e]);
      std::iota(order.begin(), order.end(), 0);
      std::stable_sort(order.begin(), order.end(), [&](int a, int b) { return p[a] > p[b]; });
      float denom = 1.0f;
      if (norm_topk) {
        float s = 0.0f;
        for (int j = 0; j < k; ++j) s += p[order[j]];
        denom = rbf(s);
      }
      for (int j = 0; j < k; ++j) {
        ids[t * k + j] = order[j];
        float sc = p[order[j]];
        scores[t * k + j] = f2bf(norm_topk ? sc / denom : sc);
      }
    }
  });
  return 0;
}

// Stable expert-major permutation of the T*k routed pairs (argsort of flat ids,
// model.cpp:688-700).  sorted_token[p] = flat_index / k, sorted_slot[p] = flat_index,
// offsets[E+1] = start of each expert's segment.
int orc_sort_pairs(const int32_t* ids, int64_t T, int k, int E, int32_t* sorted_token,
                   int32_t* sorted_flat, int32_t* offsets) {
  const int64_t P = T * k;
  std::vector<int64_t> cnt(E + 1, 0);
  for (int64_t i = 0; i < P; ++i) {
    if (ids[i] < 0 || ids[i] >= E) return 1;
    cnt[ids[i] + 1]++;
  }
  for (int e = 0; e < E; ++e) cnt[e + 1] += cnt[e];
  if (offsets)
    for (int e = 0; e <= E; ++e) offsets[e] = static_cast<int32_t>(cnt[e]);
  std::vector<int64_t> pos(cnt.begin(), cnt.end() - 1);
  for (int64_t i = 0; i < P; ++i) {  // ascending flat index == stable argsort
    int64_t p = pos[ids[i]]++;
    if (sorted_token) sorted_token[p] = static_cast<int32_t>(i / k);
    if (sorted_flat) sorted_flat[p] = static_cast<int32_t>(i);
  }
  return 0;
}

// Full MoE block (LlamaModel::moe_block, model.cpp:750-807) for x [T, H] -> y [T, H].
// forced_ids / forced_scores (nullable) replace the router's choice, so that a test can
// evaluate the experts on the routing another implementation produced.
int orc_moe_block(const orc_moe_config* cfg, const orc_moe_weights* wt, const uint16_t* x, int64_t T,
                  const int32_t* forced_ids, const uint16_t* forced_scores, uint16_t* y,
                  int32_t* ids_out, uint16_t* scores_out, int nthreads) {
  const int H = cfg->hidden, I = cfg->inter, E = cfg->num_experts, k = cfg->top_k;
  const int gs = cfg->group_size, bits = cfg->bits;
  if (!valid_quant(H, gs, bits) || !valid_quant(I, gs, bits) || k <= 0 || k > E || T < 0) return 1;
  const int64_t P = T * k;
  std::vector<int32_t> ids(P);
  std::vector<uint16_t> scores(P);
  if (forced_ids) {
    std::memcpy(ids.data(), forced_ids, P * sizeof(int32_t));
    std::memcpy(scores.data(), forced_scores, P * sizeof(uint16_t));
  } else {
    int rc = orc_route(x, T, H, wt->router_w, wt->router_s, wt->router_b, cfg->router_quantized,
                       wt->router_bias, E, k, cfg->norm_topk_prob, gs, bits, ids.data(), scores.data(),
                       nullptr, nullptr, nthreads);
    if (rc) return rc;
  }
  if (ids_out) std::memcpy(ids_out, ids.data(), P * sizeof(int32_t));
  if (scores_out) std::memcpy(scores_out, scores.data(), P * sizeof(uint16_t));

  // switch_mlp (model.cpp:673-734).  do_sort = indices.size() >= 64 (model.cpp:683):
  // the sorted path visits pairs in stable expert-major order and unsorts afterwards;
  // the unsorted path visits them in (token, slot) order.  Each pair's arithmetic is
  // identical, so both produce the same d[t, j].
  std::vector<int32_t> sorted_token(P), sorted_flat(P), offsets(E + 1);
  const bool do_sort = P >= 64;
  if (do_sort) {
    if (orc_sort_pairs(ids.data(), T, k, E, sorted_token.data(), sorted_flat.data(), offsets.data())) return 1;
  } else {
    for (int64_t i = 0; i < P; ++i)
      if (ids[i] < 0 || ids[i] >= E) return 1;
  }
  QMat mg{wt->gate.w, wt->gate.s, wt->gate.b, I, H, gs, bits};
  QMat mu{wt->up.w, wt->up.s, wt->up.b, I, H, gs, bits};
  QMat md{wt->down.w, wt->down.s, wt->down.b, H, I, gs, bits};
  std::vector<float> d_pair(static_cast<size_t>(P) * H);  // d[flat pair] (bf16 values)
  std::vector<float> xf(static_cast<size_t>(T) * H);
  to_float(x, T * H, xf.data());

  auto expert_mlp = [&](const QMat& g, const QMat& u, const QMat& dn, int e, const int32_t* rows, int R,
                        float* out_rows /* [R, H] */) {
    const int Ie = g.N;
    std::vector<float> xr(static_cast<size_t>(R) * H), gv(static_cast<size_t>(R) * Ie),
        uv(static_cast<size_t>(R) * Ie);
    for (int r = 0; r < R; ++r) std::memcpy(&xr[static_cast<size_t>(r) * H], &xf[static_cast<size_t>(rows[r]) * H], H * sizeof(float));
    grouped_rows(g, e, xr.data(), R, gv.data(), 0, Ie);
    grouped_rows(u, e, xr.data(), R, uv.data(), 0, Ie);
    // compiled swiglu (model.cpp:14-25): multiply(multiply(g, sigmoid(g)), u), bf16 per op
    for (int64_t i = 0; i < static_cast<int64_t>(R) * Ie; ++i) {
      float gg = gv[i];
      float sg = rbf(sigmoidf(gg));
      float h = rbf(gg * sg);
      gv[i] = rbf(h * uv[i]);
    }
    grouped_rows(dn, e, gv.data(), R, out_rows, 0, H);
  };

  if (do_sort) {
    parallel_for(E, nthreads, [&](int64_t lo, int64_t hi) {
      for (int64_t e = lo; e < hi; ++e) {
        int a = offsets[e], bnd = offsets[e + 1];
        if (a == bnd) continue;
        std::vector<float> dv(static_cast<size_t>(bnd - a) * H);
        expert_mlp(mg, mu, md, static_cast<int>(e), sorted_token.data() + a, bnd - a, dv.data());
        for (int p = a; p < bnd; ++p)  // unsort: take(x_down, inv_order)
          std::memcpy(&d_pair[static_cast<size_t>(sorted_flat[p]) * H], &dv[static_cast<size_t>(p - a) * H], H * sizeof(float));
      }
    });
  } else {  // unsorted gather_qmm: one (token, slot) pair at a time
    parallel_for(P, nthreads, [&](int64_t lo, int64_t hi) {
      for (int64_t i = lo; i < hi; ++i) {
        int32_t t = static_cast<int32_t>(i / k);
        expert_mlp(mg, mu, md, ids[i], &t, 1, &d_pair[static_cast<size_t>(i) * H]);
      }
    });
  }

  // weighted combine (model.cpp:780-784): bf16(d * score), fp32 sum over k, bf16
  std::vector<float> yr(static_cast<size_t>(T) * H);
  parallel_for(T, nthreads, [&](int64_t lo, int64_t hi) {
    for (int64_t t = lo; t < hi; ++t)
      for (int h = 0; h < H; ++h) {
        float acc = 0.0f;
        for (int j = 0; j < k; ++j) acc += rbf(d_pair[static_cast<size_t>(t * k + j) * H + h] * bf2f(scores[t * k + j]));
        yr[t * H + h] = rbf(acc);
      }
  });

  if (cfg->shared_inter > 0) {  // shared expert (model.cpp:736-748, 786-804)
    const int Is = cfg->shared_inter;
    if (!valid_quant(Is, gs, bits)) return 1;
    QMat sg{wt->shared_gate.w, wt->shared_gate.s, wt->shared_gate.b, Is, H, gs, bits};
    QMat su{wt->shared_up.w, wt->shared_up.s, wt->shared_up.b, Is, H, gs, bits};
    QMat sd{wt->shared_down.w, wt->shared_down.s, wt->shared_down.b, H, Is, gs, bits};
    std::vector<float> sh(static_cast<size_t>(T) * H);
    const int64_t chunk = 512;
    const int64_t nchunk = (T + chunk - 1) / chunk;
    // parallel over row blocks of the shared matrices, tokens in chunks
    for (int64_t c = 0; c < nchunk; ++c) {
      const int64_t t0 = c * chunk, R = std::min<int64_t>(chunk, T - t0);
      std::vector<float> gv(static_cast<size_t>(R) * Is), uv(static_cast<size_t>(R) * Is);
      const float* xr = xf.data() + t0 * H;
      parallel_for(Is, nthreads, [&](int64_t lo, int64_t hi) {
        grouped_rows(sg, 0, xr, static_cast<int>(R), gv.data(), static_cast<int>(lo), static_cast<int>(hi));
        grouped_rows(su, 0, xr, static_cast<int>(R), uv.data(), static_cast<int>(lo), static_cast<int>(hi));
      });
      for (int64_t i = 0; i < R * Is; ++i) {
        float gg = gv[i];
        float sgm = rbf(sigmoidf(gg));
        gv[i] = rbf(rbf(gg * sgm) * uv[i]);
      }
      parallel_for(H, nthreads, [&](int64_t lo, int64_t hi) {
        grouped_rows(sd, 0, gv.data(), static_cast<int>(R), sh.data() + t0 * H, static_cast<int>(lo), static_cast<int>(hi));
      });
    }
    // gate_val = sigmoid(x @ wg^T) (bf16 matmul or quantized_matmul), [T, 1]
    std::vector<float> gl(T);
    if (cfg->shared_gate_quantized) {
      std::vector<uint16_t> o(T);
      int rc = orc_quantized_matmul(x, T, H, static_cast<const uint32_t*>(wt->shared_expert_gate_w),
                                    wt->shared_expert_gate_s, wt->shared_expert_gate_b, 1, gs, bits, o.data(), nthreads);
      if (rc) return rc;
      for (int64_t t = 0; t < T; ++t) gl[t] = bf2f(o[t]);
    } else {
      std::vector<float> wg(H);
      to_float(static_cast<const uint16_t*>(wt->shared_expert_gate_w), H, wg.data());
      for (int64_t t = 0; t < T; ++t) gl[t] = rbf(dot(xf.data() + t * H, wg.data(), H));
    }
    for (int64_t t = 0; t < T; ++t) {
      float gv = rbf(sigmoidf(gl[t]));
      for (int h = 0; h < H; ++h) yr[t * H + h] = rbf(yr[t * H + h] + rbf(gv * sh[t * H + h]));
    }
  }
  for (int64_t i = 0; i < T * H; ++i) y[i] = f2bf(yr[i]);
  return 0;
}


// ------------------------------------------------------------------ sigmoid-routed variant
// The Nemotron-H / DeepSeek-style MoE block (server/src/nemotron_h.cpp:1010-1100):
//   logits  = bf16(x @ Wr^T)                                   (1018)
//   orig    = sigmoid(fp32(logits)); sel = orig + correction    (1025-1029)
//   n_group > 1: group score = sum of the group's top-2 sel; the n_group - topk_group
//            lowest groups get sel = 0                           (1030-1041)
//   top-k of sel (ties -> lower id), scores = orig of the picks  (1043-1045)
//   norm_topk_prob and k > 1: s / (sum s + 1e-20)               (1046-1049)
//   s *= routed_scaling_factor                                  (1050)
//   experts: h = fc2(relu2(fc1(x))), relu2 = bf16(max(x,0)^2)   (1053-1091, 53-58)
//   y = bf16( sum_k fp32(h_k) * s_k )                           (1094-1095)
//   shared (ungated): y = bf16(y + down(relu2(up(x))))          (1098-1106)
// MLX leaves argpartition's order and the score sums' order unspecified; here the picks
// are in selection order (highest sel first) and sums run in that order; equal group
// scores zero the higher group id first.
struct orc_sig_config {
  int hidden, inter, num_experts, top_k, group_size, bits;
  int norm_topk_prob;
  int shared_inter;  // ungated shared expert (up -> relu2 -> down), 0 = none
  int n_group, topk_group;
  float routed_scaling_factor;
};

struct orc_sig_weights {
  const uint16_t* router_w;      // [E, H] bf16
  const float* correction_bias;  // [E] fp32, nullable
  orc_qweight fc1, fc2;          // [E, I, H], [E, H, I]
  orc_qweight shared_up, shared_down;
};

int orc_route_sigmoid(const uint16_t* x, int64_t T, int H, const uint16_t* router_w, const float* correction_bias,
                      int E, int k, int n_group, int topk_group, int norm_topk, float scale, int32_t* ids,
                      float* scores, int nthreads) {
  if (T < 0 || E <= 0 || k <= 0 || k > E || n_group <= 0 || E % n_group || topk_group <= 0 ||
      topk_group > n_group)
    return 1;
  const int gsz = E / n_group;
  if (n_group > 1 && gsz < 2) return 1;
  std::vector<float> wf(static_cast<size_t>(E) * H);
  to_float(router_w, static_cast<int64_t>(E) * H, wf.data());
  parallel_for(T, nthreads, [&](int64_t lo, int64_t hi) {
    std::vector<float> xf(H), orig(E), sel(E), gscore(n_group);
    std::vector<int> order(E), gorder(n_group);
    for (int64_t t = lo; t < hi; ++t) {
      to_float(x + t * H, H, xf.data());
      for (int e = 0; e < E; ++e) {
        const float l = rbf(dot(xf.data(), wf.data() + static_cast<int64_t>(e) * H, H));
        orig[e] = 1.0f / (1.0f + std::exp(-l));
        sel[e] = correction_bias ? orig[e] + correction_bias[e] : orig[e];
      }
      if (n_group > 1) {
        for (int gi = 0; gi < n_group; ++gi) {
          float m1 = -INFINITY, m2 = -INFINITY;
          for (int e = gi * gsz; e < (gi + 1) * gsz; ++e) {
            if (sel[e] > m1) {
              m2 = m1;
              m1 = sel[e];
            } else if (sel[e] > m2) {
              m2 = sel[e];
            }
          }
          gscore[gi] = m1 + m2;
        }
        std::iota(gorder.begin(), gorder.end(), 0);
        // lowest scores first; among equal ones the higher group id first
        std::sort(gorder.begin(), gorder.end(), [&](int a, int b) {
          return gscore[a] != gscore[b] ? gscore[a] < gscore[b] : a > b;
        });
        for (int z = 0; z < n_group - topk_group; ++z)
          for (int e = gorder[z] * gsz; e < (gorder[z] + 1) * gsz; ++e) sel[e] = 0.0f;
      }
      std::iota(order.begin(), order.end(), 0);
      std::stable_sort(order.begin(), order.end(), [&](int a, int b) { return sel[a] > sel[b]; });
      float denom = 1.0f;
      if (norm_topk && k > 1) {
        float s = 0.0f;
        for (int j = 0; j < k; ++j) s += orig[order[j]];
        denom = s + 1e-20f;
      }
      for (int j = 0; j < k; ++j) {
        ids[t * k + j] = order[j];
        const float sc = (norm_topk && k > 1) ? orig[order[j]] / denom : orig[order[j]];
        scores[t * k + j] = sc * scale;
      }
    }
  });
  return 0;
}

int orc_moe_block_sigmoid(const orc_sig_config* cfg, const orc_sig_weights* wt, const uint16_t* x, int64_t T,
                          const int32_t* forced_ids, const float* forced_scores, uint16_t* y, int32_t* ids_out,
                          float* scores_out, int nthreads) {
  const int H = cfg->hidden, I = cfg->inter, E = cfg->num_experts, k = cfg->top_k;
  const int gs = cfg->group_size, bits = cfg->bits;
  if (!valid_quant(H, gs, bits) || !valid_quant(I, gs, bits) || k <= 0 || k > E || T < 0) return 1;
  const int64_t P = T * k;
  std::vector<int32_t> ids(P);
  std::vector<float> scores(P);
  if (forced_ids) {
    std::memcpy(ids.data(), forced_ids, P * sizeof(int32_t));
    std::memcpy(scores.data(), forced_scores, P * sizeof(float));
  } else {
    int rc = orc_route_sigmoid(x, T, H, wt->router_w, wt->correction_bias, E, k, cfg->n_group, cfg->topk_group,
                               cfg->norm_topk_prob, cfg->routed_scaling_factor, ids.data(), scores.data(), nthreads);
    if (rc) return rc;
  }
  for (int64_t i = 0; i < P; ++i)
    if (ids[i] < 0 || ids[i] >= E) return 1;
  if (ids_out) std::memcpy(ids_out, ids.data(), P * sizeof(int32_t));
  if (scores_out) std::memcpy(scores_out, scores.data(), P * sizeof(float));
  QMat m1{wt->fc1.w, wt->fc1.s, wt->fc1.b, I, H, gs, bits};
  QMat m2{wt->fc2.w, wt->fc2.s, wt->fc2.b, H, I, gs, bits};
  std::vector<float> xf(static_cast<size_t>(T) * H);
  to_float(x, T * H, xf.data());
  // per (token, slot) pair: h = fc2(relu2(fc1(x))); every pair's arithmetic is the same in
  // the sorted and unsorted gather_qmm paths
  std::vector<float> d_pair(static_cast<size_t>(P) * H);
  parallel_for(P, nthreads, [&](int64_t lo, int64_t hi) {
    std::vector<float> u(I);
    for (int64_t i = lo; i < hi; ++i) {
      const float* xr = xf.data() + (i / k) * H;
      grouped_rows(m1, ids[i], xr, 1, u.data(), 0, I);
      for (int n = 0; n < I; ++n) {
        const float r = std::max(u[n], 0.0f);
        u[n] = rbf(r * r);
      }
      grouped_rows(m2, ids[i], u.data(), 1, &d_pair[static_cast<size_t>(i) * H], 0, H);
    }
  });
  std::vector<float> yr(static_cast<size_t>(T) * H);
  for (int64_t t = 0; t < T; ++t)
    for (int h = 0; h < H; ++h) {
      float acc = 0.0f;
      for (int j = 0; j < k; ++j) acc += d_pair[static_cast<size_t>(t * k + j) * H + h] * scores[t * k + j];
      yr[t * H + h] = rbf(acc);
    }
  if (cfg->shared_inter > 0) {
    const int Is = cfg->shared_inter;
    if (!valid_quant(Is, gs, bits)) return 1;
    QMat su{wt->shared_up.w, wt->shared_up.s, wt->shared_up.b, Is, H, gs, bits};
    QMat sd{wt->shared_down.w, wt->shared_down.s, wt->shared_down.b, H, Is, gs, bits};
    parallel_for(T, nthreads, [&](int64_t lo, int64_t hi) {
      std::vector<float> u(Is), sh(H);
      for (int64_t t = lo; t < hi; ++t) {
        grouped_rows(su, 0, xf.data() + t * H, 1, u.data(), 0, Is);
        for (int n = 0; n < Is; ++n) {
          const float r = std::max(u[n], 0.0f);
          u[n] = rbf(r * r);
        }
        grouped_rows(sd, 0, u.data(), 1, sh.data(), 0, H);
        for (int h = 0; h < H; ++h) yr[t * H + h] = rbf(yr[t * H + h] + sh[h]);
      }
    });
  }
  for (int64_t i = 0; i < T * H; ++i) y[i] = f2bf(yr[i]);
  return 0;
}

}  // extern "C"
