// qgemv.cu -- small-batch expert products: 4-bit affine dequant GEMV on the legacy
// tensor pipe (mma.sync m16n8k16), for decode-sized batches (few tokens per expert).
//
// Replaces mx::gather_qmm / mx::quantized_matmul for the decode path
// (model.cpp:703-721, 741-747; decode reaches them with T*k < 64 unsorted, or sorted
// with a handful of tokens per expert).  The kernel is HBM-bound: every weight byte
// of an active expert is read once with 128-bit loads; inactive experts are never
// touched.
//
// Work unit (one CTA of 4 warps): an output-row block x a chunk of <= 32 activation
// rows x an optional K split.  Warp w owns two 16-row MMA tiles:
//   gate/up mode: gate rows [64 rb + 16 w, +16) and the same up rows (SwiGLU in regs)
//   down / plain: rows [128 rb + 32 w, +16) and [.. + 16, +16)
// Lane (g = lane/4, c = lane%4) loads 16 bytes (32 codes) of rows g and g+8 per
// 128-wide K chunk; code pairs (q_i, q_{i+4}) become bf16x2 A fragments directly,
// and the activation rows are stored with the matching within-8 pair permutation,
// so each B fragment is one 32-bit word of a 16-byte load.
#include "fm_internal.cuh"

namespace fm {

namespace {

constexpr int kGvThreads = 128;
constexpr int kGvMaxNT = 4;  // 8-token MMA column tiles per work unit

FM_DEV uint32_t word_of(const uint4& v, int i) {
  return i == 0 ? v.x : (i == 1 ? v.y : (i == 2 ? v.z : v.w));
}

FM_DEV __nv_bfloat162 bf2_splat(uint16_t b) {
  const uint32_t u = static_cast<uint32_t>(b) * 0x10001u;
  return *reinterpret_cast<const __nv_bfloat162*>(&u);
}

FM_DEV float swiglu1(float g, float u) {  // model.cpp:14-25, bf16 rounding per op
  const float gs = rbf(sigmoid_f(g));
  const float h = rbf(g * gs);
  return rbf(h * u);
}

}  // namespace

template <int MODE>
__global__ void __launch_bounds__(kGvThreads) qgemv_kernel(const GemmArgs a) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, c = lane & 3;
  const TileTable* tab = a.tab;
  if (*reinterpret_cast<volatile uint32_t*>(a.err) != 0u) return;  // an earlier kernel failed
  const int ntiles = tab->num_tiles;
  for (int tile = blockIdx.x; tile < ntiles; tile += gridDim.x) {
    const TileInfo ti = decode_tile(tab, tile);
    const bool sh = ti.expert < 0;
    const int K = (MODE == MODE_DOWN && sh) ? a.K_shared : a.K;
    const int N = sh ? a.N_shared : a.N;
    const int kw = K / 8;        // u32 words per weight row
    const int gpr = K / a.gs;    // quant groups per row
    const int64_t erow = sh ? 0 : static_cast<int64_t>(ti.expert) * N;

    const uint32_t* Wm[2];
    const uint16_t* Sm[2];
    const uint16_t* Bm[2];
    int r0[2];
    if (MODE == MODE_GATEUP) {
      Wm[0] = sh ? a.sw0 : a.w0; Sm[0] = sh ? a.ss0 : a.s0; Bm[0] = sh ? a.sb0 : a.b0;
      Wm[1] = sh ? a.sw1 : a.w1; Sm[1] = sh ? a.ss1 : a.s1; Bm[1] = sh ? a.sb1 : a.b1;
      r0[0] = r0[1] = ti.rb * 64 + warp * 16;
    } else {
      Wm[0] = Wm[1] = sh ? a.sw0 : a.w0;
      Sm[0] = Sm[1] = sh ? a.ss0 : a.s0;
      Bm[0] = Bm[1] = sh ? a.sb0 : a.b0;
      r0[0] = ti.rb * 128 + warp * 32;
      r0[1] = r0[0] + 16;
    }
    const bool mval0 = r0[0] < N, mval1 = r0[1] < N;  // N % 16 == 0 (host-checked)

    const uint32_t* wrow[2][2];
    const uint16_t* srow[2][2];
    const uint16_t* brow[2][2];
#pragma unroll
    for (int m = 0; m < 2; ++m)
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int64_t r = erow + min(r0[m] + g + 8 * h, N - 1);
        wrow[m][h] = Wm[m] + r * kw;
        srow[m][h] = Sm[m] + r * gpr;
        brow[m][h] = Bm[m] ? Bm[m] + r * gpr : nullptr;
      }

    // activation rows of the chunk: n-tile j, column g -> slot 8j + g
    const int nt = (ti.nrows + 7) >> 3;
    const uint16_t* xrow[kGvMaxNT];
#pragma unroll
    for (int j = 0; j < kGvMaxNT; ++j) {
      const int slot = 8 * j + g;
      xrow[j] = nullptr;
      if (j < nt && slot < ti.nrows) {
        const int p = ti.row0 + slot;
        int64_t src;
        const uint16_t* base;
        int64_t ld;
        if (MODE == MODE_DOWN) {
          src = p;
          base = sh ? a.act_shared : a.act;
          ld = sh ? a.act_shared_ld : a.act_ld;
        } else {
          src = sh ? p : a.sorted_token[p];
          base = sh ? a.act_shared : a.act;
          ld = sh ? a.act_shared_ld : a.act_ld;
        }
        xrow[j] = base + src * ld;
      }
    }

    const int kchunks = K / 128;
    const int kc0 = kchunks * ti.ks / ti.ksplit, kc1 = kchunks * (ti.ks + 1) / ti.ksplit;
    float acc[2][kGvMaxNT][4];
#pragma unroll
    for (int m = 0; m < 2; ++m)
#pragma unroll
      for (int j = 0; j < kGvMaxNT; ++j) acc[m][j][0] = acc[m][j][1] = acc[m][j][2] = acc[m][j][3] = 0.f;

    const uint4 z4 = make_uint4(0, 0, 0, 0);
    uint4 A[2][2];
#pragma unroll
    for (int m = 0; m < 2; ++m)
#pragma unroll
      for (int h = 0; h < 2; ++h)
        A[m][h] = (kc0 < kc1 && (m == 0 ? mval0 : mval1)) ? ldg_nc_v4(wrow[m][h] + kc0 * 16 + 4 * c) : z4;

    for (int kc = kc0; kc < kc1; ++kc) {
      // prefetch the next chunk's codes
      uint4 An[2][2];
      const bool more = kc + 1 < kc1;
#pragma unroll
      for (int m = 0; m < 2; ++m)
#pragma unroll
        for (int h = 0; h < 2; ++h)
          An[m][h] = (more && (m == 0 ? mval0 : mval1)) ? ldg_nc_v4(wrow[m][h] + (kc + 1) * 16 + 4 * c) : z4;
      // scales / biases of the group holding this lane's 32 codes
      const int grp = (kc * 128 + 32 * c) / a.gs;
      __nv_bfloat162 s2[2][2], b2[2][2];
#pragma unroll
      for (int m = 0; m < 2; ++m)
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          s2[m][h] = bf2_splat(__ldg(srow[m][h] + grp));
          b2[m][h] = bf2_splat(brow[m][h] ? __ldg(brow[m][h] + grp) : static_cast<uint16_t>(0));
        }
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        uint4 Bv[kGvMaxNT];
#pragma unroll
        for (int j = 0; j < kGvMaxNT; ++j)
          Bv[j] = xrow[j] ? __ldg(reinterpret_cast<const uint4*>(xrow[j] + kc * 128 + 32 * c + 8 * i)) : z4;
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
#pragma unroll
          for (int m = 0; m < 2; ++m) {
            if (!(m == 0 ? mval0 : mval1)) continue;
            const uint32_t wg = word_of(A[m][0], i), wg8 = word_of(A[m][1], i);
            const uint32_t a0 = deq_pair(wg, 2 * hh, s2[m][0], b2[m][0]);
            const uint32_t a1 = deq_pair(wg8, 2 * hh, s2[m][1], b2[m][1]);
            const uint32_t a2 = deq_pair(wg, 2 * hh + 1, s2[m][0], b2[m][0]);
            const uint32_t a3 = deq_pair(wg8, 2 * hh + 1, s2[m][1], b2[m][1]);
#pragma unroll
            for (int j = 0; j < kGvMaxNT; ++j)
              if (j < nt) mma_bf16_16816(acc[m][j], a0, a1, a2, a3, word_of(Bv[j], 2 * hh), word_of(Bv[j], 2 * hh + 1));
          }
        }
      }
#pragma unroll
      for (int m = 0; m < 2; ++m)
#pragma unroll
        for (int h = 0; h < 2; ++h) A[m][h] = An[m][h];
    }

    // epilogue: acc[m][j][e] is (row r0[m] + g + 8*(e>>1), slot 8j + 2c + (e&1))
#pragma unroll
    for (int j = 0; j < kGvMaxNT; ++j) {
      if (j >= nt) continue;
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int slot = 8 * j + 2 * c + (e & 1);
        if (slot >= ti.nrows) continue;
        const int p = ti.row0 + slot;
        if (MODE == MODE_GATEUP) {
          if (!mval0) continue;
          const int n = r0[0] + g + 8 * (e >> 1);
          const float gv = rbf(acc[0][j][e]), uv = rbf(acc[1][j][e]);
          uint16_t* out = sh ? a.out_shared + static_cast<int64_t>(p) * a.out_shared_ld
                             : a.out + static_cast<int64_t>(p) * a.out_ld;
          out[perm8(n)] = f2bf(swiglu1(gv, uv));
        } else {
#pragma unroll
          for (int m = 0; m < 2; ++m) {
            if (!(m == 0 ? mval0 : mval1)) continue;
            const int n = r0[m] + g + 8 * (e >> 1);
            const float v = acc[m][j][e];
            if (MODE == MODE_DOWN) {
              if (sh) {
                red_add_f32(a.ysh + static_cast<int64_t>(p) * a.y_ld + n, v);
              } else {
                const int t = a.sorted_token[p];
                red_add_f32(a.y_acc + static_cast<int64_t>(t) * a.y_ld + n, rbf(rbf(v) * a.sorted_score[p]));
              }
            } else {
              a.out[static_cast<int64_t>(a.sorted_flat[p]) * a.out_ld + n] = f2bf(v);
            }
          }
        }
      }
    }
  }
}

cudaError_t launch_qgemv(int mode, int grid, cudaStream_t stream, const GemmArgs& a) {
  switch (mode) {
    case MODE_GATEUP: qgemv_kernel<MODE_GATEUP><<<grid, kGvThreads, 0, stream>>>(a); break;
    case MODE_DOWN: qgemv_kernel<MODE_DOWN><<<grid, kGvThreads, 0, stream>>>(a); break;
    default: qgemv_kernel<MODE_PLAIN><<<grid, kGvThreads, 0, stream>>>(a); break;
  }
  return cudaGetLastError();
}

cudaError_t qgemv_blocks_per_sm(int* n) {
  return cudaOccupancyMaxActiveBlocksPerMultiprocessor(n, qgemv_kernel<MODE_GATEUP>, kGvThreads, 0);
}

// y = bf16( bf16(y_acc) + bf16( bf16(sigmoid(gate)) * bf16(ysh) ) )   (model.cpp:800-803)
// or y = bf16(y_acc) without a shared expert.
__global__ void finalize_kernel(const float* __restrict__ y_acc, const float* __restrict__ ysh,
                                const float* __restrict__ gate_sig, int64_t T, int H, uint16_t* __restrict__ y) {
  const int64_t n4 = T * H / 4;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n4;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const float4 r = reinterpret_cast<const float4*>(y_acc)[i];
    float v[4] = {rbf(r.x), rbf(r.y), rbf(r.z), rbf(r.w)};
    if (ysh) {
      const float4 s = reinterpret_cast<const float4*>(ysh)[i];
      const float gsv = gate_sig[(i * 4) / H];
      const float sv[4] = {s.x, s.y, s.z, s.w};
#pragma unroll
      for (int q = 0; q < 4; ++q) v[q] = rbf(v[q] + rbf(gsv * rbf(sv[q])));
    }
    uint2 o;
    o.x = pack_bf16x2(v[0], v[1]);
    o.y = pack_bf16x2(v[2], v[3]);
    reinterpret_cast<uint2*>(y)[i] = o;
  }
}

// TC path combine, y = bf16( bf16(sum_j y_pairs[pos(t, j)]) + bf16(gate * ysh16[t]) ):
// the k routed rows of a token are summed in fp32 in the order j = 0..k-1 (MLX sums
// the [T, k, H] product over axis -2; model.cpp:780-784), then the gated shared row
// is added as in model.cpp:800-803.  One thread per 8 outputs (16-byte accesses).
__global__ void finalize_pairs_kernel(const uint16_t* __restrict__ y_pairs, const int32_t* __restrict__ pair_pos,
                                      int k, const uint16_t* __restrict__ ysh16, const float* __restrict__ gate_sig,
                                      int64_t T, int H, uint16_t* __restrict__ y) {
  const int segs = H / 8;
  const int64_t n = T * segs;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t t = i / segs;
    const int col = static_cast<int>(i - t * segs) * 8;
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int j = 0; j < k; ++j) {
      const int pos = pair_pos[t * k + j];
      if (pos < 0) continue;
      const uint4 v = *reinterpret_cast<const uint4*>(y_pairs + static_cast<int64_t>(pos) * H + col);
      const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        acc[2 * q] += bf2f(static_cast<uint16_t>(w[q] & 0xffffu));
        acc[2 * q + 1] += bf2f(static_cast<uint16_t>(w[q] >> 16));
      }
    }
#pragma unroll
    for (int q = 0; q < 8; ++q) acc[q] = rbf(acc[q]);
    if (ysh16) {
      const float gsv = gate_sig[t];
      const uint4 s = *reinterpret_cast<const uint4*>(ysh16 + t * H + col);
      const uint32_t w[4] = {s.x, s.y, s.z, s.w};
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        acc[2 * q] = rbf(acc[2 * q] + rbf(gsv * bf2f(static_cast<uint16_t>(w[q] & 0xffffu))));
        acc[2 * q + 1] = rbf(acc[2 * q + 1] + rbf(gsv * bf2f(static_cast<uint16_t>(w[q] >> 16))));
      }
    }
    uint4 o;
    o.x = pack_bf16x2(acc[0], acc[1]);
    o.y = pack_bf16x2(acc[2], acc[3]);
    o.z = pack_bf16x2(acc[4], acc[5]);
    o.w = pack_bf16x2(acc[6], acc[7]);
    *reinterpret_cast<uint4*>(y + t * H + col) = o;
  }
}

}  // namespace fm
