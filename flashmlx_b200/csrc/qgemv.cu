// qgemv.cu -- small-batch expert products: 4-bit affine GEMV on the legacy tensor
// pipe (mma.sync m16n8k16), for decode-sized batches (few tokens per expert).
//
// Replaces mx::gather_qmm / mx::quantized_matmul for the decode path
// (model.cpp:703-721, 741-747; decode reaches them with T*k < 64 unsorted, or sorted
// with a handful of tokens per expert).  The kernel is HBM-bound: every weight byte
// of an active expert is read from HBM once (a group with more than 8 rows re-reads
// its weights from L2 per 8-row chunk); inactive experts are never touched.
//
// Arithmetic (the affine split MLX's own small-batch qmv uses): per quantization
// group g of a weight row, y += s_g * sum_k(q_k x_k) + b_g * sum_k(x_k), in fp32, with
// the exact codes q fed to the tensor core as bf16 (0x4300 | q == 128 + q, exact), so
// a code costs ~1 ALU op instead of a bf16 dequantization (the dequantizing form was
// issue-bound at a quarter of HBM bandwidth).  The 128 offset folds into the bias
// term: s*sum((128+q)x) + (b - 128 s)*sum(x).  sum(x) per token and group comes from
// one extra MMA against an all-ones A fragment.  Group sizes 64 and 128 (a 64-wide
// half chunk never straddles a group); the host sends group size 32 to tcgen05.
// K is a multiple of 128, or -- down matrices only, in the HALF instances -- of 64
// with group size 64 (K = 128 n + 64, e.g. the expert width 1856 of Nemotron-3-Nano):
// the last chunk then holds one half, and its second half runs with zero codes,
// scales, biases and activations.  Such rows hold an odd number of quant groups, so
// their scale / bias pairs are not 4-byte aligned; the HALF instances stage the unit's
// scales and biases in shared memory once per unit (4-byte cp.async of the aligned
// words around each row's range) instead of streaming them through the register ring.
//
// Work unit (one CTA of 4 warps): an output-row block x a chunk of <= 8 activation
// rows (one MMA column tile) x an optional K split.  Warp w owns two 16-row MMA tiles:
//   gate/up mode: gate rows [64 rb + 16 w, +16) and the same up rows (SwiGLU in regs)
//   down / plain: rows [128 rb + 32 w, +16) and [.. + 16, +16)
// Per 128-wide K chunk, lane (g = lane/4, c = lane%4) loads words {2c, 2c+1} and
// {8+2c, 9+2c} of rows g and g+8 (two 8-byte loads per row); MMA k-step j of half h
// takes code pairs 2(j&1), 2(j&1)+1 of word 8h + 2c + j/2, which matches the within-8
// pair order of the activation rows, so every k-step lies inside one quant group.
// Codes and scales stream through a three-chunk register ring (two chunks in flight
// per warp); the activation chunk of the unit is staged in shared memory by cp.async.
#include <type_traits>

#include "fm_ep.cuh"

namespace fm {

namespace {

constexpr int kGvThreads = 128;
constexpr int kXStride = 132;  // staged activation row stride (bf16): 264 B keeps the 8-byte fragment reads conflict-free
constexpr int kSbGroups = 62;  // HALF instances: at most 62 quant groups per row in one unit (host-checked)
constexpr int kSbStride = 66;  // u16 per staged row: <= 32 words of groups; 33 words keep the 8 rows' reads conflict-free

FM_DEV float swiglu1(float g, float u) {  // model.cpp:14-25, bf16 rounding per op
  const float gs = rbf(sigmoid_f(g));
  const float h = rbf(g * gs);
  return rbf(h * u);
}

// relu^2 of a bf16 value, rounded to bf16 (nemotron_h.cpp:53-58: maximum(x, 0), square)
FM_DEV float relu2_1(float v) {
  const float r = fmaxf(v, 0.f);
  return rbf(r * r);
}

// code pair (q_p, q_{p+4}) of a packed word as bf16x2 (128 + q_p, 128 + q_{p+4})
FM_DEV uint32_t code_pair_128(uint32_t w, int p) { return ((w >> (4 * p)) & 0x000F000Fu) | 0x43004300u; }

FM_DEV uint2 ldg_nc_v2(const uint32_t* p) {
  uint2 v;
  asm volatile("ld.global.nc.L1::no_allocate.v2.u32 {%0,%1}, [%2];" : "=r"(v.x), "=r"(v.y) : "l"(p));
  return v;
}

FM_DEV void cp_async8(uint32_t dst, const void* src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"(dst), "l"(src) : "memory");
}

FM_DEV void cp_async4(uint32_t dst, const void* src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(dst), "l"(src) : "memory");
}

}  // namespace

template <int MODE, bool HALF>
__global__ void __launch_bounds__(kGvThreads, 3) qgemv_kernel(const GemmArgs a) {
  constexpr bool kDown = MODE == MODE_DOWN || MODE == MODE_DOWN_F32;
  static_assert(!HALF || kDown, "half chunks only on the down matrices");
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, c = lane & 3;
  const TileTable* tab = a.tab;
  if (*reinterpret_cast<volatile uint32_t*>(a.err) != 0u) return;  // an earlier kernel failed
  const int ntiles = tab->num_tiles;
  // shared-memory copy of the groups' first tile ids (tile lookups stay on chip) and a
  // three-slot ring of 8 activation rows x 128 K (the B operand of one chunk)
  __shared__ int s_tb[kMaxGroups];
  __shared__ __align__(16) uint16_t s_x[3][8][kXStride];
  // HALF: scales [0, 128) and biases [128, 256) of the unit's rows (row 32 warp + 16 m + 8 h + g)
  uint16_t* sb = nullptr;
  if constexpr (HALF) {
    __shared__ __align__(16) uint16_t s_sb[2 * kGvThreads * kSbStride];
    sb = s_sb;
  }
  const int ngroups = min(tab->num_groups, kMaxGroups);
  for (int i = threadIdx.x; i < ngroups; i += blockDim.x) s_tb[i] = tab->g[i].tile_begin;
  __syncthreads();
  const bool gs128 = a.gs == 128;  // else 64: two groups per 128-wide chunk
  for (int tile = blockIdx.x; tile < ntiles; tile += gridDim.x) {
    const TileInfo ti = decode_tile(tab, s_tb, ngroups, tile);
    const bool sh = ti.expert < 0;
    const int K = (kDown && sh) ? a.K_shared : a.K;
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

    // row g of each 16-row tile (row g + 8 is 8 rows further)
    const uint32_t* wrow[2];
    const uint16_t* srow[2];
    const uint16_t* brow[2];
#pragma unroll
    for (int m = 0; m < 2; ++m) {
      const int64_t r = erow + min(r0[m] + g, N - 1);
      wrow[m] = Wm[m] + r * kw + 2 * c;
      srow[m] = Sm[m] + r * gpr;
      brow[m] = Bm[m] ? Bm[m] + r * gpr : nullptr;
    }

    const int kfull = K / 128;  // chunks with both 64-wide halves
    const int kchunks = HALF ? kfull + ((K & 127) != 0) : kfull;  // + a trailing half chunk
    const int kc0 = kchunks * ti.ks / ti.ksplit, kc1 = kchunks * (ti.ks + 1) / ti.ksplit;
    __syncthreads();  // every warp is done reading the ring (and the staged scales) of the previous unit
    // HALF: u16 index in sb of (row g + 8h of tile m, the unit's first group), biases + kBias
    constexpr int kBias = kGvThreads * kSbStride;
    uint32_t sbo[2][2] = {{0u, 0u}, {0u, 0u}};
    if constexpr (HALF) {
      const int gbase = 2 * kc0;                       // the unit's first quant group (group size 64)
      const int ng = min(2 * (kc1 - kc0), gpr - gbase);  // its groups
      if (ng > kSbGroups) {  // the host splits K so that this never happens
        if (threadIdx.x == 0) report(a.err, DEVERR_CONFIG);
        continue;
      }
      // staged rows: a warp's 32 rows (16 m + 8 h + j) of scales, then of biases, each
      // from the aligned word holding group gbase on; lpr consecutive lanes copy
      // consecutive words of one row (coalesced), 32 / lpr rows per pass
      const int lpr = ng <= 30 ? 16 : 32;  // a row's words: at most (ng + 2) / 2 <= 32
      for (int rw = lane / lpr; ng > 0 && rw < 64; rw += 32 / lpr) {  // rw = 32 * (bias) + local row;
                                                                      // an empty unit copies nothing
        const int w = lane & (lpr - 1);
        const int lr = rw & 31;
        const int rl = r0[0] + lr;  // down modes: the warp's rows are contiguous (r0[1] = r0[0] + 16)
        if (rl >= N) continue;      // whole 16-row tile past N: never read
        const uint16_t* base = (rw >> 5) ? Bm[0] : Sm[0];  // one matrix in the down modes
        if (!base) continue;
        const int64_t e = (erow + rl) * gpr + gbase;
        const int off = static_cast<int>(e & 1);
        // words [e - off, e - off + 2 nw) cover the row's groups [e, e + ng); the one u16
        // past them (off + ng odd) lies inside the array, whose length (rows x groups, rows
        // a multiple of 16) is even from a 4-byte aligned base
        if (w >= ((off + ng + 1) >> 1)) continue;
        uint16_t* d = sb + (rw >> 5) * kBias + (warp * 32 + lr) * kSbStride + 2 * w;
        cp_async4(smem_u32(d), base + (e - off) + 2 * w);
      }
#pragma unroll
      for (int m = 0; m < 2; ++m)
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int rl = min(r0[m] + g + 8 * h, N - 1);
          const int off = static_cast<int>(((erow + rl) * gpr + gbase) & 1);
          sbo[m][h] = (warp * 32 + 16 * m + 8 * h + g) * kSbStride + off;
        }
    }
    // activation rows of the unit (<= 8): thread tid copies 16 bytes (two 8-byte copies)
    // of row tid / 16 per chunk into the ring; rows past the unit are zero-filled
    const int xr = threadIdx.x >> 4, xc = threadIdx.x & 15;
    const uint16_t* xsrc = nullptr;
    if (xr < ti.nrows) {
      const int p = ti.row0 + xr;
      const int64_t src = (kDown || sh) ? p : a.sorted_token[p];
      xsrc = (sh ? a.act_shared : a.act) + src * (sh ? a.act_shared_ld : a.act_ld) + xc * 8;
    }
    auto load_x = [&](int kc, int slot) {
      uint16_t* d = &s_x[slot][xr][xc * 8];
      if (kc < kc1 && xsrc && (!HALF || kc < kfull || xc < 8)) {
        cp_async8(smem_u32(d), xsrc + kc * 128);
        cp_async8(smem_u32(d + 4), xsrc + kc * 128 + 4);
      } else {
        *reinterpret_cast<uint2*>(d) = make_uint2(0, 0);
        *reinterpret_cast<uint2*>(d + 4) = make_uint2(0, 0);
      }
      cp_async_commit();
    };

    float y[2][4];
#pragma unroll
    for (int m = 0; m < 2; ++m) y[m][0] = y[m][1] = y[m][2] = y[m][3] = 0.f;

    // Three-slot register ring: chunk kc is consumed from slot 0 while chunks kc+1 and
    // kc+2 are in flight: codes W[m][h][half] (2 words each) and the raw bf16 scale /
    // bias pairs of rows g, g+8 (groups of the two halves, low half = first group).
    constexpr int RING = 3;
    uint2 W[RING][2][2][2];
    uint32_t S2[RING][2][2], B2[RING][2][2];
    auto load_chunk = [&](int kc, uint2 (&Wd)[2][2][2], uint32_t (&Sd)[2][2], uint32_t (&Bd)[2][2]) {
      const bool in = kc < kc1, full = !HALF || kc < kfull;
#pragma unroll
      for (int m = 0; m < 2; ++m)
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const bool v = in && (m == 0 ? mval0 : mval1);
          const uint32_t* wp = wrow[m] + 8 * h * kw + kc * 16;
          Wd[m][h][0] = v ? ldg_nc_v2(wp) : make_uint2(0, 0);
          Wd[m][h][1] = (v && full) ? ldg_nc_v2(wp + 8) : make_uint2(0, 0);
          if constexpr (HALF) continue;  // scales and biases come from shared memory
          const uint16_t* sp = srow[m] + 8 * h * gpr;
          const uint16_t* bp = brow[m] ? brow[m] + 8 * h * gpr : nullptr;
          if (gs128) {
            const uint32_t sv = v ? static_cast<uint32_t>(__ldg(sp + kc)) : 0u;
            const uint32_t bv = (v && bp) ? static_cast<uint32_t>(__ldg(bp + kc)) : 0u;
            Sd[m][h] = sv * 0x10001u;
            Bd[m][h] = bv * 0x10001u;
          } else {  // groups 2kc, 2kc+1: one aligned 4-byte load (gpr is even)
            Sd[m][h] = v ? __ldg(reinterpret_cast<const uint32_t*>(sp + 2 * kc)) : 0u;
            Bd[m][h] = (v && bp) ? __ldg(reinterpret_cast<const uint32_t*>(bp + 2 * kc)) : 0u;
          }
        }
    };
#pragma unroll
    for (int r = 0; r < RING; ++r) load_chunk(kc0 + r, W[r], S2[r], B2[r]);
    load_x(kc0, 0);
    load_x(kc0 + 1, 1);

    const uint32_t ONES = 0x3F803F80u;  // bf16x2 (1, 1)
    // Chunk kc lives in ring slot (kc - kc0) % 3; the loop is unrolled by the ring size
    // so every slot is a fixed set of registers (a register copy between slots would
    // wait for that slot's loads and collapse the ring to one chunk in flight).
    auto step = [&](int kc, auto slot_c) {
      constexpr int SL = decltype(slot_c)::value;
      cp_async_wait<1>();  // this thread's copy of chunk kc has landed
      __syncthreads();     // ... and every thread's; chunk kc-1's slot is free again
      load_x(kc + 2, (SL + 2) % 3);
      const uint16_t* xrowg = &s_x[SL][g][0];
#pragma unroll
      for (int hf = 0; hf < 2; ++hf) {
        float acc[2][4], xsum[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) acc[0][e] = acc[1][e] = xsum[e] = 0.f;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int wi = j >> 1, p0 = 2 * (j & 1);
          const uint2 bx = *reinterpret_cast<const uint2*>(xrowg + (hf * 8 + 2 * c + wi) * 8 + 2 * p0);
          mma_bf16_16816(xsum, ONES, ONES, ONES, ONES, bx.x, bx.y);
#pragma unroll
          for (int m = 0; m < 2; ++m) {  // rows past N carry zero codes and scales
            const uint32_t wg = wi ? W[SL][m][0][hf].y : W[SL][m][0][hf].x;
            const uint32_t wg8 = wi ? W[SL][m][1][hf].y : W[SL][m][1][hf].x;
            mma_bf16_16816(acc[m], code_pair_128(wg, p0), code_pair_128(wg8, p0), code_pair_128(wg, p0 + 1),
                           code_pair_128(wg8, p0 + 1), bx.x, bx.y);
          }
        }
        // this half's quant group: y += s * acc + (b - 128 s) * sum(x)
#pragma unroll
        for (int m = 0; m < 2; ++m) {
          float s0, s8, b0, b8;
          if constexpr (HALF) {  // group 2(kc - kc0) + hf of the unit; the empty half of a trailing chunk is 0
            const bool gv = hf == 0 || kc < kfull;
            const uint32_t q = 2 * (kc - kc0) + hf;
            s0 = gv ? bf2f(sb[sbo[m][0] + q]) : 0.f;
            s8 = gv ? bf2f(sb[sbo[m][1] + q]) : 0.f;
            b0 = (gv && Bm[m]) ? bf2f(sb[kBias + sbo[m][0] + q]) : 0.f;
            b8 = (gv && Bm[m]) ? bf2f(sb[kBias + sbo[m][1] + q]) : 0.f;
          } else {
            s0 = bf2f(static_cast<uint16_t>(hf ? S2[SL][m][0] >> 16 : S2[SL][m][0] & 0xffffu));
            s8 = bf2f(static_cast<uint16_t>(hf ? S2[SL][m][1] >> 16 : S2[SL][m][1] & 0xffffu));
            b0 = bf2f(static_cast<uint16_t>(hf ? B2[SL][m][0] >> 16 : B2[SL][m][0] & 0xffffu));
            b8 = bf2f(static_cast<uint16_t>(hf ? B2[SL][m][1] >> 16 : B2[SL][m][1] & 0xffffu));
          }
          const float c0 = fmaf(-128.f, s0, b0), c8 = fmaf(-128.f, s8, b8);
          y[m][0] = fmaf(s0, acc[m][0], fmaf(c0, xsum[0], y[m][0]));
          y[m][1] = fmaf(s0, acc[m][1], fmaf(c0, xsum[1], y[m][1]));
          y[m][2] = fmaf(s8, acc[m][2], fmaf(c8, xsum[2], y[m][2]));
          y[m][3] = fmaf(s8, acc[m][3], fmaf(c8, xsum[3], y[m][3]));
        }
      }
      load_chunk(kc + RING, W[SL], S2[SL], B2[SL]);  // refill this slot RING chunks ahead
    };
    for (int kc = kc0; kc < kc1; kc += RING) {
      step(kc, std::integral_constant<int, 0>{});
      if (kc + 1 < kc1) step(kc + 1, std::integral_constant<int, 1>{});
      if (kc + 2 < kc1) step(kc + 2, std::integral_constant<int, 2>{});
    }

    // epilogue: y[m][e] is (row r0[m] + g + 8*(e>>1), slot 2c + (e&1))
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int slot = 2 * c + (e & 1);
      if (slot >= ti.nrows) continue;
      const int p = ti.row0 + slot;
      if (MODE == MODE_GATEUP) {
        if (!mval0) continue;
        const int n = r0[0] + g + 8 * (e >> 1);
        const float gv = rbf(y[0][e]), uv = rbf(y[1][e]);
        uint16_t* out = sh ? a.out_shared + static_cast<int64_t>(p) * a.out_shared_ld
                           : a.out + static_cast<int64_t>(p) * a.out_ld;
        out[perm8(n)] = f2bf(swiglu1(gv, uv));
      } else {
#pragma unroll
        for (int m = 0; m < 2; ++m) {
          if (!(m == 0 ? mval0 : mval1)) continue;
          const int n = r0[m] + g + 8 * (e >> 1);
          const float v = y[m][e];
          if (MODE == MODE_RELU2) {  // fc1 -> relu^2, activation rows for the down matrix
            uint16_t* out = sh ? a.out_shared + static_cast<int64_t>(p) * a.out_shared_ld
                               : a.out + static_cast<int64_t>(p) * a.out_ld;
            out[perm8(n)] = f2bf(relu2_1(rbf(v)));
          } else if (kDown) {
            if (sh) {
              red_add_f32(a.ysh + static_cast<int64_t>(p) * a.y_ld + n, v);
            } else if (MODE == MODE_DOWN_F32) {  // sigmoid routing: fp32 d * score, summed in fp32
              const int t = a.sorted_token[p];
              red_add_f32(a.y_acc + static_cast<int64_t>(t) * a.y_ld + n, rbf(v) * a.sorted_score[p]);
            } else if (a.y_rowptr) {  // one output row per pair, at its destination (peer memory)
              a.y_rowptr[p][n] = f2bf(rbf(rbf(v) * a.sorted_score[p]));
            } else if (a.y_pairs) {  // one output row per pair (expert-parallel owner side)
              a.y_pairs[static_cast<int64_t>(p) * a.y_ld + n] = f2bf(rbf(rbf(v) * a.sorted_score[p]));
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

// A K (routed or shared) that is not a multiple of 128 takes the HALF instance of a
// down mode; the host checks group size 64, 4-byte aligned scales / biases and at most
// kSbGroups groups per row and unit.
cudaError_t launch_qgemv(int mode, int grid, cudaStream_t stream, const GemmArgs& a) {
  const bool half = (a.K & 127) || ((mode == MODE_DOWN || mode == MODE_DOWN_F32) && a.N_shared > 0 && (a.K_shared & 127));
  if (half) {
    if (a.gs != 64) return cudaErrorInvalidValue;
    switch (mode) {
      case MODE_DOWN: qgemv_kernel<MODE_DOWN, true><<<grid, kGvThreads, 0, stream>>>(a); break;
      case MODE_DOWN_F32: qgemv_kernel<MODE_DOWN_F32, true><<<grid, kGvThreads, 0, stream>>>(a); break;
      default: return cudaErrorInvalidValue;
    }
    return cudaGetLastError();
  }
  switch (mode) {
    case MODE_GATEUP: qgemv_kernel<MODE_GATEUP, false><<<grid, kGvThreads, 0, stream>>>(a); break;
    case MODE_DOWN: qgemv_kernel<MODE_DOWN, false><<<grid, kGvThreads, 0, stream>>>(a); break;
    case MODE_RELU2: qgemv_kernel<MODE_RELU2, false><<<grid, kGvThreads, 0, stream>>>(a); break;
    case MODE_DOWN_F32: qgemv_kernel<MODE_DOWN_F32, false><<<grid, kGvThreads, 0, stream>>>(a); break;
    default: qgemv_kernel<MODE_PLAIN, false><<<grid, kGvThreads, 0, stream>>>(a); break;
  }
  return cudaGetLastError();
}

cudaError_t qgemv_blocks_per_sm(int* n) {
  return cudaOccupancyMaxActiveBlocksPerMultiprocessor(n, qgemv_kernel<MODE_GATEUP, false>, kGvThreads, 0);
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
// KU > 0 (k <= KU): all k rows' loads are issued before the first add (one memory
// latency per output segment, not k), in an instance whose registers fit KU rows;
// KU == 0: any k, one row at a time.
template <int KU>
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
    auto add_row = [&](const uint4& v) {
      const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        acc[2 * q] += bf2f(static_cast<uint16_t>(w[q] & 0xffffu));
        acc[2 * q + 1] += bf2f(static_cast<uint16_t>(w[q] >> 16));
      }
    };
    // the shared row's load first; the adds keep the order j = 0..k-1
    const uint4 shv = ysh16 ? *reinterpret_cast<const uint4*>(ysh16 + t * H + col) : make_uint4(0u, 0u, 0u, 0u);
    if constexpr (KU > 0) {
      int pos[KU];
      uint4 v[KU];
#pragma unroll
      for (int j = 0; j < KU; ++j) pos[j] = j < k ? pair_pos[t * k + j] : -1;
#pragma unroll
      for (int j = 0; j < KU; ++j)
        if (pos[j] >= 0) v[j] = *reinterpret_cast<const uint4*>(y_pairs + static_cast<int64_t>(pos[j]) * H + col);
#pragma unroll
      for (int j = 0; j < KU; ++j)
        if (pos[j] >= 0) add_row(v[j]);
    } else {
      for (int j = 0; j < k; ++j) {
        const int pos = pair_pos[t * k + j];
        if (pos < 0) continue;
        add_row(*reinterpret_cast<const uint4*>(y_pairs + static_cast<int64_t>(pos) * H + col));
      }
    }
#pragma unroll
    for (int q = 0; q < 8; ++q) acc[q] = rbf(acc[q]);
    if (ysh16) {
      const float gsv = gate_sig[t];
      const uint4 s = shv;
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

// the combine instance for top-k k: rows' loads batched for k <= 8
void launch_finalize_pairs(int grid, cudaStream_t stream, const uint16_t* y_pairs, const int32_t* pair_pos, int k,
                           const uint16_t* ysh16, const float* gate_sig, int64_t T, int H, uint16_t* y) {
  if (k <= 2) finalize_pairs_kernel<2><<<grid, 256, 0, stream>>>(y_pairs, pair_pos, k, ysh16, gate_sig, T, H, y);
  else if (k <= 4) finalize_pairs_kernel<4><<<grid, 256, 0, stream>>>(y_pairs, pair_pos, k, ysh16, gate_sig, T, H, y);
  else if (k <= 8) finalize_pairs_kernel<8><<<grid, 256, 0, stream>>>(y_pairs, pair_pos, k, ysh16, gate_sig, T, H, y);
  else finalize_pairs_kernel<0><<<grid, 256, 0, stream>>>(y_pairs, pair_pos, k, ysh16, gate_sig, T, H, y);
}

// The sigmoid-routed variant's combine on the tcgen05 path, y = bf16( bf16(sum_j
// bf16(d_j) * score_j) + bf16(gate * ysh16[t]) ): y_pairs holds bf16(d) per routed pair,
// the scores are the fp32 routing scores as applied (nemotron_h.cpp:1094-1100: the
// products and their sum over j = 0..k-1 stay in fp32), gate_sig is 1 for an ungated
// shared expert.  One thread per 8 outputs.
__global__ void finalize_pairs_f32_kernel(const uint16_t* __restrict__ y_pairs, const int32_t* __restrict__ pair_pos,
                                          const float* __restrict__ score, int k, const uint16_t* __restrict__ ysh16,
                                          const float* __restrict__ gate_sig, int64_t T, int H,
                                          uint16_t* __restrict__ y) {
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
      const float sc = score[t * k + j];
      const uint4 v = *reinterpret_cast<const uint4*>(y_pairs + static_cast<int64_t>(pos) * H + col);
      const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        // d * score rounded to fp32, then added (no fused multiply-add): the per-op
        // rounding of the reference's multiply then sum, and of the GEMV path's
        // red.add of the rounded product
        acc[2 * q] = __fadd_rn(acc[2 * q], __fmul_rn(bf2f(static_cast<uint16_t>(w[q] & 0xffffu)), sc));
        acc[2 * q + 1] = __fadd_rn(acc[2 * q + 1], __fmul_rn(bf2f(static_cast<uint16_t>(w[q] >> 16)), sc));
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

// Expert-parallel send buffer: row p = x_perm[sorted_token[p]] (the routed pairs in
// expert-major order, so the rows bound for each owner rank are contiguous).
__global__ void ep_gather_kernel(const uint16_t* __restrict__ x_perm, const int32_t* __restrict__ sorted_token,
                                 int64_t P, int H, uint16_t* __restrict__ send) {
  const int segs = H / 8;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < P * segs;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t p = i / segs;
    const int col = static_cast<int>(i - p * segs) * 8;
    *reinterpret_cast<uint4*>(send + p * H + col) =
        *reinterpret_cast<const uint4*>(x_perm + static_cast<int64_t>(sorted_token[p]) * H + col);
  }
}

// Expert-parallel combine on the token's rank: ret[pos] holds bf16(d) returned by the
// owner of pair (t, j); y = bf16( bf16(sum_j bf16(d * score_j)) + bf16(gate * shared) ),
// the sum over j = 0..k-1 in fp32 in that order (model.cpp:780-784, 800-803).  The
// shared rows come as fp32 sums (GEMV path) or bf16 rows (tcgen05 path).
__device__ __forceinline__ void combine_rows(const uint16_t* __restrict__ ret, const int32_t* __restrict__ pair_pos,
                                             const float* __restrict__ score, int k, const float* __restrict__ ysh32,
                                             const uint16_t* __restrict__ ysh16, const float* __restrict__ gate_sig,
                                             int64_t T, int H, uint16_t* __restrict__ y) {
  const int segs = H / 8;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < T * segs;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t t = i / segs;
    const int col = static_cast<int>(i - t * segs) * 8;
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int j = 0; j < k; ++j) {
      const int pos = pair_pos[t * k + j];
      if (pos < 0) continue;
      const float sc = score[t * k + j];
      const uint4 v = *reinterpret_cast<const uint4*>(ret + static_cast<int64_t>(pos) * H + col);
      const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        acc[2 * q] += rbf(bf2f(static_cast<uint16_t>(w[q] & 0xffffu)) * sc);
        acc[2 * q + 1] += rbf(bf2f(static_cast<uint16_t>(w[q] >> 16)) * sc);
      }
    }
#pragma unroll
    for (int q = 0; q < 8; ++q) acc[q] = rbf(acc[q]);
    if (ysh32 || ysh16) {
      const float gsv = gate_sig[t];
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        const float sv = ysh32 ? rbf(ysh32[t * H + col + q]) : bf2f(ysh16[t * H + col + q]);
        acc[q] = rbf(acc[q] + rbf(gsv * sv));
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

__global__ void finalize_ep_kernel(const uint16_t* __restrict__ ret, const int32_t* __restrict__ pair_pos,
                                   const float* __restrict__ score, int k, const float* __restrict__ ysh32,
                                   const uint16_t* __restrict__ ysh16, const float* __restrict__ gate_sig, int64_t T,
                                   int H, uint16_t* __restrict__ y) {
  combine_rows(ret, pair_pos, score, k, ysh32, ysh16, gate_sig, T, H, y);
}

// Peer-memory variant (ep.cu): wait until every owner returned its rows into this
// rank's ret buffer, then combine as finalize_ep_kernel.
__global__ void __launch_bounds__(256) ep_combine_p2p_kernel(const EpP2PArgs a, const int32_t* __restrict__ pair_pos,
                                                             const float* __restrict__ score, int k,
                                                             const float* __restrict__ ysh32,
                                                             const uint16_t* __restrict__ ysh16,
                                                             const float* __restrict__ gate_sig, int64_t T,
                                                             uint16_t* __restrict__ y) {
  if (ep_block_error(a)) return;
  if (!ep_wait_all(a, 2)) return;
  combine_rows(ep_rows(a, a.rank, a.off_ret), pair_pos, score, k, ysh32, ysh16, gate_sig, T, a.H, y);
}

}  // namespace fm
