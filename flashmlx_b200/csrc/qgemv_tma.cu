// qgemv_tma.cu -- small-batch expert products fed by TMA: the decode-path GEMV.
//
// Replaces mx::gather_qmm / mx::quantized_matmul for few tokens per expert
// (model.cpp:703-721, 741-747) with the arithmetic of qgemv.cu -- MLX's small-batch
// qmv form: per quantization group, s * sum(q x) + b * sum(x) in fp32, the exact codes
// fed to the legacy tensor core as bf16 (0x4300 | q == 128 + q), the 128 offset folded
// into the bias term, sum(x) from an MMA against ones -- with the data movement of a
// Blackwell pipeline instead of per-lane global loads:
//
//   producer warp   per stage (256 K positions of the unit's 128 weight rows): one or
//                   two TMA box loads of the codes (128B swizzle), one 1D bulk copy per
//                   activation row (<= 16 rows), 4-byte cp.async of the rows' scales and
//                   biases; all complete on the stage's mbarrier
//   4 consumer warps  read codes (LDS.64), activations (LDS.128) and scales from the
//                   stage, run the MMAs, fold each quant group into fp32 row sums, and
//                   release the stage
//
// The weight bytes reach shared memory in 16 KB boxes from one thread, so the
// consumers spend their issue slots on code unpacking and MMAs (the per-lane loads,
// address arithmetic and register ring of qgemv.cu took about half of them), and a
// 4-stage ring keeps up to 64 KB of codes per CTA in flight.  One work unit covers up to
// 16 activation rows (two 8-column MMA tiles), so a weight row is read and unpacked once
// for every 16 tokens of its expert, not once per 8 of them.
//
// Same work units and tile tables as qgemv.cu (gate/up: 64 gate + 64 up rows, SwiGLU in
// registers; down / plain: 128 rows), same outputs, same per-group accumulation order.
// Handles K % 128 == 0 with group size 64 or 128; qgemv.cu keeps the half-chunk widths
// and the variants' relu^2 / fp32-score modes.
#include "fm_ep.cuh"

namespace fm {

namespace {

constexpr int kTvConsumers = 8;                       // consumer warps (one 16-row MMA tile each)
constexpr int kTvThreads = 32 * (kTvConsumers + 1);   // + the producer warp
constexpr int kTvStages = 4;
constexpr int kTvRows = 128;                          // weight rows per unit and stage
constexpr int kTvStageK = 256;                        // K positions per stage (32 code words a row)
constexpr int kTvNt = 2;                              // 8-column MMA tiles of activation rows per unit
constexpr int kTvMaxRows = 8 * kTvNt;                 // activation rows per unit
constexpr int kTvXPitch = 528;                        // bytes per staged activation row (512 + 16:
                                                      // the LDS.128 of 8 rows x 4 lanes hit 8 bank groups)
constexpr int kTvCodeBytes = kTvRows * 128;           // 16 KB
constexpr int kTvXBytes = kTvMaxRows * kTvXPitch;
constexpr int kTvSbBytes = kTvRows * 8;               // [128 rows][4 groups] bf16 scales (or biases)
constexpr int kTvOffX = kTvStages * kTvCodeBytes;
constexpr int kTvOffSb = kTvOffX + kTvStages * kTvXBytes;
constexpr int kTvOffBar = kTvOffSb + kTvStages * 2 * kTvSbBytes;
constexpr int kTvBarBytes = 128;
constexpr int kTvSmemBytes = kTvOffBar + kTvBarBytes + 1024;  // + alignment slack
static_assert(kTvOffX % 1024 == 0, "1 KB aligned code stages (128B swizzle)");
static_assert(kTvOffBar % 16 == 0, "aligned barriers");

struct TvBars {
  uint64_t full[kTvStages];   // codes, activation rows, scales landed (1 expect_tx + 32 cp.async arrivals)
  uint64_t empty[kTvStages];  // every consumer warp is done reading the stage
  int abort;
};
static_assert(sizeof(TvBars) <= kTvBarBytes, "barrier block");
constexpr uint32_t kTvFullArrivals = 1 + 32;

FM_DEV void bulk_load(uint32_t dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

FM_DEV void cp_async4_zfill(uint32_t dst, const void* src, uint32_t src_bytes) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(dst), "l"(src), "r"(src_bytes) : "memory");
}

FM_DEV void cp_async_arrive_noinc(uint64_t* bar) {
  asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_u32(bar)) : "memory");
}

FM_DEV bool wait_done(uint64_t* bar, uint32_t parity, uint32_t* err) {  // ignores the abort flag
  const long long t0 = clock64();
  while (!mbar_try_wait(bar, parity)) {
    if (clock64() - t0 > kWaitBudgetCycles) {
      report(err, DEVERR_TIMEOUT);
      return false;
    }
  }
  return true;
}

FM_DEV float swiglu_1(float g, float u) {  // model.cpp:14-25, bf16 rounding per op
  const float gs = rbf(sigmoid_f(g));
  const float h = rbf(g * gs);
  return rbf(h * u);
}

// One work unit as both roles see it.
struct TvUnit {
  TileInfo ti;
  bool sh;
  int K, N, gpr;
  int64_t erow;   // first row of the expert's matrix in the stacked [E * N, K / 8] codes
  int st0, st1;   // stages [st0, st1) of the unit's K range
};

template <int MODE>
FM_DEV TvUnit tv_unit(const GemmArgs& a, const TileTable* tab, const int* s_tb, int ngroups, int tile, int gs) {
  TvUnit u;
  u.ti = decode_tile(tab, s_tb, ngroups, tile);
  u.sh = u.ti.expert < 0;
  u.K = (MODE == MODE_DOWN && u.sh) ? a.K_shared : a.K;
  u.N = u.sh ? a.N_shared : a.N;
  u.gpr = u.K / gs;
  u.erow = u.sh ? 0 : static_cast<int64_t>(u.ti.expert) * u.N;
  const int nst = (u.K + kTvStageK - 1) / kTvStageK;
  u.st0 = nst * u.ti.ks / u.ti.ksplit;
  u.st1 = nst * (u.ti.ks + 1) / u.ti.ksplit;
  return u;
}

// first output row of the unit's block and the unit's matrix row of local row t (0..127)
template <int MODE>
FM_DEV int tv_row(const TvUnit& u, int t) {
  return MODE == MODE_GATEUP ? u.ti.rb * 64 + (t & 63) : u.ti.rb * 128 + t;
}

// One stage of one consumer warp: its 16-row MMA tile (rows g and g + 8 of the lane
// group; the second row rstep bytes after the first in the code stage), NH valid
// 64-wide halves (4, or 2 at a K tail), NT 8-column MMA tiles of activation rows.  The
// halves are unrolled without branches, so the compiler overlaps the shared-memory
// reads, code unpacking, MMAs and group folds of different halves.
//   cs: this lane's code bytes in the stage (row g of the tile); chunk_x: (c / 2) ^ g, so
//       half h's 16-byte chunk after the 128B swizzle is (2h) ^ chunk_x
//   xs: its activation bytes (row g, K positions 16 c ..), rows of tile n 8 * pitch further
//   S0 / S1, B0 / B1: scales / biases of the tile's rows g and g + 8 (4 groups each, bf16)
// Per half: words 8h + 2c, 8h + 2c + 1 of both rows; code pair p of a word is
// (q_p, q_{p+4}) as bf16x2 (128 + q_p, 128 + q_{p+4}); MMA step ps of a word takes pairs
// 2 ps, 2 ps + 1 against the activation slots of the same positions, the two steps in
// separate accumulators (short MMA chains), sum(x) in one; per group
// y += s * acc + (b - 128 s) * sum(x).
template <int GS, int NT, int NH>
FM_DEV void tv_stage(const uint8_t* cs, uint32_t rstep, uint32_t chunk_x, const uint8_t* xs, uint2 S0,
                     uint2 S1, uint2 B0, uint2 B1, float (&y)[kTvNt][4]) {
  constexpr uint32_t ONES = 0x3F803F80u;  // bf16x2 (1, 1)
  float acc[NT][2][4], xsum[NT][4];
#pragma unroll
  for (int h = 0; h < NH; ++h) {
    uint2 w[2];
    uint4 xv[NT][2];
#pragma unroll
    for (int r = 0; r < 2; ++r) w[r] = *reinterpret_cast<const uint2*>(cs + (((2u * h) ^ chunk_x) << 4) + r * rstep);
#pragma unroll
    for (int n = 0; n < NT; ++n) {
      xv[n][0] = *reinterpret_cast<const uint4*>(xs + n * 8 * kTvXPitch + 128 * h);
      xv[n][1] = *reinterpret_cast<const uint4*>(xs + n * 8 * kTvXPitch + 128 * h + 16);
    }
    if (GS == 64 || (h & 1) == 0) {
#pragma unroll
      for (int n = 0; n < NT; ++n)
#pragma unroll
        for (int ps = 0; ps < 2; ++ps)
#pragma unroll
          for (int e = 0; e < 4; ++e) xsum[n][e] = acc[n][ps][e] = 0.f;
    }
#pragma unroll
    for (int wi = 0; wi < 2; ++wi) {
      uint32_t q[2][4];  // [row g / g + 8][pair]
#pragma unroll
      for (int r = 0; r < 2; ++r) {
        const uint32_t v = wi ? w[r].y : w[r].x;
#pragma unroll
        for (int pp = 0; pp < 4; ++pp) q[r][pp] = ((v >> (4 * pp)) & 0x000F000Fu) | 0x43004300u;
      }
#pragma unroll
      for (int n = 0; n < NT; ++n) {
        const uint4& x = xv[n][wi];
#pragma unroll
        for (int ps = 0; ps < 2; ++ps) {
          const uint32_t b0 = ps ? x.z : x.x, b1 = ps ? x.w : x.y;
          mma_bf16_16816(xsum[n], ONES, ONES, ONES, ONES, b0, b1);
          mma_bf16_16816(acc[n][ps], q[0][2 * ps], q[1][2 * ps], q[0][2 * ps + 1], q[1][2 * ps + 1], b0, b1);
        }
      }
    }
    if (GS == 64 || (h & 1) == 1 || h + 1 == NH) {  // the group ends with this half
      const int gi = GS == 64 ? h : h >> 1;          // group within the stage
      const uint32_t sw0 = gi < 2 ? S0.x : S0.y, sw8 = gi < 2 ? S1.x : S1.y;
      const uint32_t bw0 = gi < 2 ? B0.x : B0.y, bw8 = gi < 2 ? B1.x : B1.y;
      const float s0 = __uint_as_float((gi & 1) ? (sw0 & 0xFFFF0000u) : (sw0 << 16));
      const float s8 = __uint_as_float((gi & 1) ? (sw8 & 0xFFFF0000u) : (sw8 << 16));
      const float c0 = fmaf(-128.f, s0, __uint_as_float((gi & 1) ? (bw0 & 0xFFFF0000u) : (bw0 << 16)));
      const float c8 = fmaf(-128.f, s8, __uint_as_float((gi & 1) ? (bw8 & 0xFFFF0000u) : (bw8 << 16)));
#pragma unroll
      for (int n = 0; n < NT; ++n)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float sv = e < 2 ? s0 : s8, cv = e < 2 ? c0 : c8;
          y[n][e] = fmaf(sv, acc[n][0][e] + acc[n][1][e], fmaf(cv, xsum[n][e], y[n][e]));
        }
    }
  }
}

}  // namespace

template <int MODE, int GS>
__global__ void __launch_bounds__(kTvThreads, 2) qgemv_tma_kernel(const GemmArgs a, const __grid_constant__ TcMaps maps) {
  static_assert(MODE == MODE_GATEUP || MODE == MODE_DOWN || MODE == MODE_PLAIN, "modes of the TMA GEMV");
  static_assert(GS == 64 || GS == 128, "group sizes of the GEMV");
  constexpr int G = kTvStageK / GS;  // quant groups per row and stage
  extern __shared__ uint8_t smem_raw[];
  __shared__ int s_tb[kMaxGroups];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  TvBars* bars = reinterpret_cast<TvBars*>(smem + kTvOffBar);
  volatile int* abort_flag = &bars->abort;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (*reinterpret_cast<volatile uint32_t*>(a.err) != 0u) return;  // an earlier kernel failed
  const TileTable* tab = a.tab;
  const int ntiles = tab->num_tiles;
  const int ngroups = min(tab->num_groups, kMaxGroups);
  for (int i = threadIdx.x; i < ngroups; i += blockDim.x) s_tb[i] = tab->g[i].tile_begin;
  if (threadIdx.x == 0) {
    for (int s = 0; s < kTvStages; ++s) {
      mbar_init(&bars->full[s], kTvFullArrivals);
      mbar_init(&bars->empty[s], kTvConsumers);
    }
    bars->abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();

  if (warp == kTvConsumers) {
    // ------------------------------------------------------------------ producer
    int it = 0;
    for (int tile = blockIdx.x; tile < ntiles && !*abort_flag; tile += gridDim.x) {
      const TvUnit u = tv_unit<MODE>(a, tab, s_tb, ngroups, tile, GS);
      if (u.ti.nrows > kTvMaxRows) {  // the host plans at most kTvMaxRows rows per unit; both roles skip it
        if (lane == 0) report(a.err, DEVERR_CONFIG);
        continue;
      }
      // this lane's activation row (lane < nrows) and scale rows (lane + 32 i)
      const uint16_t* xsrc = nullptr;
      if (lane < u.ti.nrows) {
        const int p = u.ti.row0 + lane;
        const int64_t src = (MODE == MODE_DOWN || u.sh) ? p : a.sorted_token[p];
        xsrc = (u.sh ? a.act_shared : a.act) + src * (u.sh ? a.act_shared_ld : a.act_ld);
      }
      const uint16_t* srow[4];
      const uint16_t* brow[4];
      bool rv[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int t = lane + 32 * i;
        const int row = tv_row<MODE>(u, t);
        const bool second = MODE == MODE_GATEUP && t >= 64;  // up rows
        const uint16_t* S = u.sh ? (second ? a.ss1 : a.ss0) : (second ? a.s1 : a.s0);
        const uint16_t* B = u.sh ? (second ? a.sb1 : a.sb0) : (second ? a.b1 : a.b0);
        rv[i] = row < u.N;
        const int64_t r = u.erow + (rv[i] ? row : 0);
        srow[i] = S + r * u.gpr;
        brow[i] = B ? B + r * u.gpr : nullptr;
      }
      const int map0 = u.sh ? 2 : 0;
      const int box_row = static_cast<int>(u.erow) + (MODE == MODE_GATEUP ? u.ti.rb * 64 : u.ti.rb * 128);
      for (int st = u.st0; st < u.st1; ++st, ++it) {
        const int slot = it % kTvStages;
        if (!__all_sync(0xffffffffu, mbar_wait(&bars->empty[slot], ((it / kTvStages) & 1) ^ 1, abort_flag, a.err)))
          break;
        const int kvalid = min(kTvStageK, u.K - st * kTvStageK);  // K positions of this stage
        const uint32_t xbytes = static_cast<uint32_t>(kvalid) * 2u;
        if (elect_one()) {
          mbar_arrive_expect_tx(&bars->full[slot], kTvCodeBytes + xbytes * u.ti.nrows);
          const uint32_t dst = smem_u32(smem + slot * kTvCodeBytes);
          tma_load_2d(dst, &maps.code[map0], st * 32, box_row, &bars->full[slot]);
          if (MODE == MODE_GATEUP) tma_load_2d(dst + 64 * 128, &maps.code[map0 + 1], st * 32, box_row, &bars->full[slot]);
        }
        __syncwarp();
        if (xsrc)
          bulk_load(smem_u32(smem + kTvOffX + slot * kTvXBytes + lane * kTvXPitch), xsrc + st * kTvStageK, xbytes,
                    &bars->full[slot]);
        // scales and biases of the stage's groups: [row][4] bf16 (G of them used)
        uint16_t* sc = reinterpret_cast<uint16_t*>(smem + kTvOffSb + slot * 2 * kTvSbBytes);
        uint16_t* bi = sc + kTvRows * 4;
        const int g0 = st * G;
        if ((u.gpr & 1) == 0) {  // pairs of groups are 4-byte aligned: copies, counted by the barrier
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const int t = lane + 32 * i;
#pragma unroll
            for (int g = 0; g < G; g += 2) {
              const bool in = rv[i] && g0 + g < u.gpr;
              cp_async4_zfill(smem_u32(sc + t * 4 + g), in ? srow[i] + g0 + g : srow[i], in ? 4u : 0u);
              cp_async4_zfill(smem_u32(bi + t * 4 + g), (in && brow[i]) ? brow[i] + g0 + g : srow[i],
                              (in && brow[i]) ? 4u : 0u);
            }
          }
          cp_async_arrive_noinc(&bars->full[slot]);
        } else {  // odd groups per row (group size 128): 2-byte loads
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const int t = lane + 32 * i;
#pragma unroll
            for (int g = 0; g < G; ++g) {
              const bool in = rv[i] && g0 + g < u.gpr;
              sc[t * 4 + g] = in ? __ldg(srow[i] + g0 + g) : static_cast<uint16_t>(0);
              bi[t * 4 + g] = (in && brow[i]) ? __ldg(brow[i] + g0 + g) : static_cast<uint16_t>(0);
            }
          }
          mbar_arrive(&bars->full[slot]);
        }
      }
    }
    // no copy may land after the CTA exits: wait (ignoring the abort flag) for the last
    // stages this warp issued
    for (int i = max(0, it - kTvStages); i < it; ++i)
      if (!__all_sync(0xffffffffu, wait_done(&bars->full[i % kTvStages], (i / kTvStages) & 1, a.err))) break;
    cp_async_wait<0>();
    __syncwarp();
    return;
  }

  // -------------------------------------------------------------------- consumers
  // Warp w owns one 16-row MMA tile of the unit: in gate/up mode the gate rows of
  // outputs 8w .. 8w + 7 (MMA rows g) and the up rows of the same outputs (rows g + 8),
  // so a thread holds both halves of its SwiGLUs; in down / plain mode rows 16w .. 16w + 15.
  const int g = lane >> 2, c = lane & 3;
  const int lr0 = MODE == MODE_GATEUP ? 8 * warp : 16 * warp;  // code row of MMA row 0
  // code-stage bytes from MMA row g to row g + 8: the up half (64 rows on) or 8 rows on
  constexpr uint32_t kRstep = MODE == MODE_GATEUP ? 64u * 128u : 8u * 128u;
  const int lr8 = MODE == MODE_GATEUP ? 64 + lr0 : lr0 + 8;    // code row of MMA row 8
  // this lane's bytes in a code stage: row lr0 + g, the 8-byte half c & 1 of its 16-byte
  // chunk, and per 64-wide half h the chunk 2h + c / 2 after the 128B swizzle (row & 7 == g)
  const uint32_t code_lane = static_cast<uint32_t>(lr0 + g) * 128u + 8u * static_cast<uint32_t>(c & 1);
  const uint32_t chunk_x = static_cast<uint32_t>(c >> 1) ^ static_cast<uint32_t>(g);  // (2h + c/2) ^ g == 2h ^ chunk_x
  const uint32_t x_lane = static_cast<uint32_t>(g) * kTvXPitch + 32u * static_cast<uint32_t>(c);
  int it = 0;
  for (int tile = blockIdx.x; tile < ntiles; tile += gridDim.x) {
    const TvUnit u = tv_unit<MODE>(a, tab, s_tb, ngroups, tile, GS);
    if (u.ti.nrows > kTvMaxRows) continue;  // reported by the producer
    const int ntn = (u.ti.nrows + 7) >> 3;  // 8-column MMA tiles of activation rows (1 or 2)
    float y[kTvNt][4];
#pragma unroll
    for (int n = 0; n < kTvNt; ++n) y[n][0] = y[n][1] = y[n][2] = y[n][3] = 0.f;
    bool ok = true;
    for (int st = u.st0; st < u.st1; ++st, ++it) {
      const int slot = it % kTvStages;
      if (!mbar_wait(&bars->full[slot], (it / kTvStages) & 1, abort_flag, a.err)) {
        ok = false;
        break;
      }
      const uint8_t* cs = smem + slot * kTvCodeBytes + code_lane;
      const uint8_t* xs = smem + kTvOffX + slot * kTvXBytes + x_lane;
      const uint16_t* sc = reinterpret_cast<const uint16_t*>(smem + kTvOffSb + slot * 2 * kTvSbBytes);
      const uint16_t* bi = sc + kTvRows * 4;
      const int nh = min(4, (u.K - st * kTvStageK) / 64);  // valid 64-wide halves (4, or 2 at a tail: K % 128 == 0)
      // scales / biases of the tile's rows g and g + 8: 4 groups each
      const uint2 S0 = *reinterpret_cast<const uint2*>(sc + (lr0 + g) * 4);
      const uint2 S1 = *reinterpret_cast<const uint2*>(sc + (lr8 + g) * 4);
      const uint2 B0 = *reinterpret_cast<const uint2*>(bi + (lr0 + g) * 4);
      const uint2 B1 = *reinterpret_cast<const uint2*>(bi + (lr8 + g) * 4);
      if (nh == 4) {
        if (ntn == 1) tv_stage<GS, 1, 4>(cs, kRstep, chunk_x, xs, S0, S1, B0, B1, y);
        else tv_stage<GS, 2, 4>(cs, kRstep, chunk_x, xs, S0, S1, B0, B1, y);
      } else {
        if (ntn == 1) tv_stage<GS, 1, 2>(cs, kRstep, chunk_x, xs, S0, S1, B0, B1, y);
        else tv_stage<GS, 2, 2>(cs, kRstep, chunk_x, xs, S0, S1, B0, B1, y);
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars->empty[slot]);
    }
    if (!ok) break;

    // epilogue: y[n][e] is (MMA row g + 8 (e >> 1), activation row 8n + 2c + (e & 1))
    if (MODE == MODE_GATEUP) {
      const int nn = u.ti.rb * 64 + lr0 + g;  // output (gate row e < 2, up row e >= 2)
      if (u.ti.rb * 64 + lr0 < u.N) {         // N % 8 == 0: the warp's 8 outputs are in or out together
#pragma unroll
        for (int n = 0; n < kTvNt; ++n) {
          if (n >= ntn) break;
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const int slot_r = 8 * n + 2 * c + e;
            if (slot_r >= u.ti.nrows) continue;
            const int p = u.ti.row0 + slot_r;
            const float gv = rbf(y[n][e]), uv = rbf(y[n][e + 2]);
            uint16_t* out = u.sh ? a.out_shared + static_cast<int64_t>(p) * a.out_shared_ld
                                 : a.out + static_cast<int64_t>(p) * a.out_ld;
            out[perm8(nn)] = f2bf(swiglu_1(gv, uv));
          }
        }
      }
    } else {
      const int n0 = u.ti.rb * 128 + lr0;
      if (n0 < u.N) {  // N % 16 == 0
#pragma unroll
        for (int n = 0; n < kTvNt; ++n) {
          if (n >= ntn) break;
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int slot_r = 8 * n + 2 * c + (e & 1);
            if (slot_r >= u.ti.nrows) continue;
            const int p = u.ti.row0 + slot_r;
            const int nn = n0 + g + 8 * (e >> 1);
            const float v = y[n][e];
            if (MODE == MODE_DOWN) {
              if (u.sh) {
                red_add_f32(a.ysh + static_cast<int64_t>(p) * a.y_ld + nn, v);
              } else if (a.y_rowptr) {  // one output row per pair, at its destination (peer memory)
                a.y_rowptr[p][nn] = f2bf(rbf(rbf(v) * a.sorted_score[p]));
              } else if (a.y_pairs) {  // one output row per pair (expert-parallel owner side)
                a.y_pairs[static_cast<int64_t>(p) * a.y_ld + nn] = f2bf(rbf(rbf(v) * a.sorted_score[p]));
              } else {
                const int t = a.sorted_token[p];
                red_add_f32(a.y_acc + static_cast<int64_t>(t) * a.y_ld + nn, rbf(rbf(v) * a.sorted_score[p]));
              }
            } else {
              a.out[static_cast<int64_t>(a.sorted_flat[p]) * a.out_ld + nn] = f2bf(v);
            }
          }
        }
      }
    }
  }
}

namespace {
template <int MODE, int GS>
cudaError_t tv_launch(int grid, cudaStream_t stream, const GemmArgs& a, const TcMaps& maps) {
  // the shared-memory opt-in, once per device (setting it again is harmless)
  static bool attr_set[64] = {};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 64 || !attr_set[dev]) {
    e = cudaFuncSetAttribute(qgemv_tma_kernel<MODE, GS>, cudaFuncAttributeMaxDynamicSharedMemorySize, kTvSmemBytes);
    if (e != cudaSuccess) return e;
    if (dev >= 0 && dev < 64) attr_set[dev] = true;
  }
  qgemv_tma_kernel<MODE, GS><<<grid, kTvThreads, kTvSmemBytes, stream>>>(a, maps);
  return cudaGetLastError();
}
}  // namespace

bool qgemv_tma_supports(int mode, int K, int K_shared, int gs) {
  if (mode != MODE_GATEUP && mode != MODE_DOWN && mode != MODE_PLAIN) return false;
  if (gs != 64 && gs != 128) return false;
  return K % 128 == 0 && K_shared % 128 == 0;
}

// grid: resident CTAs (blocks_per_sm x SMs); persistent over the tile table
cudaError_t launch_qgemv_tma(int mode, int grid, cudaStream_t stream, const GemmArgs& a, const TcMaps& maps) {
  const bool g128 = a.gs == 128;
  switch (mode) {
    case MODE_GATEUP: return g128 ? tv_launch<MODE_GATEUP, 128>(grid, stream, a, maps)
                                  : tv_launch<MODE_GATEUP, 64>(grid, stream, a, maps);
    case MODE_DOWN: return g128 ? tv_launch<MODE_DOWN, 128>(grid, stream, a, maps)
                                : tv_launch<MODE_DOWN, 64>(grid, stream, a, maps);
    case MODE_PLAIN: return g128 ? tv_launch<MODE_PLAIN, 128>(grid, stream, a, maps)
                                 : tv_launch<MODE_PLAIN, 64>(grid, stream, a, maps);
    default: return cudaErrorInvalidValue;
  }
}

cudaError_t qgemv_tma_blocks_per_sm(int* n) {
  cudaError_t e = cudaFuncSetAttribute(qgemv_tma_kernel<MODE_GATEUP, 64>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       kTvSmemBytes);
  if (e != cudaSuccess) return e;
  return cudaOccupancyMaxActiveBlocksPerMultiprocessor(n, qgemv_tma_kernel<MODE_GATEUP, 64>, kTvThreads, kTvSmemBytes);
}

int qgemv_tma_max_rows() { return kTvMaxRows; }

}  // namespace fm
