// qgemm_tc.cu -- grouped 4-bit expert GEMM on the 5th-generation tensor cores.
//
// Replaces mx::gather_qmm (sorted, model.cpp:703-721) and mx::quantized_matmul
// (model.cpp:741-747) for prefill-sized batches.  One persistent CTA per SM walks a
// device-built tile table (expert / shared-expert group, 128-row output block, chunk
// of <= 192 activation rows).  D[128 x N] accumulates in TMEM:
//   gate/up mode: A rows 0..63 = gate rows, 64..127 = the same up rows, so one
//                 accumulator holds g and u of a row block; the epilogue applies
//                 silu(g)*u and writes the pair-permuted activation rows for down.
//   down mode:    A = 128 down rows; the epilogue rounds d, scales by the routing
//                 weight and red.adds into the fp32 combine buffer (token-indexed).
//   plain mode:   quantized_matmul / gather_qmm output, bf16.
//
// Data movement: the packed 4-bit codes arrive by TMA, 4 k-steps (128 B x 128 rows)
// per load, 128B-swizzled, into a 3-deep ring.  Contiguous activation rows (down
// projection, shared expert) arrive by TMA in 64-row boxes straight into the UMMA B
// stage; token-gathered rows are copied with cp.async (the TMA unit's per-instruction
// cost makes 4-row gather4 boxes too slow at 36-48 instructions per k-step).
//
// Roles (512 threads):
//   warps 0-7   dequant producers: thread t owns half of A row t/2.  Per k-step: one
//               16-byte code read, bf16 fma of the exact codes with the group's scale
//               and bias (prefetched in registers a super-step ahead), four 16-byte
//               stores into the 128B-swizzled K-major A stage.
//   warp 8      code loader (one lane issues the TMA of each super-step).
//   warps 9-10  activation loaders: cp.async gather of token rows (24 per thread, row
//               indices in registers) or TMA of contiguous 64-row boxes.
//   warp 11     TMEM allocator and single-thread tcgen05.mma issuer (M=128, N<=192,
//               K=16 x 4 per stage); tcgen05.commit frees stages / publishes tiles.
//   warps 12-15 epilogue: tcgen05.ld of the four 32-lane TMEM quadrants; double-
//               buffered accumulators (2 x 256 columns) overlap the next mainloop.
// No cluster multicast anywhere; every TMA source is this GPU's own memory.  Every
// wait is bounded.
#include "fm_internal.cuh"

namespace fm {
namespace tc {

constexpr int BM = 128;
constexpr int BN = 192;          // max activation rows per tile (MMA N)
constexpr int ACC_COLS = 256;    // TMEM columns per accumulator buffer
constexpr int STAGES = 4;
constexpr int NC = 3;            // code ring depth (super-steps of 4 k-steps)
constexpr int KS_PER_SS = 4;
constexpr int A_BYTES = BM * 128;
constexpr int B_BYTES = BN * 128;
constexpr int C_BYTES = BM * 128;  // 128 rows x 32 words
constexpr int XCHG_HALF = 16 * 64 * 2;
constexpr int OFF_A = 0;
constexpr int OFF_B = OFF_A + STAGES * A_BYTES;
constexpr int OFF_C = OFF_B + STAGES * B_BYTES;
constexpr int OFF_XCHG = OFF_C + NC * C_BYTES;
constexpr int OFF_TB = OFF_XCHG + 4 * XCHG_HALF;     // tile_begin of every group
constexpr int OFF_BAR = OFF_TB + ((kMaxGroups * 4 + 255) / 256) * 256;
constexpr int BAR_BYTES = 256;
constexpr int SMEM_BYTES = OFF_BAR + BAR_BYTES + 1024;  // + alignment slack
constexpr int NA = 256;          // dequant-producer threads (two per A row)
constexpr int CODE_WARP = 8;
constexpr int ACT_WARP = 9;      // two activation-loader warps: 9 and 10
constexpr int NB = 64;
constexpr int B_ROWS = BN / 8;   // rows per activation-loader thread (24)
constexpr int B_LAG = 2;
constexpr int MMA_WARP = 11;
constexpr int EPI_WARP = 12;     // first of the four epilogue warps (TMEM lane quadrant = warp % 4)
constexpr int THREADS = (EPI_WARP + 4) * 32;
constexpr uint32_t TMEM_COLS = 512;

static_assert(OFF_B % 1024 == 0 && OFF_C % 1024 == 0 && B_BYTES % 1024 == 0, "1 KB aligned stages");

struct Bars {
  uint64_t full[STAGES];
  uint64_t empty[STAGES];
  uint64_t cfull[NC];
  uint64_t cempty[NC];
  uint64_t accf[2];
  uint64_t acce[2];
  uint64_t done;
  uint32_t tmem_base;
  int abort;
  int epi_ok[2][4];
};
static_assert(sizeof(Bars) <= BAR_BYTES, "barrier block");

FM_DEV int tile_ksteps(const GemmArgs& a, const TileInfo& ti, int mode) {
  const int K = (mode == MODE_DOWN && ti.expert < 0) ? a.K_shared : a.K;
  return K / 64;
}

// iterator over the (tile, super-step) pairs of this CTA
struct SIter {
  int tile;
  int ss;
  int nss;
  int nks;
  TileInfo ti;
  bool valid;
};

// tile table with a shared-memory copy of the groups' first tile ids
struct TileDir {
  const TileTable* tab;
  const int* tb;
  int ng;
  FM_DEV TileInfo get(int tile) const { return decode_tile(tab, tb, ng, tile); }
};

FM_DEV void siter_load(SIter& it, const GemmArgs& a, const TileDir& dir, int tile, int ntiles, int mode) {
  it.tile = tile;
  it.ss = 0;
  it.valid = tile < ntiles;
  if (it.valid) {
    it.ti = dir.get(tile);
    it.nks = tile_ksteps(a, it.ti, mode);
    it.nss = (it.nks + KS_PER_SS - 1) / KS_PER_SS;
  }
}

FM_DEV void siter_next(SIter& it, const GemmArgs& a, const TileDir& dir, int ntiles, int mode) {
  if (!it.valid) return;
  if (++it.ss >= it.nss) siter_load(it, a, dir, it.tile + gridDim.x, ntiles, mode);
}

FM_DEV bool wait_done(uint64_t* bar, uint32_t parity, uint32_t* err) {  // ignores abort
  const long long t0 = clock64();
  while (!mbar_try_wait(bar, parity)) {
    if (clock64() - t0 > kWaitBudgetCycles) {
      report(err, DEVERR_TIMEOUT);
      return false;
    }
  }
  return true;
}

// silu(g) * u with the bf16 rounding of each MLX op (model.cpp:14-25); g, u already bf16
FM_DEV float swiglu1(float g, float u) {
  const float sg = rbf(__frcp_rn(1.0f + __expf(-g)));
  const float h = rbf(g * sg);
  return rbf(h * u);
}

FM_DEV void red_add_v2(float* p, float a, float b) {
  asm volatile("red.global.add.v2.f32 [%0], {%1, %2};" ::"l"(p), "f"(a), "f"(b) : "memory");
}

// A row t (0..127 of the tile) -> row inside its weight matrix, and the matrix's
// scale / bias arrays
template <int MODE>
FM_DEV void a_row_info(const GemmArgs& a, const TileInfo& ti, int t, int& row, const uint16_t*& S,
                       const uint16_t*& B) {
  const bool sh = ti.expert < 0;
  if (MODE == MODE_GATEUP) {
    const bool up = t >= 64;
    row = ti.rb * 64 + (t & 63);
    S = up ? (sh ? a.ss1 : a.s1) : (sh ? a.ss0 : a.s0);
    B = up ? (sh ? a.sb1 : a.b1) : (sh ? a.sb0 : a.b0);
  } else {
    row = ti.rb * 128 + t;
    S = sh ? a.ss0 : a.s0;
    B = sh ? a.sb0 : a.b0;
  }
}

// Scale / bias of the group each of the super-step's (up to) 4 k-steps uses for this
// thread's half row (one group per half k-step for group sizes 32 / 64 / 128).
template <int MODE>
FM_DEV void load_scales(const GemmArgs& a, const SIter& it, int t, int half, uint32_t (&sv)[4], uint32_t (&bv)[4]) {
#pragma unroll
  for (int kk = 0; kk < 4; ++kk) sv[kk] = bv[kk] = 0u;
  if (!it.valid) return;
  const TileInfo& ti = it.ti;
  const bool sh = ti.expert < 0;
  const int K = (MODE == MODE_DOWN && sh) ? a.K_shared : a.K;
  const int N = sh ? a.N_shared : a.N;
  int row;
  const uint16_t* S;
  const uint16_t* B;
  a_row_info<MODE>(a, ti, t, row, S, B);
  if (row >= N) return;
  const int gpr = K / a.gs;
  const int64_t r = (sh ? 0 : static_cast<int64_t>(ti.expert) * N) + row;
  const uint16_t* srow = S + r * gpr;
  const uint16_t* brow = B ? B + r * gpr : nullptr;
  if (a.gs == 64 && (gpr & 1) == 0) {
    // groups g0..g0+3 as two 4-byte aligned pairs
    const int g0 = it.ss * KS_PER_SS;
    const uint32_t s0 = g0 < gpr ? __ldg(reinterpret_cast<const uint32_t*>(srow + g0)) : 0u;
    const uint32_t s1 = g0 + 2 < gpr ? __ldg(reinterpret_cast<const uint32_t*>(srow + g0 + 2)) : 0u;
    const uint32_t b0 = (brow && g0 < gpr) ? __ldg(reinterpret_cast<const uint32_t*>(brow + g0)) : 0u;
    const uint32_t b1 = (brow && g0 + 2 < gpr) ? __ldg(reinterpret_cast<const uint32_t*>(brow + g0 + 2)) : 0u;
    sv[0] = s0 & 0xffffu; sv[1] = s0 >> 16; sv[2] = s1 & 0xffffu; sv[3] = s1 >> 16;
    bv[0] = b0 & 0xffffu; bv[1] = b0 >> 16; bv[2] = b1 & 0xffffu; bv[3] = b1 >> 16;
  } else {
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      const int ks = it.ss * KS_PER_SS + kk;
      if (ks < it.nks) {
        const int g = (ks * 64 + 32 * half) / a.gs;
        sv[kk] = __ldg(srow + g);
        bv[kk] = brow ? __ldg(brow + g) : 0u;
      }
    }
  }
}

template <int MODE>
__global__ void __launch_bounds__(THREADS, 1) qgemm_tc_kernel(const GemmArgs a, const __grid_constant__ TcMaps maps) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  Bars* bars = reinterpret_cast<Bars*>(smem + OFF_BAR);
  const int tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31;
  // an earlier kernel of this call reported a device error: the tile table is not trusted
  const int ntiles = (*reinterpret_cast<volatile uint32_t*>(a.err) != 0u) ? 0 : a.tab->num_tiles;
  volatile int* abort_flag = &bars->abort;

  if (tid == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&bars->full[s], NA + NB);
      mbar_init(&bars->empty[s], 1);
    }
    for (int c = 0; c < NC; ++c) {
      mbar_init(&bars->cfull[c], 1);
      mbar_init(&bars->cempty[c], NA / 32);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&bars->accf[b], 1);
      mbar_init(&bars->acce[b], 4);
    }
    mbar_init(&bars->done, 1);
    bars->abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == MMA_WARP) {
    tmem_alloc(&bars->tmem_base, TMEM_COLS);
    tmem_relinquish();
  }
  int* s_tb = reinterpret_cast<int*>(smem + OFF_TB);
  const int ngroups = ntiles > 0 ? min(a.tab->num_groups, kMaxGroups) : 0;
  for (int i = tid; i < ngroups; i += THREADS) s_tb[i] = a.tab->g[i].tile_begin;
  const TileDir dir{a.tab, s_tb, ngroups};
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = bars->tmem_base;

  if (warp < NA / 32) {
    // ------------------------------------------------------------ dequant producers
    const int t = tid >> 1;    // A row
    const int half = tid & 1;  // 16-byte half of the row's 32 bytes of codes per k-step
    SIter cur;
    siter_load(cur, a, dir, blockIdx.x, ntiles, MODE);
    uint32_t sv[4], bv[4];
    load_scales<MODE>(a, cur, t, half, sv, bv);
    int cs = 0, it = 0;
    bool ok = true;
    while (cur.valid && ok) {
      SIter nx = cur;
      siter_next(nx, a, dir, ntiles, MODE);
      uint32_t nsv[4], nbv[4];
      load_scales<MODE>(a, nx, t, half, nsv, nbv);  // a super-step ahead
      const int slot = cs % NC;
      if (!mbar_wait(&bars->cfull[slot], (cs / NC) & 1, abort_flag, a.err)) break;
      const TileInfo& ti = cur.ti;
      const bool sh = ti.expert < 0;
      const int N = sh ? a.N_shared : a.N;
      const int row = (MODE == MODE_GATEUP) ? ti.rb * 64 + (t & 63) : ti.rb * 128 + t;
      const uint8_t* code = smem + OFF_C + slot * C_BYTES + t * 128;
      const int nk = min(KS_PER_SS, cur.nks - cur.ss * KS_PER_SS);
#pragma unroll
      for (int kk = 0; kk < KS_PER_SS; ++kk) {
        if (kk >= nk) break;
        const int stage = it % STAGES;
        if (!mbar_wait(&bars->empty[stage], ((it / STAGES) & 1) ^ 1, abort_flag, a.err)) {
          ok = false;
          break;
        }
        if (row < N) {
          const uint4 w = *reinterpret_cast<const uint4*>(code + (((2 * kk + half) ^ (t & 7)) << 4));
          const uint32_t s2u = sv[kk] * 0x10001u, b2u = bv[kk] * 0x10001u;
          const __nv_bfloat162 s2 = *reinterpret_cast<const __nv_bfloat162*>(&s2u);
          const __nv_bfloat162 b2 = *reinterpret_cast<const __nv_bfloat162*>(&b2u);
          const uint32_t words[4] = {w.x, w.y, w.z, w.w};
          uint8_t* As = smem + OFF_A + stage * A_BYTES;
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            uint4 o;
            o.x = deq_pair(words[i], 0, s2, b2);
            o.y = deq_pair(words[i], 1, s2, b2);
            o.z = deq_pair(words[i], 2, s2, b2);
            o.w = deq_pair(words[i], 3, s2, b2);
            *reinterpret_cast<uint4*>(As + sw128_off(t, half * 4 + i)) = o;
          }
        }
        fence_proxy_async();
        mbar_arrive(&bars->full[stage]);
        ++it;
      }
      if (!ok) break;
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars->cempty[slot]);
      ++cs;
      cur = nx;
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
        sv[kk] = nsv[kk];
        bv[kk] = nbv[kk];
      }
    }
  } else if (warp == CODE_WARP) {
    // ------------------------------------------------------------ code loader (TMA)
    if (lane == 0) {
      SIter cur;
      siter_load(cur, a, dir, blockIdx.x, ntiles, MODE);
      int cs = 0;
      while (cur.valid) {
        const int slot = cs % NC;
        if (!mbar_wait(&bars->cempty[slot], ((cs / NC) & 1) ^ 1, abort_flag, a.err)) break;
        const TileInfo& ti = cur.ti;
        const bool sh = ti.expert < 0;
        const int N = sh ? a.N_shared : a.N;
        const int erow = sh ? 0 : ti.expert * N;
        const uint32_t dst = smem_u32(smem + OFF_C + slot * C_BYTES);
        const int x = cur.ss * (KS_PER_SS * 8);
        mbar_arrive_expect_tx(&bars->cfull[slot], C_BYTES);
        if (MODE == MODE_GATEUP) {
          const int r0 = erow + ti.rb * 64;
          tma_load_2d(dst, &maps.code[sh ? 2 : 0], x, r0, &bars->cfull[slot]);
          tma_load_2d(dst + 64 * 128, &maps.code[sh ? 3 : 1], x, r0, &bars->cfull[slot]);
        } else {
          tma_load_2d(dst, &maps.code[sh ? 2 : 0], x, erow + ti.rb * 128, &bars->cfull[slot]);
        }
        ++cs;
        siter_next(cur, a, dir, ntiles, MODE);
      }
    }
    __syncwarp();
  } else if (warp == ACT_WARP || warp == ACT_WARP + 1) {
    // ------------------------------------------------------------ activation loaders
    const int bt = tid - ACT_WARP * 32;   // 0..63
    const int cc = bt & 7, rg = bt >> 3;  // 16-byte chunk, first row (rows rg + 8 i)
    // swizzled destination of row rg + 8 i: (rg + 8 i) * 128 + ((cc ^ rg) << 4)
    const uint32_t dst0 = static_cast<uint32_t>(rg) * 128u + (static_cast<uint32_t>(cc ^ rg) << 4);
    int it = 0, pend = 0;  // pend: oldest k-step whose cp.async rows are not yet published
    bool ok = true;
    for (int tile = blockIdx.x; tile < ntiles && ok; tile += gridDim.x) {
      const TileInfo ti = dir.get(tile);
      const bool sh = ti.expert < 0;
      const int nks = tile_ksteps(a, ti, MODE);
      const bool gather = (MODE != MODE_DOWN) && !sh;
      uint32_t srow[B_ROWS];
      const uint16_t* base = sh ? a.act_shared : a.act;
      const uint64_t ld_bytes = static_cast<uint64_t>(sh ? a.act_shared_ld : a.act_ld) * 2u;
      if (gather) {
#pragma unroll
        for (int i = 0; i < B_ROWS; ++i) {
          const int r = rg + 8 * i;
          srow[i] = (r < ti.nrows) ? static_cast<uint32_t>(a.sorted_token[ti.row0 + r]) : 0u;
        }
      }
      const int nblk = (ti.nrows + 63) >> 6;
      for (int ks = 0; ks < nks; ++ks) {
        const int stage = it % STAGES;
        if (!mbar_wait(&bars->empty[stage], ((it / STAGES) & 1) ^ 1, abort_flag, a.err)) {
          ok = false;
          break;
        }
        if (gather) {
          const uint32_t bs = smem_u32(smem + OFF_B + stage * B_BYTES) + dst0;
          const uint64_t src_k = reinterpret_cast<uint64_t>(base) + static_cast<uint64_t>(ks * 128 + cc * 16);
#pragma unroll
          for (int i = 0; i < B_ROWS; ++i) {
            if (rg + 8 * i < ti.nrows)
              cp_async16(bs + static_cast<uint32_t>(i) * 1024u,
                         reinterpret_cast<const void*>(src_k + static_cast<uint64_t>(srow[i]) * ld_bytes));
          }
          cp_async_commit();
          if (it - pend >= B_LAG) {  // publish the k-step B_LAG behind
            cp_async_wait<B_LAG>();
            fence_proxy_async();
            mbar_arrive(&bars->full[pend % STAGES]);
            ++pend;
          }
        } else {
          if (pend < it) {  // publish every gathered k-step still in flight
            cp_async_wait<0>();
            fence_proxy_async();
            for (; pend < it; ++pend) mbar_arrive(&bars->full[pend % STAGES]);
          }
          if (bt == 0) {
            mbar_arrive_expect_tx(&bars->full[stage], static_cast<uint32_t>(nblk) * 8192u);
            const uint32_t bs = smem_u32(smem + OFF_B + stage * B_BYTES);
            const CUtensorMap* map = &maps.act[sh ? 1 : 0];
            for (int b = 0; b < nblk; ++b)
              tma_load_2d(bs + b * 8192, map, ks * 64, ti.row0 + b * 64, &bars->full[stage]);
          } else {
            mbar_arrive(&bars->full[stage]);
          }
          pend = it + 1;
        }
        ++it;
      }
    }
    cp_async_wait<0>();
    fence_proxy_async();
    for (; pend < it; ++pend) mbar_arrive(&bars->full[pend % STAGES]);
  } else if (warp == MMA_WARP) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      int it = 0, lt = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < ntiles && ok; tile += gridDim.x, ++lt) {
        const TileInfo ti = dir.get(tile);
        const int nks = tile_ksteps(a, ti, MODE);
        const int buf = lt & 1;
        if (!mbar_wait(&bars->acce[buf], ((lt >> 1) & 1) ^ 1, abort_flag, a.err)) break;
        tc_fence_after();
        const int nmma = max(16, (ti.nrows + 15) & ~15);
        const uint32_t idesc = idesc_bf16(BM, nmma);
        const uint32_t d = tmem_base + static_cast<uint32_t>(buf * ACC_COLS);
        for (int ks = 0; ks < nks; ++ks) {
          const int stage = it % STAGES;
          if (!mbar_wait(&bars->full[stage], (it / STAGES) & 1, abort_flag, a.err)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t ad = sdesc_sw128(smem_u32(smem + OFF_A + stage * A_BYTES));
          const uint64_t bd = sdesc_sw128(smem_u32(smem + OFF_B + stage * B_BYTES));
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) umma_bf16(d, ad + 2 * kk, bd + 2 * kk, idesc, (ks | kk) != 0);
          umma_commit(&bars->empty[stage]);
          ++it;
        }
        if (ok) umma_commit(&bars->accf[buf]);
      }
      umma_commit(&bars->done);
      wait_done(&bars->done, 0, a.err);
    }
    __syncwarp();
  } else if (warp >= EPI_WARP && warp < EPI_WARP + 4) {
    // ------------------------------------------------------------ epilogue
    const int q = warp - EPI_WARP;
    const int row_in = q * 32 + lane;  // TMEM lane == A row
    uint16_t* xchg = reinterpret_cast<uint16_t*>(smem + OFF_XCHG);
    int lt = 0, xit = 0;
    for (int tile = blockIdx.x; tile < ntiles; tile += gridDim.x, ++lt) {
      const TileInfo ti = dir.get(tile);
      const bool sh = ti.expert < 0;
      const int N = sh ? a.N_shared : a.N;
      const int buf = lt & 1;
      const bool got = mbar_wait(&bars->accf[buf], (lt >> 1) & 1, abort_flag, a.err);
      // make the go / no-go decision uniform across the four epilogue warps
      if (lane == 0) bars->epi_ok[buf][q] = got ? 1 : 0;
      named_bar_sync(1, 128);
      const bool all_ok = bars->epi_ok[buf][0] && bars->epi_ok[buf][1] && bars->epi_ok[buf][2] && bars->epi_ok[buf][3];
      if (!all_ok) break;
      tc_fence_after();
      const uint32_t tbase = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + static_cast<uint32_t>(buf * ACC_COLS);
      const int nchunks = (ti.nrows + 31) >> 5;
      for (int j = 0; j < nchunks; ++j, ++xit) {
        float v[32];
        tmem_ld32(tbase + j * 32, v);
        if (MODE == MODE_GATEUP) {
          // gate warps (q 0,1) finish columns 0..15, up warps (q 2,3) columns 16..31;
          // each hands the partner the other half of its rows through shared memory
          uint16_t* to_up = xchg + (xit & 1) * (2 * 16 * 64);  // gate values, cols 16..31
          uint16_t* to_gate = to_up + 16 * 64;                  // up values, cols 0..15
          const int r64 = row_in & 63;
          if (q < 2) {
#pragma unroll
            for (int c = 0; c < 16; ++c) to_up[c * 64 + r64] = f2bf(v[16 + c]);
          } else {
#pragma unroll
            for (int c = 0; c < 16; ++c) to_gate[c * 64 + r64] = f2bf(v[c]);
          }
          named_bar_sync(1, 128);
          const int n = ti.rb * 64 + r64;
          uint16_t* outb = sh ? a.out_shared : a.out;
          const int64_t ld = sh ? a.out_shared_ld : a.out_ld;
          const int pn = perm8(n);  // even for n % 8 < 4: (n, n+4) share one 32-bit word
          const int c0 = (q < 2) ? 0 : 16;
          uint32_t res[16];  // all 16 columns first: independent chains for the scheduler
#pragma unroll
          for (int c = 0; c < 16; ++c) {
            float gv, uv;
            if (q < 2) {
              gv = rbf(v[c]);
              uv = bf2f(to_gate[c * 64 + r64]);
            } else {
              gv = bf2f(to_up[c * 64 + r64]);
              uv = rbf(v[16 + c]);
            }
            res[c] = f2bf(swiglu1(gv, uv));
          }
          uint16_t* orow = outb + static_cast<int64_t>(ti.row0 + j * 32 + c0) * ld + pn;
#pragma unroll
          for (int c = 0; c < 16; ++c) {
            const uint32_t other = __shfl_xor_sync(0xffffffffu, res[c], 4);
            if (j * 32 + c0 + c < ti.nrows && (lane & 4) == 0 && n < N)
              *reinterpret_cast<uint32_t*>(orow + static_cast<int64_t>(c) * ld) = res[c] | (other << 16);
          }
        } else {
          // lanes (2m, 2m+1) hold rows (n, n+1); the even lane finishes column c and
          // the odd lane column c+1, each as one 2-wide red / 4-byte store
          const int n = ti.rb * 128 + row_in;
          const bool odd = lane & 1;
          const int n0 = n & ~1;
          // lane c fetches column c's metadata once; the loop reads it by shuffle
          const int pc = ti.row0 + min(j * 32 + lane, ti.nrows - 1);
          const float my_score = (MODE == MODE_DOWN && !sh) ? a.sorted_score[pc] : 1.f;
          const int my_dst = (MODE == MODE_DOWN) ? (sh ? pc : a.sorted_token[pc]) : a.sorted_flat[pc];
#pragma unroll
          for (int c = 0; c < 32; c += 2) {
            const int col = j * 32 + c + (odd ? 1 : 0);
            const bool colok = col < ti.nrows;
            const int dst_row = __shfl_sync(0xffffffffu, my_dst, c + (odd ? 1 : 0));
            float mine_c = v[c], mine_c1 = v[c + 1];
            if (MODE == MODE_DOWN && !sh) {  // bf16(bf16(d) * score) per MLX op
              const float se = __shfl_sync(0xffffffffu, my_score, c);
              const float so = __shfl_sync(0xffffffffu, my_score, c + 1);
              mine_c = rbf(rbf(mine_c) * se);
              mine_c1 = rbf(rbf(mine_c1) * so);
            }
            // even lane sends its column c+1 value, odd lane its column c value
            const float give = odd ? mine_c : mine_c1;
            const float got2 = __shfl_xor_sync(0xffffffffu, give, 1);
            const float lo = odd ? got2 : mine_c;    // row n0, column (c or c+1)
            const float hi = odd ? mine_c1 : got2;   // row n0+1
            if (!colok || n0 >= N) continue;
            if (MODE == MODE_DOWN) {
              if (sh)  // each shared-expert element is produced by exactly one tile
                *reinterpret_cast<float2*>(a.ysh + static_cast<int64_t>(dst_row) * a.y_ld + n0) = make_float2(lo, hi);
              else
                red_add_v2(a.y_acc + static_cast<int64_t>(dst_row) * a.y_ld + n0, lo, hi);
            } else {
              *reinterpret_cast<uint32_t*>(a.out + static_cast<int64_t>(dst_row) * a.out_ld + n0) = pack_bf16x2(lo, hi);
            }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars->acce[buf]);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == MMA_WARP) {
    tc_fence_after();
    tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

int max_rows() { return BN; }

cudaError_t init() {
  cudaError_t e = cudaFuncSetAttribute(qgemm_tc_kernel<MODE_GATEUP>, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(qgemm_tc_kernel<MODE_DOWN>, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(qgemm_tc_kernel<MODE_PLAIN>, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
  return e;
}

cudaError_t launch(int mode, int grid, cudaStream_t stream, const GemmArgs& a, const TcMaps& maps) {
  switch (mode) {
    case MODE_GATEUP: qgemm_tc_kernel<MODE_GATEUP><<<grid, THREADS, SMEM_BYTES, stream>>>(a, maps); break;
    case MODE_DOWN: qgemm_tc_kernel<MODE_DOWN><<<grid, THREADS, SMEM_BYTES, stream>>>(a, maps); break;
    default: qgemm_tc_kernel<MODE_PLAIN><<<grid, THREADS, SMEM_BYTES, stream>>>(a, maps); break;
  }
  return cudaGetLastError();
}

}  // namespace tc
}  // namespace fm
