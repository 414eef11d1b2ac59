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
// Roles (544 threads; the producer / consumer roles spread over the 4 SM sub-partitions):
//   warps 0-7   dequant producers: thread t owns half of A row t/2.  Codes, scales and
//               biases of k-step s+9 stream into a private cp.async ring (deep enough
//               to cover HBM latency under load); k-step s is dequantized (bf16 fma of
//               exact codes) into the 128B-swizzled K-major A stage.
//   warps 8-11  activation producers: cp.async gather of up to 192 rows x 128 B per
//               k-step into the swizzled B stage; each thread keeps its 12 rows'
//               indices in registers (one wide multiply-add per copy).
//   warps 12-15 epilogue: tcgen05.ld of the four 32-lane TMEM quadrants; double-
//               buffered accumulators (2 x 256 columns) overlap the next mainloop.
//   warp 16     TMEM allocator and single-thread tcgen05.mma issuer (M=128, N<=192,
//               K=16 x 4 per stage); tcgen05.commit frees stages / publishes tiles.
// No TMA and no cluster multicast anywhere.  Every wait is bounded.
#include "fm_internal.cuh"

namespace fm {
namespace tc {

constexpr int BM = 128;
constexpr int BN = 192;          // max activation rows per tile (MMA N)
constexpr int ACC_COLS = 256;    // TMEM columns per accumulator buffer
constexpr int STAGES = 4;
constexpr int NRING = 10;
constexpr int A_BYTES = BM * 128;
constexpr int B_BYTES = BN * 128;
constexpr int RING_CODES = BM * 32;             // packed codes of one k-step
constexpr int RING_BYTES = RING_CODES + BM * 8; // + scale pair + bias pair per row
constexpr int XCHG_HALF = 16 * 64 * 2;          // 16 columns x 64 rows, bf16
constexpr int OFF_A = 0;
constexpr int OFF_B = OFF_A + STAGES * A_BYTES;
constexpr int OFF_RING = OFF_B + STAGES * B_BYTES;
constexpr int OFF_XCHG = OFF_RING + NRING * RING_BYTES;
constexpr int OFF_BAR = OFF_XCHG + 4 * XCHG_HALF;  // {gate->up, up->gate} x 2 buffers
constexpr int BAR_BYTES = 256;
constexpr int SMEM_BYTES = OFF_BAR + BAR_BYTES + 1024;  // + alignment slack
constexpr int NA = 256;          // dequant-producer threads (two per A row)
constexpr int NB = 128;          // activation-producer threads
constexpr int B_ROWS = BN * 8 / NB;  // rows per activation-producer thread (12)
constexpr int EPI_WARP = 12;     // first of the four epilogue warps
constexpr int MMA_WARP = 16;
constexpr int THREADS = (MMA_WARP + 1) * 32;
constexpr int B_LAG = 2;
constexpr uint32_t TMEM_COLS = 512;

struct Bars {
  uint64_t full[STAGES];
  uint64_t empty[STAGES];
  uint64_t accf[2];
  uint64_t acce[2];
  uint64_t done;
  uint32_t tmem_base;
  int abort;
  int epi_ok[2][4];
};

// iterator over (tile, k-step) pairs of this CTA
struct KIter {
  int tile;
  int ks;
  int nks;
  TileInfo ti;
  bool valid;
};

FM_DEV int tile_ksteps(const GemmArgs& a, const TileInfo& ti, int mode) {
  const int K = (mode == MODE_DOWN && ti.expert < 0) ? a.K_shared : a.K;
  return K / 64;
}

FM_DEV void kiter_load(KIter& it, const GemmArgs& a, int tile, int ntiles, int mode) {
  it.tile = tile;
  it.ks = 0;
  it.valid = tile < ntiles;
  if (it.valid) {
    it.ti = decode_tile(a.tab, tile);
    it.nks = tile_ksteps(a, it.ti, mode);
  }
}

FM_DEV void kiter_next(KIter& it, const GemmArgs& a, int ntiles, int mode) {
  if (!it.valid) return;
  if (++it.ks >= it.nks) kiter_load(it, a, it.tile + gridDim.x, ntiles, mode);
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

template <int MODE>
__global__ void __launch_bounds__(THREADS, 1) qgemm_tc_kernel(const GemmArgs a) {
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
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = bars->tmem_base;

  if (warp < 8) {
    // ------------------------------------------------------------ dequant producers
    const int t = tid >> 1;    // A row
    const int half = tid & 1;  // words [4 half, 4 half + 4) of the row's 8 per k-step
    KIter cur, pf;
    kiter_load(cur, a, blockIdx.x, ntiles, MODE);
    pf = cur;
    int pf_count = 0;
    auto issue = [&](const KIter& k, int slot) {
      const TileInfo& ti = k.ti;
      const bool sh = ti.expert < 0;
      const int K = (MODE == MODE_DOWN && sh) ? a.K_shared : a.K;
      const int N = sh ? a.N_shared : a.N;
      int row;
      const uint32_t* W;
      const uint16_t* S;
      const uint16_t* B;
      if (MODE == MODE_GATEUP) {
        const bool up = t >= 64;
        row = ti.rb * 64 + (t & 63);
        W = up ? (sh ? a.sw1 : a.w1) : (sh ? a.sw0 : a.w0);
        S = up ? (sh ? a.ss1 : a.s1) : (sh ? a.ss0 : a.s0);
        B = up ? (sh ? a.sb1 : a.b1) : (sh ? a.sb0 : a.b0);
      } else {
        row = ti.rb * 128 + t;
        W = sh ? a.sw0 : a.w0;
        S = sh ? a.ss0 : a.s0;
        B = sh ? a.sb0 : a.b0;
      }
      if (row < N) {
        const int64_t r = (sh ? 0 : static_cast<int64_t>(ti.expert) * N) + row;
        const int gpr = K / a.gs;
        uint8_t* ring = smem + OFF_RING + slot * RING_BYTES;
        cp_async16(smem_u32(ring + t * 32 + half * 16), W + r * (K / 8) + k.ks * 8 + half * 4);
        // half 0 fetches the scale pair, half 1 the bias pair
        const uint16_t* SB = half ? B : S;
        uint8_t* dst = ring + RING_CODES + t * 8 + half * 4;
        const int g0 = (k.ks * 64) / a.gs;
        if (!SB) {
          *reinterpret_cast<uint32_t*>(dst) = 0u;
        } else if ((gpr & 1) == 0) {
          // 4-byte aligned group pair holding this k-step's group(s)
          asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_u32(dst)), "l"(SB + r * gpr + (g0 & ~1))
                       : "memory");
        } else {
          // odd group count per row (group size >= 64, one group per k-step): scalar
          // load, the value duplicated into both halves of the slot
          *reinterpret_cast<uint32_t*>(dst) = static_cast<uint32_t>(__ldg(SB + r * gpr + g0)) * 0x10001u;
        }
      }
    };
    // prologue: NRING-1 k-steps in flight
    for (int d = 0; d < NRING - 1; ++d) {
      if (pf.valid) {
        issue(pf, pf_count % NRING);
        kiter_next(pf, a, ntiles, MODE);
      }
      ++pf_count;
      cp_async_commit();
    }
    int it = 0;
    while (cur.valid) {
      if (pf.valid) {
        issue(pf, pf_count % NRING);
        kiter_next(pf, a, ntiles, MODE);
      }
      ++pf_count;
      cp_async_commit();
      cp_async_wait<NRING - 1>();
      // the pair of threads of a row read each other's scale / bias word
      __syncwarp();
      const int slot = it % NRING, stage = it % STAGES;
      if (!mbar_wait(&bars->empty[stage], ((it / STAGES) & 1) ^ 1, abort_flag, a.err)) break;
      const TileInfo& ti = cur.ti;
      const bool sh = ti.expert < 0;
      const int N = sh ? a.N_shared : a.N;
      const int row = (MODE == MODE_GATEUP) ? ti.rb * 64 + (t & 63) : ti.rb * 128 + t;
      if (row < N) {
        const uint8_t* ring = smem + OFF_RING + slot * RING_BYTES;
        const uint4 w = *reinterpret_cast<const uint4*>(ring + t * 32 + half * 16);
        const uint32_t sp = *reinterpret_cast<const uint32_t*>(ring + RING_CODES + t * 8);
        const uint32_t bp = *reinterpret_cast<const uint32_t*>(ring + RING_CODES + t * 8 + 4);
        const uint32_t words[4] = {w.x, w.y, w.z, w.w};
        uint8_t* As = smem + OFF_A + stage * A_BYTES;
        const int g0 = (cur.ks * 64) / a.gs;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int cc = half * 4 + i;
          const int gi = (cur.ks * 64 + 8 * cc) / a.gs;
          const int hi = (gi - (g0 & ~1)) & 1;
          const uint16_t sv = static_cast<uint16_t>(hi ? (sp >> 16) : (sp & 0xffffu));
          const uint16_t bv = static_cast<uint16_t>(hi ? (bp >> 16) : (bp & 0xffffu));
          const uint32_t s2u = static_cast<uint32_t>(sv) * 0x10001u, b2u = static_cast<uint32_t>(bv) * 0x10001u;
          const __nv_bfloat162 s2 = *reinterpret_cast<const __nv_bfloat162*>(&s2u);
          const __nv_bfloat162 b2 = *reinterpret_cast<const __nv_bfloat162*>(&b2u);
          uint4 o;
          o.x = deq_pair(words[i], 0, s2, b2);
          o.y = deq_pair(words[i], 1, s2, b2);
          o.z = deq_pair(words[i], 2, s2, b2);
          o.w = deq_pair(words[i], 3, s2, b2);
          *reinterpret_cast<uint4*>(As + sw128_off(t, cc)) = o;
        }
      }
      fence_proxy_async();
      mbar_arrive(&bars->full[stage]);
      ++it;
      kiter_next(cur, a, ntiles, MODE);
    }
    cp_async_wait<0>();
  } else if (warp < EPI_WARP) {
    // ------------------------------------------------------------ activation producers
    const int bt = tid - NA;
    const int cc = bt & 7, rg = bt >> 3;  // 16-byte chunk of the row, first row (0..15)
    // swizzled destination of row rg + 16 i: (rg + 16 i) * 128 + ((cc ^ (rg & 7)) << 4)
    const uint32_t dst0 = static_cast<uint32_t>(rg) * 128u + ((static_cast<uint32_t>(cc ^ (rg & 7))) << 4);
    int it = 0;
    bool ok = true;
    for (int tile = blockIdx.x; tile < ntiles && ok; tile += gridDim.x) {
      const TileInfo ti = decode_tile(a.tab, tile);
      const bool sh = ti.expert < 0;
      const int nks = tile_ksteps(a, ti, MODE);
      const uint16_t* base = sh ? a.act_shared : a.act;
      const uint64_t ld_bytes = static_cast<uint64_t>(sh ? a.act_shared_ld : a.act_ld) * 2u;
      // source rows of this thread's rows (rg + 16 i), kept in registers
      uint32_t srow[B_ROWS];
#pragma unroll
      for (int i = 0; i < B_ROWS; ++i) {
        const int r = rg + 16 * i;
        uint32_t s = 0;
        if (r < ti.nrows) {
          const int p = ti.row0 + r;
          s = static_cast<uint32_t>((MODE == MODE_DOWN || sh) ? p : a.sorted_token[p]);
        }
        srow[i] = s;
      }
      const int nvalid = ti.nrows;
      for (int ks = 0; ks < nks; ++ks) {
        const int stage = it % STAGES;
        if (!mbar_wait(&bars->empty[stage], ((it / STAGES) & 1) ^ 1, abort_flag, a.err)) {
          ok = false;
          break;
        }
        const uint32_t bs = smem_u32(smem + OFF_B + stage * B_BYTES) + dst0;
        const uint64_t src_k = reinterpret_cast<uint64_t>(base) + static_cast<uint64_t>(ks * 128 + cc * 16);
#pragma unroll
        for (int i = 0; i < B_ROWS; ++i) {
          if (rg + 16 * i < nvalid)
            cp_async16(bs + static_cast<uint32_t>(i) * 2048u,
                       reinterpret_cast<const void*>(src_k + static_cast<uint64_t>(srow[i]) * ld_bytes));
        }
        cp_async_commit();
        if (it >= B_LAG) {
          cp_async_wait<B_LAG>();
          fence_proxy_async();
          mbar_arrive(&bars->full[(it - B_LAG) % STAGES]);
        }
        ++it;
      }
    }
    cp_async_wait<0>();
    fence_proxy_async();
    for (int j = (it >= B_LAG ? it - B_LAG : 0); j < it; ++j) mbar_arrive(&bars->full[j % STAGES]);
  } else if (warp == MMA_WARP) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      int it = 0, lt = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < ntiles && ok; tile += gridDim.x, ++lt) {
        const TileInfo ti = decode_tile(a.tab, tile);
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
      const TileInfo ti = decode_tile(a.tab, tile);
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
#pragma unroll
          for (int c = 0; c < 16; ++c) {
            const int col = j * 32 + c0 + c;
            float gv, uv;
            if (q < 2) {
              gv = rbf(v[c]);
              uv = bf2f(to_gate[c * 64 + r64]);
            } else {
              gv = bf2f(to_up[c * 64 + r64]);
              uv = rbf(v[16 + c]);
            }
            const uint32_t mine = f2bf(swiglu1(gv, uv));
            const uint32_t other = __shfl_xor_sync(0xffffffffu, mine, 4);
            if (col < ti.nrows && (lane & 4) == 0 && n < N)
              *reinterpret_cast<uint32_t*>(outb + static_cast<int64_t>(ti.row0 + col) * ld + pn) = mine | (other << 16);
          }
        } else {
          // lanes (2m, 2m+1) hold rows (n, n+1); the even lane finishes column c and
          // the odd lane column c+1, each as one 2-wide red / 4-byte store
          const int n = ti.rb * 128 + row_in;
          const bool odd = lane & 1;
          const int n0 = n & ~1;
#pragma unroll
          for (int c = 0; c < 32; c += 2) {
            const int col = j * 32 + c + (odd ? 1 : 0);
            const bool colok = col < ti.nrows;
            const int p = ti.row0 + (colok ? col : 0);
            float mine_c = v[c], mine_c1 = v[c + 1];
            if (MODE == MODE_DOWN && !sh) {  // bf16(bf16(d) * score) per MLX op
              const int pe = ti.row0 + min(j * 32 + c, ti.nrows - 1);
              const int po = ti.row0 + min(j * 32 + c + 1, ti.nrows - 1);
              const float se = a.sorted_score[pe], so = a.sorted_score[po];
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
              if (sh) {
                red_add_v2(a.ysh + static_cast<int64_t>(p) * a.y_ld + n0, lo, hi);
              } else {
                const int tok = a.sorted_token[p];
                red_add_v2(a.y_acc + static_cast<int64_t>(tok) * a.y_ld + n0, lo, hi);
              }
            } else {
              *reinterpret_cast<uint32_t*>(a.out + static_cast<int64_t>(a.sorted_flat[p]) * a.out_ld + n0) =
                  pack_bf16x2(lo, hi);
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

cudaError_t launch(int mode, int grid, cudaStream_t stream, const GemmArgs& a) {
  switch (mode) {
    case MODE_GATEUP: qgemm_tc_kernel<MODE_GATEUP><<<grid, THREADS, SMEM_BYTES, stream>>>(a); break;
    case MODE_DOWN: qgemm_tc_kernel<MODE_DOWN><<<grid, THREADS, SMEM_BYTES, stream>>>(a); break;
    default: qgemm_tc_kernel<MODE_PLAIN><<<grid, THREADS, SMEM_BYTES, stream>>>(a); break;
  }
  return cudaGetLastError();
}

}  // namespace tc
}  // namespace fm
