// qgemm_tc.cu -- grouped 4-bit expert GEMM on the 5th-generation tensor cores, run by
// CTA pairs (2-CTA clusters) issuing tcgen05.mma.cta_group::2.
//
// Replaces mx::gather_qmm (sorted, model.cpp:703-721) and mx::quantized_matmul
// (model.cpp:741-747) for prefill-sized batches.  Each pair walks a device-built tile
// table (expert / shared-expert group, 256-row weight block, chunk of <= 224
// activation rows).  One tile is D[256 x N] = A[256 x K] * B[N x K]^T:
//   A (dequantized weights): rows 0..127 in CTA 0's tensor memory, 128..255 in CTA 1's;
//   B (activation rows):     rows 0..N/2-1 in CTA 0's shared memory, N/2..N-1 in CTA 1's;
//   D (fp32, TMEM):          CTA r holds its 128 A rows x all N columns.
// Per SM and 64-wide k-step that is 4 KB of codes and <= 14 KB of activations from
// L2 for <= 3.7 MFLOP, half the L2 bytes per FLOP of a one-CTA tile, which the
// L2 -> SM bandwidth (~11 TB/s on B200) could not feed.  A lives in TMEM (the MMA's
// A-from-tensor-memory form) because with A in shared memory the dequantized stores
// and the MMA's reads of them came on top of the activation and code traffic there.
// TMEM (512 columns): two accumulator buffers of 224 columns, two A stages of 32.
//   gate/up mode: CTA r's A rows 0..63 = gate rows f0 + 64r .. +63, rows 64..127 =
//                 the same up rows (f0 = 128 x block), so one CTA's accumulator holds
//                 g and u of a row; the epilogue applies silu(g)*u and stores the
//                 pair-permuted activation rows for down.
//   down mode:    A = 128 down rows per CTA; the epilogue stores bf16(bf16(d)*score)
//                 per routed pair (expert-major rows; the combine kernel sums the k
//                 pairs of a token in a fixed order) or bf16(d) per shared row.
//   plain mode:   quantized_matmul / gather_qmm output rows, bf16.
//   relu2 mode:   A = 128 rows of one ungated matrix (fc1) per CTA; the epilogue stores
//                 bf16(relu(bf16(acc))^2) as pair-permuted activation rows for down (the
//                 sigmoid-routed variant, nemotron_h.cpp:53-58).
//
// Data movement: packed 4-bit codes arrive by TMA, 4 k-steps (128 B x 128 rows) per
// load, 128B-swizzled, into a 3-deep ring per CTA.  Contiguous activation rows arrive
// by TMA in 32-row boxes (128-row boxes for halves over 64 rows) straight into the
// UMMA B stage of an 8-deep ring, completing on the leader
// CTA's stage barrier; token-gathered rows are copied with cp.async.  Outputs go
// through a shared-memory staging tile and leave as coalesced 16-byte stores.
//
// Roles (512 threads per CTA):
//   warps 0-7   dequant producers in two groups of four that take alternate k-steps;
//               the thread in TMEM lane L owns A row L.  Per k-step: two 16-byte code
//               reads, bf16 fma of the exact codes with the group's scale and bias
//               (staged in shared memory by the code loader), one 32-column tcgen05.st
//               into its lane of the A stage; one arrival per warp on the leader's
//               stage barrier.
//   warp 8      code loader (an elected lane issues the TMA of each super-step; all
//               lanes copy the scales).
//   warps 9-10  activation loaders (this CTA's half of the tile's rows).
//   warp 11     TMEM allocation (both CTAs) and, in the leader CTA only, the
//               tcgen05.mma issuer (M=256, N<=224, K=16 x 4 per stage): the whole warp
//               walks the k-steps with warp-uniform operands, one elected lane issues;
//               commits free the stage / publish the accumulator in both CTAs.
// Single-thread tcgen05 / TMA instructions are issued from a converged warp through
// elect.sync with operands the warp computed uniformly (warp index and values read
// from memory broadcast from lane 0): a thread computing them on its own paid ~90
// cycles of issue per MMA, more than an N = 128 MMA takes to execute.
//   warps 12-15 epilogue: tcgen05.ld of the four 32-lane TMEM quadrants; double-
//               buffered accumulators (2 x 224 columns) overlap the next mainloop.
// Cross-CTA signalling: mbarrier arrivals on the peer's barriers through mapa
// addresses, tcgen05.commit to each CTA's barrier, and the 2-CTA form of the TMA
// load whose completion lands on the leader's barrier.  No load is multicast; every
// TMA source is this GPU's own memory.  Every wait is bounded.
#include "fm_internal.cuh"

namespace fm {
namespace tc {

constexpr int BM = 128;          // A rows per CTA (M = 256 per pair)
constexpr int ACC_COLS = 224;    // TMEM columns per accumulator buffer (two buffers)
constexpr int BN = ACC_COLS;     // max activation rows per pair tile (MMA N)
constexpr int BNH = BN / 2;      // B rows per CTA
constexpr int STAGES = 2;        // A stages (TMEM)
constexpr int RING = 8;          // k-step ring: B stages (shared memory) and the full / empty barriers
constexpr int A_COLS = 32;                        // TMEM columns of one A stage: 64 bf16 per lane
constexpr uint32_t A_TMEM0 = 2u * ACC_COLS;       // first column of the A stages
static_assert(A_TMEM0 + STAGES * A_COLS <= 512, "accumulators and A stages fit the 512 TMEM columns");
constexpr int NC = 3;            // code ring depth (super-steps of 4 k-steps)
constexpr int KS_PER_SS = 4;
constexpr int B_BYTES = ((BNH + 31) / 32 * 32 > kActBigBoxRows ? (BNH + 31) / 32 * 32 : kActBigBoxRows) * 128;  // whole TMA boxes
constexpr int C_BYTES = BM * 128;  // 128 rows x 32 words
constexpr int SC_GROUPS = 8;                     // max quant groups per row per super-step (gs 32)
constexpr int SC_BYTES = 2 * BM * SC_GROUPS * 2; // scales + biases of one code slot
constexpr int STG_BYTES = 32 * 256;              // 32 rows x 128 bf16 outputs
constexpr int OFF_B = 0;
constexpr int OFF_C = OFF_B + RING * B_BYTES;
constexpr int OFF_SC = OFF_C + NC * C_BYTES;
constexpr int OFF_STG = OFF_SC + NC * SC_BYTES;  // two staging tiles
constexpr int OFF_TB = OFF_STG + 2 * STG_BYTES;  // tile_begin of every group
constexpr int OFF_BAR = OFF_TB + ((kMaxGroups * 4 + 255) / 256) * 256;
constexpr int BAR_BYTES = 512;
constexpr int SMEM_BYTES = OFF_BAR + BAR_BYTES + 1024;  // + alignment slack
constexpr int DQ_GROUPS = 2;     // group g dequantizes the k-steps with (k-step % 2) == g
constexpr int NA = 128 * DQ_GROUPS;  // dequant-producer threads: groups of 128, one A row per thread
constexpr int CODE_WARP = NA / 32;
constexpr int ACT_WARP = CODE_WARP + 1;  // two activation-loader warps
constexpr int NB = 64;
constexpr int B_ROWS = BNH / 8;  // rows per activation-loader thread (14)
constexpr int B_LAG = 4;
constexpr int MMA_WARP = ACT_WARP + 2;
constexpr int EPI_WARP = MMA_WARP + 1;  // first of the four epilogue warps (TMEM lane quadrant = warp % 4)
static_assert(EPI_WARP % 4 == 0, "epilogue warp q reads TMEM lane quadrant q");
constexpr int THREADS = (EPI_WARP + 4) * 32;
constexpr uint32_t TMEM_COLS = 512;
constexpr int FULL_ARRIVALS = 2 * (NA / 32 / DQ_GROUPS + NB / 32);  // per k-step: one dequant group and the activation loaders, both CTAs
constexpr int CFULL_ARRIVALS = 1 + 32;  // code-loader lane 0 (meta + expect_tx) + one per lane's scale copies
constexpr int ACCE_ARRIVALS = 2 * 4;                     // epilogue warps of both CTAs

static_assert(OFF_B % 1024 == 0 && OFF_C % 1024 == 0 && B_BYTES % 1024 == 0, "1 KB aligned stages");
static_assert(B_BYTES >= kActBigBoxRows * 128, "a big activation box fits one B stage");
static_assert(SMEM_BYTES <= 232448, "shared memory budget");

struct Bars {
  uint64_t full[RING];   // leader: k-step j % RING's A and B stages of both CTAs ready
  uint64_t empty[RING];  // each CTA: k-step j % RING's MMAs are done (A stage j % STAGES, B stage j % RING)
  uint64_t cfull[NC];
  uint64_t cempty[NC];
  uint64_t accf[2];        // each CTA: accumulator buffer complete
  uint64_t acce[2];        // leader: accumulator buffer drained by both epilogues
  uint64_t done;
  uint32_t tmem_base;
  int abort;
  int epi_ok[2][4];
  int slot_nk[NC];    // k-steps in the code slot's super-step; 0 marks the end of work
};
static_assert(sizeof(Bars) <= BAR_BYTES, "barrier block");

// ---------------------------------------------------------------- cluster helpers
FM_DEV uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
FM_DEV uint32_t cluster_id_x() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%clusterid.x;" : "=r"(r));
  return r;
}
FM_DEV uint32_t num_clusters_x() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%nclusterid.x;" : "=r"(r));
  return r;
}
// shared::cluster address of the same shared-memory location in CTA `rank`
FM_DEV uint32_t map_to_rank(const void* p, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_u32(p)), "r"(rank));
  return r;
}
FM_DEV void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
  asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// Arrival on a barrier of either CTA of the pair, with the default (.release, .cta)
// semantics: the data it publishes is read by the tensor core through the async
// proxy (after fence.proxy.async) or by TMA completion, not by the peer's threads,
// and a .cluster-scope release costs ~900 cycles per arrival on B200.
FM_DEV void mbar_arrive_cluster(uint32_t caddr) {
  asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(caddr) : "memory");
}
FM_DEV void mbar_arrive_expect_tx_cluster(uint32_t caddr, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cluster.b64 _, [%0], %1;" ::"r"(caddr), "r"(bytes) : "memory");
}
// 2D TMA into this CTA's shared memory whose completion is counted on the pair
// leader's barrier (caddr: shared::cluster address of that barrier)
FM_DEV void tma_load_2d_pair(uint32_t dst, const void* map, int x, int y, uint32_t caddr) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], "
      "[%4];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(caddr)
      : "memory");
}

// 4-byte cp.async that reads src_bytes (4 or 0) and zero-fills the rest
FM_DEV void cp_async4(uint32_t dst, const void* src, uint32_t src_bytes) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(dst), "l"(src), "r"(src_bytes) : "memory");
}
// one arrival on *bar once every cp.async this thread issued so far has landed
FM_DEV void cp_async_arrive_noinc(uint64_t* bar) {
  asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_u32(bar)) : "memory");
}
FM_DEV void mbar_arrive_cnt(uint64_t* bar, uint32_t n) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(n) : "memory");
}

// ---------------------------------------------------------------- 2-CTA tcgen05
FM_DEV void tmem_alloc2(uint32_t* dst_smem, uint32_t ncols) {  // one warp in each CTA
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}
FM_DEV void tmem_relinquish2() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
FM_DEV void tmem_dealloc2(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
// D[tmem, both CTAs] (+)= A[tmem, lanes 0..127 of each CTA: 256 rows over the pair, 16 K
// per 8 columns] * B[smem, N rows over the pair]^T
FM_DEV void umma2_bf16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc, uint32_t idesc, uint32_t accum) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accum)
      : "memory");
}
// arrive once on the barrier at caddr (either CTA of the pair) when all previously
// issued tcgen05.mma of this thread complete
FM_DEV void umma2_commit(uint32_t caddr) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(caddr)
               : "memory");
}

// tile `tile` of group G (index lo) of a tcgen05 tile table, whose groups have no K split
FM_DEV TileInfo tile_tc(const TileGroup& G, int lo, int tile) {
  const int local = tile - G.tile_begin;
  const int rb = local / G.chunks;
  const int ch = local - rb * G.chunks;
  TileInfo t;
  t.group = lo;
  t.expert = G.expert;
  t.ksplit = 1;
  t.ks = 0;
  t.rb = rb;
  t.row0 = G.row_begin + ch * G.chunk_rows;
  t.nrows = min(G.chunk_rows, G.rows - ch * G.chunk_rows);
  return t;
}

FM_DEV int tile_ksteps(const GemmArgs& a, const TileInfo& ti, int mode) {
  const int K = (mode == MODE_DOWN && ti.expert < 0) ? a.K_shared : a.K;
  return K / 64;
}

// MMA N of a tile: rows rounded up to 16 (8 per CTA half)
FM_DEV int tile_nmma(int nrows) { return max(16, (nrows + 15) & ~15); }

// iterator over the (tile, super-step) pairs of this pair
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
  // group index of a tile (shared-memory search only)
  FM_DEV int find(int tile) const {
    int lo = 0, hi = ng - 1;
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (tb[mid] <= tile) lo = mid; else hi = mid - 1;
    }
    return lo;
  }
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

FM_DEV void siter_next(SIter& it, const GemmArgs& a, const TileDir& dir, int ntiles, int stride, int mode) {
  if (!it.valid) return;
  if (++it.ss >= it.nss) siter_load(it, a, dir, it.tile + stride, ntiles, mode);
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
  const float sg = rbf(__fdividef(1.0f, 1.0f + __expf(-g)));
  const float h = rbf(g * sg);
  return rbf(h * u);
}

// A row t (0..127 of this CTA's half) -> row inside its weight matrix, and the
// matrix's scale / bias arrays
template <int MODE>
FM_DEV void a_row_info(const GemmArgs& a, const TileInfo& ti, int rank, int t, int& row, const uint16_t*& S,
                       const uint16_t*& B) {
  const bool sh = ti.expert < 0;
  if (MODE == MODE_GATEUP) {
    const bool up = t >= 64;
    row = ti.rb * 128 + rank * 64 + (t & 63);
    S = up ? (sh ? a.ss1 : a.s1) : (sh ? a.ss0 : a.s0);
    B = up ? (sh ? a.sb1 : a.b1) : (sh ? a.sb0 : a.b0);
  } else {
    row = ti.rb * 256 + rank * 128 + t;
    S = sh ? a.ss0 : a.s0;
    B = sh ? a.sb0 : a.b0;
  }
}

// The 128 epilogue threads copy a staged 32-row tile (row stride 256 B, `cols` bf16
// columns per row) to global memory as 16-byte stores; staged row i goes to the output
// row starting at dst_row(i) (this GPU's memory or a peer's), or nowhere when null.
template <class RowFn>
FM_DEV void store_staged(const uint8_t* stg, int cols, int col0, int ncols_valid, RowFn dst_row, int et) {
  const int segs_per_row = cols / 8;
  const int nseg = 32 * segs_per_row;
  for (int s = et; s < nseg; s += 128) {
    const int i = s / segs_per_row, part = s - i * segs_per_row;
    uint16_t* row = dst_row(i);
    if (!row || part * 8 >= ncols_valid) continue;
    const uint4 v = *reinterpret_cast<const uint4*>(stg + i * 256 + part * 16);
    *reinterpret_cast<uint4*>(row + col0 + part * 8) = v;
  }
}

template <int MODE>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(THREADS, 1)
    qgemm_tc_kernel(const GemmArgs a, const __grid_constant__ TcMaps maps) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  Bars* bars = reinterpret_cast<Bars*>(smem + OFF_BAR);
  const int tid = threadIdx.x;
  // warp index broadcast from lane 0: provably warp-uniform, so each role's values
  // derived from it can live in uniform registers
  const int warp = __shfl_sync(0xffffffffu, tid >> 5, 0), lane = tid & 31;
  const int rank = static_cast<int>(cluster_rank());
  const bool leader = rank == 0;
  const int pair = static_cast<int>(cluster_id_x());
  const int npairs = static_cast<int>(num_clusters_x());
  // an earlier kernel of this call reported a device error: the tile table is not trusted
  const int ntiles = (*reinterpret_cast<volatile uint32_t*>(a.err) != 0u) ? 0 : a.tab->num_tiles;
  volatile int* abort_flag = &bars->abort;

  if (tid == 0) {
    for (int s = 0; s < RING; ++s) {
      mbar_init(&bars->full[s], FULL_ARRIVALS);
      mbar_init(&bars->empty[s], 1);
    }
    for (int c = 0; c < NC; ++c) {
      mbar_init(&bars->cfull[c], CFULL_ARRIVALS);
      mbar_init(&bars->cempty[c], NA / 32);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&bars->accf[b], 1);
      mbar_init(&bars->acce[b], ACCE_ARRIVALS);
    }
    mbar_init(&bars->done, 1);
    bars->abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == MMA_WARP) {
    tmem_alloc2(&bars->tmem_base, TMEM_COLS);
    tmem_relinquish2();
  }
  int* s_tb = reinterpret_cast<int*>(smem + OFF_TB);
  const int ngroups = ntiles > 0 ? min(a.tab->num_groups, kMaxGroups) : 0;
  for (int i = tid; i < ngroups; i += THREADS) s_tb[i] = a.tab->g[i].tile_begin;
  const TileDir dir{a.tab, s_tb, ngroups};
  tc_fence_before();
  __syncthreads();
  cluster_sync_all();  // the peer's barriers are initialised before any remote arrival
  tc_fence_after();
  const uint32_t tmem_base = bars->tmem_base;
  // the leader's stage / accumulator-drain barriers, as shared::cluster addresses
  const uint32_t full0 = map_to_rank(&bars->full[0], 0);
  const uint32_t acce0 = map_to_rank(&bars->acce[0], 0);

  if (warp < NA / 32) {
    // ------------------------------------------------------------ dequant producers
    const int grp = warp / 4;               // takes the k-steps with (k-step % DQ_GROUPS) == grp
    const int L = (warp % 4) * 32 + lane;   // A row = TMEM lane it writes (the warp's lane quadrant)
    // code / scale row of the slot that A row L holds: in gate/up mode code rows 0..63
    // are gate rows f and 64..127 the up rows f of the same outputs, and A interleaves
    // them in blocks of 8 (gate f -> 16 (f / 8) + f % 8, up f -> the same + 8), so an
    // epilogue warp holds both halves of its SwiGLUs in lanes L and L ^ 8
    const int t = (MODE == MODE_GATEUP) ? 64 * ((L >> 3) & 1) + 8 * (L >> 4) + (L & 7) : L;
    // this thread's lane of the A stages; column A_TMEM0 + 32 s + c of stage s holds
    // the bf16 pair (2c, 2c + 1) of the k-step's 64 (pair-permuted) weights
    const uint32_t a_taddr = tmem_base + (static_cast<uint32_t>((warp % 4) * 32) << 16) + A_TMEM0;
    const int gs_shift = __ffs(a.gs) - 1;  // group sizes are powers of two (32, 64, 128)
    int cs = 0, it0 = 0;                   // super-step, k-steps before it
    bool ok = true;
    while (ok) {
      const int slot = cs % NC;
      if (!__all_sync(0xffffffffu, mbar_wait(&bars->cfull[slot], (cs / NC) & 1, abort_flag, a.err))) {
        ok = false;
        break;
      }
      const int nk = bars->slot_nk[slot];
      if (nk == 0) break;  // end of this pair's tiles
      const uint8_t* code = smem + OFF_C + slot * C_BYTES + t * 128;
      const uint16_t* sc = reinterpret_cast<const uint16_t*>(smem + OFF_SC + slot * SC_BYTES) + t * SC_GROUPS;
      const uint16_t* bi = sc + BM * SC_GROUPS;
#pragma unroll
      for (int kk = grp; kk < KS_PER_SS; kk += DQ_GROUPS) {
        if (kk >= nk) break;
        const int it = it0 + kk;
        const int stage = it % STAGES;
        // the k-step's 64 weights into registers first (codes and scales are in the
        // code slot already), so the math overlaps the wait for the stage to drain.
        // Rows past the matrix end need no test: the code loader gives them zero scales
        // and biases, so they dequantize to zeros (and their outputs are never stored)
        uint4 o[8];
        {
#pragma unroll
          for (int h = 0; h < 2; ++h) {  // the two 32-element halves of the k-step
            const uint4 w = *reinterpret_cast<const uint4*>(code + (((2 * kk + h) ^ (t & 7)) << 4));
            const int g = (kk * 64 + 32 * h) >> gs_shift;
            const uint32_t s2u = static_cast<uint32_t>(sc[g]) * 0x10001u;
            const uint32_t b2u = static_cast<uint32_t>(bi[g]) * 0x10001u;
            const __nv_bfloat162 s2 = *reinterpret_cast<const __nv_bfloat162*>(&s2u);
            const __nv_bfloat162 b2 = *reinterpret_cast<const __nv_bfloat162*>(&b2u);
            const uint32_t words[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              o[h * 4 + i].x = deq_pair(words[i], 0, s2, b2);
              o[h * 4 + i].y = deq_pair(words[i], 1, s2, b2);
              o[h * 4 + i].z = deq_pair(words[i], 2, s2, b2);
              o[h * 4 + i].w = deq_pair(words[i], 3, s2, b2);
            }
          }
        }
        const int jr = it - STAGES;  // the k-step whose MMAs read this A stage last
        if (jr >= 0 && !__all_sync(0xffffffffu, mbar_wait(&bars->empty[jr % RING], (jr / RING) & 1, abort_flag, a.err))) {
          ok = false;
          break;
        }
        // the MMAs that read the stage before are complete (commit -> empty): order
        // the TMEM stores after them, make them complete, and publish
        tc_fence_after();
        tmem_st32(a_taddr + static_cast<uint32_t>(stage * A_COLS), o);
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive_cluster(full0 + (it % RING) * 8);
      }
      if (!ok) break;
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars->cempty[slot]);
      it0 += nk;
      ++cs;
    }
    const int it = it0;
    // drain: the last commits of every stage land before this CTA may exit
    if (warp == 0 && ok) {
      for (int j = max(0, it - RING); j < it; ++j)
        if (!__all_sync(0xffffffffu, mbar_wait(&bars->empty[j % RING], (j / RING) & 1, abort_flag, a.err)))
          break;
    }
  } else if (warp == CODE_WARP) {
    // ------------------------------------------------------------ code loader (TMA)
    // Per super-step: the TMA of the codes (one elected lane, operands warp-uniform), the
    // scales and biases (all lanes: 4 A rows each, row pointers set once per tile) and
    // the slot metadata; after the last tile a slot with nk = 0 ends the consumers.
    // Scales land as sc[t][g], bi[t][g] (u16, row stride SC_GROUPS, G = 256 / gs groups
    // of the super-step); rows outside the matrix and groups past the row end are zero.
    // Rows with an even group count use 4-byte cp.async tracked by the slot barrier,
    // odd ones 2-byte loads and stores.  Every lane counts one arrival on cfull.
    SIter cur;
    siter_load(cur, a, dir, pair, ntiles, MODE);
    const int gs_shift = __ffs(a.gs) - 1;  // group sizes are powers of two
    const int G = 256 >> gs_shift;         // quant groups per row per super-step
    const uint16_t* srow[4];
    const uint16_t* brow[4];
    bool rv[4];
    int gpr = 0, tile_ready = -1;
    int u_row = 0, u_map0 = 0;
    int cs = 0;
    while (true) {
      const int slot = cs % NC;
      if (!__all_sync(0xffffffffu, mbar_wait(&bars->cempty[slot], ((cs / NC) & 1) ^ 1, abort_flag, a.err))) break;
      if (!cur.valid) {
        if (elect_one()) {
          bars->slot_nk[slot] = 0;
          mbar_arrive_cnt(&bars->cfull[slot], CFULL_ARRIVALS);
        }
        __syncwarp();
        break;
      }
      if (cur.tile != tile_ready) {  // a new tile: this lane's scale rows and the tile's TMA rows
        tile_ready = cur.tile;
        const TileInfo& ti = cur.ti;
        const bool sh = ti.expert < 0;
        const int K = (MODE == MODE_DOWN && sh) ? a.K_shared : a.K;
        const int N = sh ? a.N_shared : a.N;
        gpr = K >> gs_shift;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          int row;
          const uint16_t* S;
          const uint16_t* B;
          a_row_info<MODE>(a, ti, rank, lane + 32 * i, row, S, B);
          rv[i] = row < N;
          const int64_t r = (sh ? 0 : static_cast<int64_t>(ti.expert) * N) + (rv[i] ? row : 0);
          srow[i] = S + r * gpr;
          brow[i] = B ? B + r * gpr : nullptr;
        }
        const int base = (MODE == MODE_GATEUP) ? ti.rb * 128 + rank * 64 : ti.rb * 256 + rank * 128;
        u_row = __shfl_sync(0xffffffffu, (sh ? 0 : ti.expert * N) + base, 0);
        u_map0 = __shfl_sync(0xffffffffu, sh ? 2 : 0, 0);
      }
      const int ss = __shfl_sync(0xffffffffu, cur.ss, 0);
      const int nk = __shfl_sync(0xffffffffu, min(KS_PER_SS, cur.nks - cur.ss * KS_PER_SS), 0);
      uint16_t* sc = reinterpret_cast<uint16_t*>(smem + OFF_SC + slot * SC_BYTES);
      uint16_t* bi = sc + BM * SC_GROUPS;
      const int g0 = ss * G;
      if ((gpr & 1) == 0) {  // 4-byte copies: the pair of groups is inside the row or past it
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int t = lane + 32 * i;
          for (int g = 0; g < G; g += 2) {
            const bool in = rv[i] && g0 + g < gpr;
            cp_async4(smem_u32(sc + t * SC_GROUPS + g), in ? srow[i] + g0 + g : srow[i], in ? 4u : 0u);
            cp_async4(smem_u32(bi + t * SC_GROUPS + g), (in && brow[i]) ? brow[i] + g0 + g : srow[i],
                      (in && brow[i]) ? 4u : 0u);
          }
        }
        cp_async_arrive_noinc(&bars->cfull[slot]);
      } else {
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int t = lane + 32 * i;
          for (int g = 0; g < G; ++g) {
            const bool in = rv[i] && g0 + g < gpr;
            sc[t * SC_GROUPS + g] = in ? __ldg(srow[i] + g0 + g) : static_cast<uint16_t>(0);
            bi[t * SC_GROUPS + g] = (in && brow[i]) ? __ldg(brow[i] + g0 + g) : static_cast<uint16_t>(0);
          }
        }
        mbar_arrive(&bars->cfull[slot]);
      }
      const uint32_t dst = smem_u32(smem + OFF_C + slot * C_BYTES);
      const int x = ss * (KS_PER_SS * 8);
      if (elect_one()) {
        bars->slot_nk[slot] = nk;
        mbar_arrive_expect_tx(&bars->cfull[slot], C_BYTES);  // also publishes the metadata
        tma_load_2d(dst, &maps.code[u_map0], x, u_row, &bars->cfull[slot]);
        if (MODE == MODE_GATEUP) tma_load_2d(dst + 64 * 128, &maps.code[u_map0 + 1], x, u_row, &bars->cfull[slot]);
      }
      __syncwarp();
      ++cs;
      siter_next(cur, a, dir, ntiles, npairs, MODE);
    }
    cp_async_wait<0>();
    __syncwarp();
  } else if (warp == ACT_WARP || warp == ACT_WARP + 1) {
    // ------------------------------------------------------------ activation loaders
    const int bt = tid - ACT_WARP * 32;   // 0..63
    const int cc = bt & 7, rg = bt >> 3;  // 16-byte chunk, first row (rows rg + 8 i)
    // swizzled destination of row rg + 8 i: (rg + 8 i) * 128 + ((cc ^ rg) << 4)
    const uint32_t dst0 = static_cast<uint32_t>(rg) * 128u + (static_cast<uint32_t>(cc ^ rg) << 4);
    int it = 0, pend = 0;  // pend: oldest k-step whose cp.async rows are not yet published
    bool ok = true;
    for (int tile = pair; tile < ntiles && ok; tile += npairs) {
      const TileInfo ti = dir.get(tile);
      const bool sh = ti.expert < 0;
      const int nks = tile_ksteps(a, ti, MODE);
      const bool gather = (MODE != MODE_DOWN) && !sh;
      const int hrows = tile_nmma(ti.nrows) / 2;              // B rows per CTA
      const int rbeg = rank * hrows;                           // first tile row of this CTA
      const int rmine = max(0, min(hrows, ti.nrows - rbeg));  // rows of this CTA holding data
      uint32_t srow[B_ROWS];
      const uint16_t* base = sh ? a.act_shared : a.act;
      const uint64_t ld_bytes = static_cast<uint64_t>(sh ? a.act_shared_ld : a.act_ld) * 2u;
      if (gather) {
#pragma unroll
        for (int i = 0; i < B_ROWS; ++i) {
          const int r = rg + 8 * i;
          srow[i] = (r < rmine) ? static_cast<uint32_t>(a.sorted_token[ti.row0 + rbeg + r]) : 0u;
        }
      }
      // TMA boxes per k-step: up to two of 32 rows, or one of kActBigBoxRows rows (whose
      // rows past the tile are read but never used by the MMA)
      const bool big_box = hrows > 64;
      const int nblk = big_box ? 1 : (hrows + 31) >> 5;
      const uint32_t box_bytes = big_box ? kActBigBoxRows * 128u : 4096u;
      for (int ks = 0; ks < nks; ++ks) {
        const int stage = it % RING;
        if (!__all_sync(0xffffffffu, mbar_wait(&bars->empty[stage], ((it / RING) & 1) ^ 1, abort_flag, a.err))) {
          ok = false;
          break;
        }
        if (gather) {
          const uint32_t bs = smem_u32(smem + OFF_B + stage * B_BYTES) + dst0;
          const uint64_t src_k = reinterpret_cast<uint64_t>(base) + static_cast<uint64_t>(ks * 128 + cc * 16);
#pragma unroll
          for (int i = 0; i < B_ROWS; ++i) {
            if (rg + 8 * i < rmine)
              cp_async16(bs + static_cast<uint32_t>(i) * 1024u,
                         reinterpret_cast<const void*>(src_k + static_cast<uint64_t>(srow[i]) * ld_bytes));
          }
          cp_async_commit();
          if (it - pend >= B_LAG) {  // publish the k-step B_LAG behind
            cp_async_wait<B_LAG>();
            fence_proxy_async();
            __syncwarp();
            if (lane == 0) mbar_arrive_cluster(full0 + (pend % RING) * 8);
            ++pend;
          }
        } else {
          if (pend < it) {  // publish every gathered k-step still in flight
            cp_async_wait<0>();
            fence_proxy_async();
            __syncwarp();
            for (; pend < it; ++pend)
              if (lane == 0) mbar_arrive_cluster(full0 + (pend % RING) * 8);
          }
          if (warp == ACT_WARP) {  // the whole warp: operands warp-uniform, one lane issues
            const int row_base = __shfl_sync(0xffffffffu, ti.row0 + rbeg, 0);
            const int nb = __shfl_sync(0xffffffffu, nblk, 0);
            const uint32_t bb = __shfl_sync(0xffffffffu, box_bytes, 0);
            const CUtensorMap* map = &maps.act[__shfl_sync(0xffffffffu, (sh ? 1 : 0) + (big_box ? 2 : 0), 0)];
            const uint32_t bs = smem_u32(smem + OFF_B + stage * B_BYTES);
            if (elect_one()) {
              mbar_arrive_expect_tx_cluster(full0 + stage * 8, static_cast<uint32_t>(nb) * bb);
              for (int b = 0; b < nb; ++b)
                tma_load_2d_pair(bs + b * 4096, map, ks * 64, row_base + b * 32, full0 + stage * 8);
            }
            __syncwarp();
          } else if (lane == 0) {
            mbar_arrive_cluster(full0 + stage * 8);
          }
          pend = it + 1;
        }
        ++it;
      }
    }
    cp_async_wait<0>();
    fence_proxy_async();
    __syncwarp();
    for (; pend < it; ++pend)
      if (lane == 0) mbar_arrive_cluster(full0 + (pend % RING) * 8);
  } else if (warp == MMA_WARP) {
    // ------------------------------------------------------------ MMA issuer (leader)
    // The whole warp walks the loop with every MMA operand (TMEM address, descriptors,
    // instruction descriptor) warp-uniform -- broadcast from lane 0 where it comes from
    // memory -- and one elected lane issues.  A single thread computing them itself
    // costs ~90 cycles of issue per MMA, more than an N = 128 MMA takes to run.
    // elect.sync picks the same (lowest) lane every time, so the commits track that
    // lane's MMAs.
    if (leader) {
      const uint32_t empty_l = map_to_rank(&bars->empty[0], 0), empty_p = map_to_rank(&bars->empty[0], 1);
      const uint32_t accf_l = map_to_rank(&bars->accf[0], 0), accf_p = map_to_rank(&bars->accf[0], 1);
      const uint32_t tbase = __shfl_sync(0xffffffffu, tmem_base, 0);
      const uint32_t b_base = smem_u32(smem + OFF_B);
      const int ntl = __shfl_sync(0xffffffffu, ntiles, 0);
      int kc = 0, lt = 0;  // k-steps issued so far, tiles started
      bool ok = true;
      // The next tile's group is found (a forward scan from the current group) and its
      // global-memory record loaded after the current tile's first MMAs are issued; the
      // tile change then only does one division (a binary search, the record's load
      // latency and the general decode took ~1300 cycles there with the tensor pipe idle)
      int g_next = pair < ntl ? dir.find(pair) : 0;
      TileGroup G_next = a.tab->g[g_next];
      for (int tile = pair; tile < ntl && ok; tile += npairs, ++lt) {
        const TileInfo ti = tile_tc(G_next, g_next, tile);
        const int nks = __shfl_sync(0xffffffffu, tile_ksteps(a, ti, MODE), 0);
        const uint32_t idesc = __shfl_sync(0xffffffffu, idesc_bf16(2 * BM, tile_nmma(ti.nrows)), 0);
        const int buf = lt & 1;
        if (!mbar_wait_lane0(&bars->acce[buf], ((lt >> 1) & 1) ^ 1, abort_flag, a.err)) break;
        tc_fence_after();
        const uint32_t d = tbase + static_cast<uint32_t>(buf * ACC_COLS);
        for (int ks = 0; ks < nks; ++ks, ++kc) {
          const int slot = kc % RING;
          // one lane polls (the A and B stages of the k-step complete one barrier)
          if (!mbar_wait_lane0(&bars->full[slot], (kc / RING) & 1, abort_flag, a.err)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t at = tbase + A_TMEM0 + static_cast<uint32_t>((kc % STAGES) * A_COLS);  // lane 0 of both CTAs
          const uint64_t bd = sdesc_sw128(b_base + static_cast<uint32_t>(slot * B_BYTES));
          if (elect_one()) {
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) umma2_bf16_ts(d, at + 8 * kk, bd + 2 * kk, idesc, (ks | kk) != 0);
            umma2_commit(empty_l + slot * 8);
            umma2_commit(empty_p + slot * 8);
          }
          __syncwarp();
          if (ks == 0 && tile + npairs < ntl) {
            const int nt = tile + npairs;
            while (g_next + 1 < dir.ng && dir.tb[g_next + 1] <= nt) ++g_next;
            G_next = a.tab->g[g_next];
          }
        }
        if (ok && elect_one()) {
          umma2_commit(accf_l + buf * 8);
          umma2_commit(accf_p + buf * 8);
        }
        __syncwarp();
      }
      if (elect_one()) {
        umma2_commit(map_to_rank(&bars->done, 0));
        wait_done(&bars->done, 0, a.err);
      }
    }
    __syncwarp();
  } else if (warp >= EPI_WARP && warp < EPI_WARP + 4) {
    // ------------------------------------------------------------ epilogue
    const int q = warp - EPI_WARP;
    const int row_in = q * 32 + lane;    // TMEM lane == A row of this CTA
    const int et = tid - EPI_WARP * 32;  // 0..127
    int lt = 0, xit = 0;
    for (int tile = pair; tile < ntiles; tile += npairs, ++lt) {
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
        uint8_t* stg = smem + OFF_STG + (xit & 1) * STG_BYTES;
        const int c_lim = ti.nrows - j * 32;  // valid columns of this chunk (may exceed 32)
        const int prow = ti.row0 + j * 32;
        if (MODE == MODE_GATEUP) {
          // TMEM lane L of warp q holds gate row f and lane L ^ 8 up row f (the dequant
          // warps interleave them in blocks of 8): the gate lane finishes columns 0..15,
          // the up lane 16..31, trading the other half as bf16 pairs of adjacent columns
          const bool is_up = lane & 8;
          const int f = q * 16 + 8 * (lane >> 4) + (lane & 7);  // output row of this CTA's 64
          const int c0 = is_up ? 16 : 0;
          // silu(g) * u per MLX op, two columns at a time: sg = bf16(sigmoid(g)) from
          // fp32, then h = bf16(g * sg) and bf16(h * u) as bf16x2 products (each
          // rounded once, as the per-op rounding of swiglu1)
          uint32_t res2[8];
#pragma unroll
          for (int c = 0; c < 8; ++c) {
            const uint32_t lo2 = pack_bf16x2(v[2 * c], v[2 * c + 1]);         // my row, columns 2c, 2c+1
            const uint32_t hi2 = pack_bf16x2(v[16 + 2 * c], v[17 + 2 * c]);   // my row, columns 16+2c, 17+2c
            const uint32_t got = __shfl_xor_sync(0xffffffffu, is_up ? lo2 : hi2, 8);
            const uint32_t g2 = is_up ? got : lo2;
            const uint32_t u2 = is_up ? hi2 : got;
            const float ga = __uint_as_float(g2 << 16), gb = __uint_as_float(g2 & 0xffff0000u);
            const uint32_t s2 = pack_bf16x2(__fdividef(1.0f, 1.0f + __expf(-ga)), __fdividef(1.0f, 1.0f + __expf(-gb)));
            res2[c] = bmul2(bmul2(g2, s2), u2);
          }
          // staging row = token column (c0 + c), 64 outputs at their pair-permuted
          // slots; outputs f and f ^ 4 (lanes L and L ^ 4) share one 32-bit word
          const int pn = perm8(f);
#pragma unroll
          for (int c = 0; c < 8; ++c) {
            const uint32_t other = __shfl_xor_sync(0xffffffffu, res2[c], 4);
            if ((f & 4) == 0) {
              *reinterpret_cast<uint32_t*>(stg + (c0 + 2 * c) * 256 + pn * 2) = __byte_perm(res2[c], other, 0x5410);
              *reinterpret_cast<uint32_t*>(stg + (c0 + 2 * c + 1) * 256 + pn * 2) = __byte_perm(res2[c], other, 0x7632);
            }
          }
          named_bar_sync(1, 128);
          uint16_t* outb = sh ? a.out_shared : a.out;
          const int64_t ld = sh ? a.out_shared_ld : a.out_ld;
          const int col0 = ti.rb * 128 + rank * 64;
          store_staged(stg, 64, col0, N - col0,
                       [&](int i) -> uint16_t* { return i < c_lim ? outb + static_cast<int64_t>(prow + i) * ld : nullptr; },
                       et);
        } else if (MODE == MODE_RELU2) {
          // staging row = token column c, this CTA's 128 outputs at their pair-permuted
          // slots (n -> perm8(n)); outputs n and n + 4 (lanes L and L ^ 4) share one word
          const int pn = perm8(row_in);
#pragma unroll
          for (int c = 0; c < 32; ++c) {
            const float r = fmaxf(rbf(v[c]), 0.f);
            const uint32_t mine = f2bf(r * r);
            const uint32_t other = __shfl_xor_sync(0xffffffffu, mine, 4);
            if ((row_in & 4) == 0) *reinterpret_cast<uint32_t*>(stg + c * 256 + pn * 2) = mine | (other << 16);
          }
          named_bar_sync(1, 128);
          uint16_t* outb = sh ? a.out_shared : a.out;
          const int64_t ld = sh ? a.out_shared_ld : a.out_ld;
          const int col0 = ti.rb * 256 + rank * 128;
          store_staged(stg, 128, col0, N - col0,
                       [&](int i) -> uint16_t* { return i < c_lim ? outb + static_cast<int64_t>(prow + i) * ld : nullptr; },
                       et);
        } else {
          // staging row = token column c, 128 outputs; lanes (2m, 2m+1) hold rows
          // (n, n+1): the even lane stores even columns, the odd lane odd columns
          const bool odd = lane & 1;
          const int pc = ti.row0 + min(j * 32 + lane, ti.nrows - 1);
          // routing scores are bf16 values, so bf16(bf16(d) * score) per MLX op is one
          // bf16x2 product per column pair; lane c (even) holds the scores of columns c, c+1
          uint32_t s_pair = 0x3F803F80u;  // (1, 1)
          if (MODE == MODE_DOWN && !sh && !a.unit_score) {
            const float my_score = a.sorted_score[pc];
            s_pair = pack_bf16x2(my_score, __shfl_down_sync(0xffffffffu, my_score, 1));
          }
          const uint32_t psel = odd ? 0x7632u : 0x5410u;
#pragma unroll
          for (int c = 0; c < 32; c += 2) {
            uint32_t r2 = pack_bf16x2(v[c], v[c + 1]);  // this row, columns c and c+1
            if (MODE == MODE_DOWN && !sh && !a.unit_score) r2 = bmul2(r2, __shfl_sync(0xffffffffu, s_pair, c));
            // lanes (2m, 2m+1) hold rows (n0, n0+1): the even lane stores column c, the
            // odd lane column c+1, each word holding both rows
            const uint32_t other = __shfl_xor_sync(0xffffffffu, r2, 1);
            const uint32_t w = odd ? __byte_perm(other, r2, psel) : __byte_perm(r2, other, psel);
            const int col = c + (odd ? 1 : 0);
            *reinterpret_cast<uint32_t*>(stg + col * 256 + (row_in & ~1) * 2) = w;
          }
          named_bar_sync(1, 128);
          const int col0 = ti.rb * 256 + rank * 128;
          if (MODE == MODE_DOWN) {
            if (!sh && a.y_rowptr) {
              store_staged(stg, 128, col0, N - col0,
                           [&](int i) -> uint16_t* { return i < c_lim ? a.y_rowptr[prow + i] : nullptr; }, et);
            } else {
              uint16_t* outb = sh ? a.ysh16 : a.y_pairs;
              store_staged(
                  stg, 128, col0, N - col0,
                  [&](int i) -> uint16_t* { return i < c_lim ? outb + static_cast<int64_t>(prow + i) * a.y_ld : nullptr; },
                  et);
            }
          } else {
            store_staged(stg, 128, col0, N - col0,
                         [&](int i) -> uint16_t* {
                           return i < c_lim ? a.out + static_cast<int64_t>(a.sorted_flat[prow + i]) * a.out_ld : nullptr;
                         },
                         et);
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(acce0 + buf * 8);
    }
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync_all();  // no remote arrival or MMA read of this CTA's memory after this
  if (warp == MMA_WARP) {
    tc_fence_after();
    tmem_dealloc2(tmem_base, TMEM_COLS);
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

// CTA pairs that can be resident at once (the persistent grid is twice that)
cudaError_t max_pairs(int* n) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2, 1, 1);
  cfg.blockDim = dim3(THREADS, 1, 1);
  cfg.dynamicSmemBytes = SMEM_BYTES;
  cudaLaunchAttribute attr;
  attr.id = cudaLaunchAttributeClusterDimension;
  attr.val.clusterDim.x = 2;
  attr.val.clusterDim.y = 1;
  attr.val.clusterDim.z = 1;
  cfg.attrs = &attr;
  cfg.numAttrs = 1;
  return cudaOccupancyMaxActiveClusters(n, qgemm_tc_kernel<MODE_GATEUP>, &cfg);
}

cudaError_t launch(int mode, int pairs, cudaStream_t stream, const GemmArgs& a, const TcMaps& maps) {
  const int grid = 2 * pairs;
  switch (mode) {
    case MODE_GATEUP: qgemm_tc_kernel<MODE_GATEUP><<<grid, THREADS, SMEM_BYTES, stream>>>(a, maps); break;
    case MODE_DOWN: qgemm_tc_kernel<MODE_DOWN><<<grid, THREADS, SMEM_BYTES, stream>>>(a, maps); break;
    case MODE_RELU2: {
      // its shared-memory limit is set here, on first use, not with the others at fm_create
      const cudaError_t e =
          cudaFuncSetAttribute(qgemm_tc_kernel<MODE_RELU2>, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
      if (e != cudaSuccess) return e;
      qgemm_tc_kernel<MODE_RELU2><<<grid, THREADS, SMEM_BYTES, stream>>>(a, maps);
      break;
    }
    default: qgemm_tc_kernel<MODE_PLAIN><<<grid, THREADS, SMEM_BYTES, stream>>>(a, maps); break;
  }
  return cudaGetLastError();
}

}  // namespace tc
}  // namespace fm
