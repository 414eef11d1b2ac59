// ep.cu -- expert-parallel exchange over NVLink peer memory, without host
// synchronization (no counterpart in the reference, which is single-process).
//
// Every rank owns one region of device memory with the same layout, mapped into every
// other rank's address space (CUDA IPC):
//   flags  [3][W] u32   per (kind, source rank) the epoch of the last post:
//                       kind 0 counts posted, 1 rows posted, 2 results returned
//   counts [W][E] i32   pairs of source rank s routed to global expert e (all-gathered)
//   recv   [cap_recv][H] bf16   rows received by this rank as an owner: source-major,
//                               expert-major within a source
//   ret    [cap_ret][H]  bf16   bf16(d) rows returned to this rank as a token owner, in
//                               the rank's own expert-major send order
// One layer call (epoch e) on rank r:
//   ep_dispatch_kernel   post r's per-expert counts to every rank's board (flag 0), wait
//                        for every rank's counts, then write r's routed rows straight into
//                        their owners' recv buffers at offsets computed from the board, and
//                        release flag 1 on every owner
//   ep_p2p_plan_kernel   (owner) wait for flag 1 of every source; tile tables over the
//                        (source, local expert) segments and, per received row, its source
//                        rank and position in that source's send order
//   the expert GEMMs     gate/up on the received rows; the down GEMM's epilogue stores
//                        every bf16(d) row straight into its source rank's ret buffer
//   ep_release_kernel    release flag 2 on every rank
//   ep_combine_p2p_kernel  wait for flag 2 of every owner, then combine as fm_ep_combine
// Ranks run calls in lockstep: a rank can only start call e+1 after its combine of call e
// saw every owner's returns, which every owner issues after its GEMMs of call e finished
// reading its recv buffer and board, so no buffer of call e is overwritten while in use.
// Every wait is bounded (kWaitBudgetCycles); on expiry the kernel records DEVERR_TIMEOUT
// and later kernels of the call skip their work.
#include "fm_ep.cuh"

namespace fm {

// Cooperative launch (the blocks wait on block 0's own post of this rank's counts).
__global__ void __launch_bounds__(256) ep_dispatch_kernel(const EpP2PArgs a) {
  __shared__ int64_t s_start[kEpMaxWorld], s_off[kEpMaxWorld];
  if (ep_block_error(a)) return;
  const int W = a.world, E = a.E, me = a.rank;
  if (blockIdx.x == 0) {
    for (int r = 0; r < W; ++r) {
      int32_t* dst = ep_board(a, r) + static_cast<int64_t>(me) * E;
      for (int e = threadIdx.x; e < E; e += blockDim.x) dst[e] = a.offsets[e + 1] - a.offsets[e];
    }
    __threadfence_system();
    __syncthreads();
    if (threadIdx.x < W) st_release_sys(ep_flag(a, threadIdx.x, 0, me), a.epoch);
  }
  if (!ep_wait_all(a, 0)) return;
  // where this rank's rows go: owner r's rows start at s_start[r] of the send order
  // (expert-major), there are s_rows[r] of them, and they land at s_off[r] of r's recv
  const int32_t* cnt = ep_board(a, me);
  if (threadIdx.x < W) {
    const int r = threadIdx.x;
    int first, count;
    ep_owner_range(E, r, W, first, count);
    int64_t start = 0, rows = 0, off = 0;
    for (int e = 0; e < first; ++e) start += cnt[static_cast<int64_t>(me) * E + e];
    for (int e = first; e < first + count; ++e) rows += cnt[static_cast<int64_t>(me) * E + e];
    for (int s = 0; s < me; ++s)
      for (int e = first; e < first + count; ++e) off += cnt[static_cast<int64_t>(s) * E + e];
    if (off + rows > a.cap_recv) report(a.err, DEVERR_BOUNDS);
    s_start[r] = start;
    s_off[r] = off;
  }
  if (ep_block_error(a)) return;
  const int segs = a.H / 8;
  const int64_t routed = a.offsets[E];  // pairs with an expert (at most P)
  const int64_t Pv = routed < a.P ? routed : a.P;
  const int64_t n = Pv * segs;
  // The rows are owner-contiguous and the grid walks them in order, so every rank starts
  // at its own rows and goes on to the next owners': at any moment the ranks write to
  // different owners rather than all of them into one owner's memory.
  const int64_t rot = s_start[me] < Pv ? s_start[me] : 0;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t p0 = i / segs;
    const int col = static_cast<int>(i - p0 * segs) * 8;
    const int64_t p = (p0 + rot < Pv) ? p0 + rot : p0 + rot - Pv;
    int r = 0;
    while (r + 1 < W && p >= s_start[r + 1]) ++r;
    const int64_t row = s_off[r] + (p - s_start[r]);
    *reinterpret_cast<uint4*>(ep_rows(a, r, a.off_recv) + row * a.H + col) =
        *reinterpret_cast<const uint4*>(a.x_perm + static_cast<int64_t>(a.sorted_token[p]) * a.H + col);
  }
  ep_release_when_grid_done(a, 1);
}

// Owner side, after the down GEMM wrote every d row into its source's ret buffer:
// release flag 2 on every rank (one block; the GEMM's stores precede it in stream order).
__global__ void ep_release_kernel(const EpP2PArgs a, int kind) {
  if (ep_block_error(a)) return;
  __threadfence_system();
  if (threadIdx.x < a.world) st_release_sys(ep_flag(a, threadIdx.x, kind, a.rank), a.epoch);
}

}  // namespace fm
