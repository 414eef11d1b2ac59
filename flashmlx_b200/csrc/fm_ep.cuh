// fm_ep.cuh -- device helpers of the expert-parallel exchange over peer memory
// (kernels in ep.cu, route.cu, qgemv.cu; layout described in ep.cu).
#pragma once

#include "fm_internal.cuh"

namespace fm {

FM_DEV void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
FM_DEV uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

FM_DEV uint32_t* ep_flag(const EpP2PArgs& a, int rank, int kind, int src) {
  return reinterpret_cast<uint32_t*>(a.peer[rank] + a.off_flags) + kind * a.world + src;
}
FM_DEV int32_t* ep_board(const EpP2PArgs& a, int rank) {
  return reinterpret_cast<int32_t*>(a.peer[rank] + a.off_counts);
}
FM_DEV uint16_t* ep_rows(const EpP2PArgs& a, int rank, int64_t off) {
  return reinterpret_cast<uint16_t*>(a.peer[rank] + off);
}

// Block-uniform read of the device error word (a barrier).
FM_DEV bool ep_block_error(const EpP2PArgs& a) {
  return __syncthreads_or(*reinterpret_cast<volatile uint32_t*>(a.err) != 0u) != 0;
}

// Threads 0..W-1 wait until this rank's flag [kind][thread] holds the call's epoch.
// Block-uniform result; false after a timeout or an earlier error (recorded).
FM_DEV bool ep_wait_all(const EpP2PArgs& a, int kind) {
  bool ok = true;
  if (threadIdx.x < a.world) {
    const uint32_t* f = ep_flag(a, a.rank, kind, threadIdx.x);
    const long long t0 = clock64();
    while (ld_acquire_sys(f) != a.epoch) {
      if (*reinterpret_cast<volatile uint32_t*>(a.err) != 0u) {
        ok = false;
        break;
      }
      if (clock64() - t0 > kWaitBudgetCycles) {
        report(a.err, DEVERR_TIMEOUT);
        ok = false;
        break;
      }
    }
  }
  return __syncthreads_and(ok) != 0;
}

// The last block of the grid to get here (after its own peer stores) releases flag
// [kind][this rank] on every rank.
FM_DEV void ep_release_when_grid_done(const EpP2PArgs& a, int kind) {
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) {
    const int prev = atomicAdd(a.done_counter, 1);
    if (prev == static_cast<int>(gridDim.x) - 1) {
      *a.done_counter = 0;  // ready for the next launch
      __threadfence_system();
      for (int r = 0; r < a.world; ++r) st_release_sys(ep_flag(a, r, kind, a.rank), a.epoch);
    }
  }
}

// contiguous experts of rank r (the rule of fm_ep_range)
FM_DEV void ep_owner_range(int E, int r, int W, int& first, int& count) {
  const int base = E / W, rem = E % W;
  count = base + (r < rem ? 1 : 0);
  first = r * base + min(r, rem);
}

}  // namespace fm
