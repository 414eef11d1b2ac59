// fm_common.cuh -- device helpers shared by the libflashmoe kernels (sm_100a only).
//
// bf16 rounding helpers, bounded waits (every spin in this library gives up after a
// clock budget, records FM_DEVERR_TIMEOUT in the device error word and returns),
// mbarrier / cp.async / tcgen05 wrappers written as inline PTX.
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ < 1000)
#error "libflashmoe targets sm_100a only"
#endif

#define FM_DEV __device__ __forceinline__

namespace fm {

// bits of the device error word (workspace), read back by fm_sync_status
enum : uint32_t {
  DEVERR_TIMEOUT = 1u,   // a bounded wait ran out
  DEVERR_BOUNDS = 2u,    // an index failed its bounds check and the access was skipped
  DEVERR_CONFIG = 4u,    // a kernel found a shape it does not support
};

// ~1-2 s at B200 clocks; far above any legitimate wait inside one launch
constexpr long long kWaitBudgetCycles = 3ll << 30;

FM_DEV float bf2f(uint16_t b) { return __uint_as_float(static_cast<uint32_t>(b) << 16); }

FM_DEV uint16_t f2bf(float f) {
  __nv_bfloat16 h = __float2bfloat16_rn(f);
  return *reinterpret_cast<uint16_t*>(&h);
}

FM_DEV float rbf(float f) { return bf2f(f2bf(f)); }

FM_DEV uint32_t pack_bf16x2(float lo, float hi) {  // both rounded to nearest even, one instruction
  __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}
// bf16x2 product of two bf16 pairs, each rounded once (= rbf(a * b) per lane)
FM_DEV uint32_t bmul2(uint32_t a, uint32_t b) {
  __nv_bfloat162 r = __hmul2(*reinterpret_cast<const __nv_bfloat162*>(&a), *reinterpret_cast<const __nv_bfloat162*>(&b));
  return *reinterpret_cast<uint32_t*>(&r);
}

FM_DEV float sigmoid_f(float v) { return 1.0f / (1.0f + expf(-v)); }

// position of column n inside a row stored with the within-8 pair permutation
// (storage slot 2i <- element i, slot 2i+1 <- element i+4, i = 0..3)
FM_DEV int perm8(int n) {
  const int j = n & 7;
  return (n & ~7) | ((j < 4) ? (2 * j) : (2 * (j - 4) + 1));
}

FM_DEV uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

FM_DEV void report(uint32_t* err, uint32_t bits) {
  if (err) atomicOr(err, bits);
}

// ---------------------------------------------------------------- mbarrier
FM_DEV void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

FM_DEV void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

FM_DEV bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait on an mbarrier phase.  *abort (shared) lets one role's timeout stop
// every other role of the CTA quickly.  Returns false on timeout / abort.
FM_DEV bool mbar_wait(uint64_t* bar, uint32_t parity, volatile int* abort, uint32_t* err) {
  if (mbar_try_wait(bar, parity)) return true;
  const long long t0 = clock64();
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if (*abort) return false;
    if (clock64() - t0 > kWaitBudgetCycles) {
      *abort = 1;
      report(err, DEVERR_TIMEOUT);
      return false;
    }
  }
}

// The same wait polled by lane 0 alone, the result broadcast to the warp (which must be
// converged); lane 0 is the lane that then acts for the warp (elect.sync's choice).
FM_DEV bool mbar_wait_lane0(uint64_t* bar, uint32_t parity, volatile int* abort, uint32_t* err) {
  int ok = 1;
  if ((threadIdx.x & 31) == 0) ok = mbar_wait(bar, parity, abort, err) ? 1 : 0;
  return __shfl_sync(0xffffffffu, ok, 0) != 0;
}

FM_DEV void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}

// ---------------------------------------------------------------- TMA (no multicast)
// 2D tiled load of the map's box at element coordinates (x inner, y outer) into this
// CTA's shared memory, completing `bytes` of transaction count on *bar.
FM_DEV void tma_load_2d(uint32_t dst, const void* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

// four rows (y0..y3) of a one-row-high box, stacked in shared memory
FM_DEV void tma_gather4(uint32_t dst, const void* map, int x, int y0, int y1, int y2, int y3, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile::gather4.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, "
      "%4, %5, %6}], [%7];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y0), "r"(y1), "r"(y2), "r"(y3), "r"(smem_u32(bar))
      : "memory");
}

// ---------------------------------------------------------------- cp.async
FM_DEV void cp_async16(uint32_t dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
FM_DEV void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
FM_DEV void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}
// order this thread's generic-proxy shared-memory writes before later async-proxy reads
FM_DEV void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

FM_DEV void named_bar_sync(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// ---------------------------------------------------------------- global memory
FM_DEV uint4 ldg_nc_v4(const void* p) {  // streaming read-only load (weights)
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

FM_DEV void red_add_f32(float* p, float v) {
  asm volatile("red.global.add.f32 [%0], %1;" ::"l"(p), "f"(v) : "memory");
}

// ---------------------------------------------------------------- 4-bit dequant
// One packed word holds 8 codes q0..q7 (q_j at bits 4j).  Pair p (0..3) is
// (q_p, q_{p+4}) as a bf16x2 of the exact code values, via the exponent trick
// 0x4300 | q == 128 + q, then minus 128 (exact).
FM_DEV __nv_bfloat162 code_pair(uint32_t w, int p) {
  const uint32_t v = ((w >> (4 * p)) & 0x000F000Fu) | 0x43004300u;
  const __nv_bfloat162 magic = __floats2bfloat162_rn(128.0f, 128.0f);
  return __hsub2(*reinterpret_cast<const __nv_bfloat162*>(&v), magic);
}

// bf16(s*q + b) with a single rounding, for a pair of codes
FM_DEV uint32_t deq_pair(uint32_t w, int p, __nv_bfloat162 s2, __nv_bfloat162 b2) {
  __nv_bfloat162 r = __hfma2(code_pair(w, p), s2, b2);
  return *reinterpret_cast<uint32_t*>(&r);
}

// ---------------------------------------------------------------- tcgen05 / TMEM
FM_DEV void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {  // whole warp
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}
FM_DEV void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
FM_DEV void tmem_dealloc(uint32_t taddr, uint32_t ncols) {  // whole warp
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
FM_DEV void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
FM_DEV void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// One lane of a converged warp (the lowest): lets the compiler keep the operands of a
// single-thread tcgen05 / TMA instruction in the warp's uniform registers when the whole
// warp computed them.
FM_DEV bool elect_one() {
  uint32_t p = 0;
  asm volatile(
      "{\n\t.reg .pred P;\n\t"
      "elect.sync _|P, 0xffffffff;\n\t"
      "selp.u32 %0, 1, 0, P;\n\t}"
      : "=r"(p));
  return p != 0;
}

// D[tmem] (+)= A[smem] * B[smem]^T, kind::f16 (bf16 in, fp32 accumulate)
FM_DEV void umma_bf16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t accum) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accum)
      : "memory");
}

// arrive once on *bar when all previously issued tcgen05.mma of this thread complete
FM_DEV void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
               : "memory");
}

// Instruction descriptor: kind::f16, A/B bf16, D fp32, both K-major, shape M x N.
FM_DEV uint32_t idesc_bf16(int M, int N) {
  return (1u << 4)                                  // D format: f32
         | (1u << 7)                                // A format: bf16
         | (1u << 10)                               // B format: bf16
         | (static_cast<uint32_t>(N >> 3) << 17)    // N / 8
         | (static_cast<uint32_t>(M >> 4) << 24);   // M / 16
}

// Shared-memory matrix descriptor for a K-major tile in the 128-byte swizzle layout:
// rows of 64 bf16 (128 B), 8-row groups 1024 B apart, tile base 1024-B aligned.
FM_DEV uint64_t sdesc_sw128(uint32_t saddr) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>(1u) << 16;                 // leading byte offset (unused here)
  d |= static_cast<uint64_t>(1024u >> 4) << 32;         // stride byte offset: 8 rows
  d |= static_cast<uint64_t>(1u) << 46;                 // descriptor version (sm100)
  d |= static_cast<uint64_t>(2u) << 61;                 // SWIZZLE_128B
  return d;
}

// byte offset of 16-byte chunk c (0..7) of row r inside a 128B-swizzled tile
FM_DEV uint32_t sw128_off(int r, int c) {
  return static_cast<uint32_t>(r) * 128u + ((static_cast<uint32_t>(c) ^ (static_cast<uint32_t>(r) & 7u)) << 4);
}

// 32 lanes x 32 columns of fp32 from TMEM (lane quadrant fixed by the warp id)
FM_DEV void tmem_ld32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]),
        "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]),
        "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]),
        "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// 32 lanes x 32 columns of 32-bit values into TMEM (lane quadrant fixed by the warp
// id): column c of this thread's lane receives word c % 4 of v[c / 4]
FM_DEV void tmem_st32(uint32_t taddr, const uint4 (&v)[8]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(v[0].x), "r"(v[0].y), "r"(v[0].z), "r"(v[0].w), "r"(v[1].x), "r"(v[1].y), "r"(v[1].z), "r"(v[1].w),
      "r"(v[2].x), "r"(v[2].y), "r"(v[2].z), "r"(v[2].w), "r"(v[3].x), "r"(v[3].y), "r"(v[3].z), "r"(v[3].w),
      "r"(v[4].x), "r"(v[4].y), "r"(v[4].z), "r"(v[4].w), "r"(v[5].x), "r"(v[5].y), "r"(v[5].z), "r"(v[5].w),
      "r"(v[6].x), "r"(v[6].y), "r"(v[6].z), "r"(v[6].w), "r"(v[7].x), "r"(v[7].y), "r"(v[7].z), "r"(v[7].w)
      : "memory");
}
// this thread's earlier tcgen05.st are complete
FM_DEV void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// ---------------------------------------------------------------- legacy mma
// mma.sync m16n8k16, bf16 in, fp32 accumulate (used by the small-token GEMV path,
// where the tensor pipe only absorbs the FMAs of a bandwidth-bound kernel)
FM_DEV void mma_bf16_16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                           uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// ---------------------------------------------------------------- grid barrier
// Sense-free generation barrier for a cooperative launch.  Bounded: gives up after
// kWaitBudgetCycles, records a timeout and returns false (all blocks then exit).
struct GridSync {
  unsigned int count;
  unsigned int gen;
};

FM_DEV bool grid_sync(GridSync* gs, unsigned int nblocks, uint32_t* err, int* s_flag) {
  __syncthreads();
  if (threadIdx.x == 0) {
    volatile unsigned int* vgen = &gs->gen;
    const unsigned int g = *vgen;
    __threadfence();
    const unsigned int arrived = atomicAdd(&gs->count, 1u);
    int ok = 1;
    if (arrived == nblocks - 1) {
      atomicExch(&gs->count, 0u);
      __threadfence();
      atomicAdd(&gs->gen, 1u);
    } else {
      const long long t0 = clock64();
      while (*vgen == g) {
        if (clock64() - t0 > kWaitBudgetCycles) {
          report(err, DEVERR_TIMEOUT);
          ok = 0;
          break;
        }
        __nanosleep(64);
      }
    }
    __threadfence();
    *s_flag = ok;
  }
  __syncthreads();
  return *s_flag != 0;
}

}  // namespace fm
