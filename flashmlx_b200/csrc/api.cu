// api.cu -- host implementation of the libflashmoe C ABI (include/flashmoe.h).
//
// Mirrors the reference's operator boundary: fm_quantized_matmul / fm_gather_qmm take
// MLX's argument lists (model.cpp:478-479, 703-721), fm_moe_block takes the layer
// config and stacked weights of LlamaModel::moe_block (model.cpp:750-807, model.h:40-72).
// Every call is stream-ordered; no call allocates once fm_reserve() has sized the
// workspace for the largest batch.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <mutex>
#include <cstdio>
#include <cstring>
#include <map>
#include <string>
#include <vector>

#include "flashmoe.h"
#include "fm_internal.cuh"

namespace fm {
__global__ void route_kernel(const RouteArgs a);
__global__ void route_kernel_sigmoid(const RouteArgs a);
__global__ void route_kernel_wide(const RouteArgs a);
__global__ void route_kernel_sigmoid_wide(const RouteArgs a);
__global__ void route_last_kernel(const RouteArgs a);
__global__ void route_last_kernel_sigmoid(const RouteArgs a);
__global__ void route_cluster_kernel(const RouteArgs a);
__global__ void route_cluster_kernel_sigmoid(const RouteArgs a);
__global__ void dense_prep_kernel(const RouteArgs a);
__global__ void finalize_kernel(const float* y_acc, const float* ysh, const float* gate_sig, int64_t T, int H,
                                uint16_t* y);
void launch_finalize_pairs(int grid, cudaStream_t stream, const uint16_t* y_pairs, const int32_t* pair_pos, int k,
                           const uint16_t* ysh16, const float* gate_sig, int64_t T, int H, uint16_t* y);
__global__ void finalize_pairs_f32_kernel(const uint16_t* y_pairs, const int32_t* pair_pos, const float* score, int k,
                                          const uint16_t* ysh16, const float* gate_sig, int64_t T, int H, uint16_t* y);
__global__ void ep_plan_kernel(const EpPlanArgs a);
__global__ void ep_gather_kernel(const uint16_t* x_perm, const int32_t* sorted_token, int64_t P, int H, uint16_t* send);
__global__ void finalize_ep_kernel(const uint16_t* ret, const int32_t* pair_pos, const float* score, int k,
                                   const float* ysh32, const uint16_t* ysh16, const float* gate_sig, int64_t T, int H,
                                   uint16_t* y);
__global__ void ep_dispatch_kernel(const EpP2PArgs a);
__global__ void ep_p2p_plan_kernel(const EpP2PArgs a, EpPlanArgs pa);
__global__ void ep_release_kernel(const EpP2PArgs a, int kind);
__global__ void ep_combine_p2p_kernel(const EpP2PArgs a, const int32_t* pair_pos, const float* score, int k,
                                      const float* ysh32, const uint16_t* ysh16, const float* gate_sig, int64_t T,
                                      uint16_t* y);
cudaError_t launch_qgemv(int mode, int grid, cudaStream_t stream, const GemmArgs& a);
cudaError_t launch_dequant(const uint32_t* w, const uint16_t* s, const uint16_t* b, int64_t N, int K, int gs,
                           uint16_t* out, int num_sms, cudaStream_t st);
cudaError_t launch_embed(const uint16_t* table, int64_t V, int H, const int32_t* ids, int64_t T, uint16_t* y,
                         uint32_t* err, int num_sms, cudaStream_t st);
cudaError_t launch_rms_norm(const uint16_t* x, const uint16_t* r, const uint16_t* w, int64_t T, int H, float eps,
                            uint16_t* h_out, uint16_t* y, cudaStream_t st);
cudaError_t attn_init();
cudaError_t launch_attention(const AttnArgs& a, cudaStream_t st);
cudaError_t launch_swiglu(const uint16_t* gate, const uint16_t* up, int64_t n, uint16_t* out, int num_sms,
                          cudaStream_t st);
cudaError_t launch_argmax(const uint16_t* logits, int64_t T, int64_t V, int32_t* ids, cudaStream_t st);
cudaError_t qgemv_blocks_per_sm(int* n);
bool qgemv_tma_supports(int mode, int K, int K_shared, int gs);
cudaError_t launch_qgemv_tma(int mode, int grid, cudaStream_t stream, const GemmArgs& a, const TcMaps& maps);
cudaError_t qgemv_tma_blocks_per_sm(int* n);
int qgemv_tma_max_rows();
namespace tc {
int max_rows();
cudaError_t init();
cudaError_t max_pairs(int* n);
cudaError_t launch(int mode, int pairs, cudaStream_t stream, const GemmArgs& a, const TcMaps& maps);
}  // namespace tc
}  // namespace fm

struct fm_handle {
  int device = 0;
  cudaStream_t stream = nullptr;
  std::string last_error;
  int num_sms = 0;
  int route_blocks_per_sm = 0;
  int route_sig_blocks_per_sm = 0;  // route_kernel_sigmoid
  int route_wide_blocks_per_sm = 0;      // route_kernel_wide
  int route_sig_wide_blocks_per_sm = 0;  // route_kernel_sigmoid_wide
  int gemv_blocks_per_sm = 0;
  int gemv_tma_blocks_per_sm = 0;  // TMA-fed GEMV (qgemv_tma.cu); 0: not available
  int tc_pairs = 0;  // resident 2-CTA clusters of the tcgen05 kernel
  int path = FM_PATH_AUTO;
  int last_path = 0;  // expert-product path the last call took (fm_last_path)
  int route_mode = FM_ROUTE_AUTO;
  bool attn_ready = false;  // attention kernels' shared-memory opt-in done (first fm_attention)
  uint8_t* ws = nullptr;
  size_t ws_bytes = 0;
  bool borrowed_ws = false;  // ws is fixed scratch the handle must never grow or free
  // expert parallelism (fm_ep_*): this rank's place, the dispatch the next calls
  // refer to, and the owner-side workspace (sized by the rows received)
  int ep_rank = 0;
  int ep_world = 1;
  int64_t ep_T = -1;       // tokens of the last fm_ep_dispatch (-1: none)
  int64_t ep_R = 0;        // rows received by the last fm_ep_experts
  int ep_stage = 0;        // 1 after dispatch, 2 after experts
  bool ep_ysh_bf16 = false;
  bool ep_shared = false;
  uint8_t* ep_ws = nullptr;
  size_t ep_ws_bytes = 0;
  // peer-memory exchange (fm_ep_p2p_*): this rank's region, every rank's mapping of it
  struct P2P {
    uint8_t* region = nullptr;  // own region (cudaMalloc, exported by CUDA IPC)
    size_t bytes = 0;
    uint8_t* peer[fm::kEpMaxWorld] = {};
    bool mapped[fm::kEpMaxWorld] = {};  // peer[r] opened from an IPC handle
    bool open = false;
    int world = 0, E = 0, H = 0, k = 0;
    int64_t max_tokens = 0;
    int64_t off_flags = 0, off_counts = 0, off_recv = 0, off_ret = 0, cap_recv = 0, cap_ret = 0;
    uint32_t epoch = 0;
    int coop_blocks = 0;  // co-resident blocks of the dispatch kernel
  } p2p;
  // kernel timing (fm_profile_enable)
  bool profile = false;
  struct Pending {
    const char* name;
    cudaEvent_t a, b;
  };
  std::vector<Pending> pending;
  std::vector<cudaEvent_t> event_pool;
  struct Total {
    const char* name;  // static string literal
    int64_t launches;
    double ms;
  };
  std::map<std::string, Total> totals;
  const char* open_name = nullptr;
  cudaEvent_t open_ev = nullptr;
};

namespace {

using fm::GemmArgs;
using fm::RouteArgs;
using fm::TileTable;

constexpr size_t kCtrlBytes = 256;  // error word + grid-sync counters, persistent

int set_err(fm_handle* h, int status, const std::string& msg) {
  if (h) h->last_error = msg;
  return status;
}

int cuda_err(fm_handle* h, cudaError_t e, const char* what) {
  return set_err(h, FM_ECUDA, std::string(what) + ": " + cudaGetErrorString(e));
}

size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Per-call workspace carve-up.
struct Plan {
  size_t total = 0;
  size_t partial, x_perm, topk_ids, topk_score, gate_sig, row_src, chunk_counts, pair_rank, totals, offsets,
      sorted_token, sorted_score, sorted_flat, pair_pos, tab_a, tab_b, a_sorted, a_shared, y_acc, ysh, y_pairs, ysh16;
  size_t add(size_t bytes) {
    const size_t off = total;
    total = align_up(total + bytes, 256);
    return off;
  }
};

// tcp: the expert products run on the tcgen05 path (per-pair bf16 down rows combined
// by finalize_pairs_kernel) rather than the GEMV path (fp32 atomic combine buffers)
Plan make_plan(int64_t T, int64_t x_rows, int H, int E, int k, int epad, int ksplit, int64_t a_cols,
               int64_t ash_cols, bool shared, bool moe, bool tcp) {
  Plan p;
  p.total = kCtrlBytes;
  const int64_t P = T * k;
  const int64_t nchunks = (T + fm::kRouteChunk - 1) / fm::kRouteChunk;
  p.partial = p.add(moe ? sizeof(float) * ksplit * T * epad : 0);
  p.x_perm = p.add(sizeof(uint16_t) * x_rows * H);
  p.topk_ids = p.add(sizeof(int32_t) * P);
  p.topk_score = p.add(sizeof(float) * P);
  p.gate_sig = p.add(sizeof(float) * T);
  p.row_src = p.add(sizeof(int32_t) * T);
  p.chunk_counts = p.add(sizeof(int32_t) * nchunks * E);
  p.pair_rank = p.add(sizeof(int32_t) * P);
  p.totals = p.add(sizeof(int32_t) * E);
  p.offsets = p.add(sizeof(int32_t) * (E + 1));
  p.sorted_token = p.add(sizeof(int32_t) * P);
  p.sorted_score = p.add(sizeof(float) * P);
  p.sorted_flat = p.add(sizeof(int32_t) * P);
  p.pair_pos = p.add(moe && tcp ? sizeof(int32_t) * P : 0);
  p.tab_a = p.add(sizeof(TileTable));
  p.tab_b = p.add(moe ? sizeof(TileTable) : 0);
  p.a_sorted = p.add(moe ? sizeof(uint16_t) * P * a_cols : 0);
  p.a_shared = p.add(moe && shared ? sizeof(uint16_t) * T * ash_cols : 0);
  p.y_acc = p.add(moe && !tcp ? sizeof(float) * T * H : 0);
  p.ysh = p.add(moe && shared && !tcp ? sizeof(float) * T * H : 0);
  p.y_pairs = p.add(moe && tcp ? sizeof(uint16_t) * P * H : 0);
  p.ysh16 = p.add(moe && shared && tcp ? sizeof(uint16_t) * T * H : 0);
  return p;
}

// the allocation ensure_ws makes for a request of `bytes` (1/8 slack, whole MiB)
size_t ws_alloc_bytes(size_t bytes) { return align_up(bytes + bytes / 8, 1 << 20); }

// workspace of the largest MoE-block call of max_tokens tokens on either expert path
// (the router's K split at its maximum)
size_t reserve_need(const fm_moe_config* c, int64_t max_tokens) {
  const int epad = (c->num_experts + 1 + 7) / 8 * 8;
  size_t need = 0;
  for (bool tcp : {false, true})
    need = std::max(need, make_plan(max_tokens, max_tokens, c->hidden, c->num_experts, c->top_k, epad,
                                    fm::kRouterMaxKsplit, c->inter, c->shared_inter, c->shared_inter > 0, true, tcp)
                              .total);
  return need;
}

int ensure_ws(fm_handle* h, size_t bytes) {
  if (bytes <= h->ws_bytes) return FM_OK;
  if (h->borrowed_ws) return set_err(h, FM_ETOOLARGE, "request exceeds the fixed scratch");
  cudaError_t e = cudaStreamSynchronize(h->stream);
  if (e != cudaSuccess) return cuda_err(h, e, "cudaStreamSynchronize");
  if (h->ws) cudaFree(h->ws);
  h->ws = nullptr;
  h->ws_bytes = 0;
  const size_t want = ws_alloc_bytes(bytes);
  e = cudaMalloc(&h->ws, want);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return set_err(h, FM_ENOMEM, std::string("workspace allocation failed: ") + cudaGetErrorString(e));
  }
  h->ws_bytes = want;
  e = cudaMemsetAsync(h->ws, 0, kCtrlBytes, h->stream);
  if (e != cudaSuccess) return cuda_err(h, e, "cudaMemsetAsync");
  return FM_OK;
}

cudaEvent_t take_event(fm_handle* h) {
  if (!h->event_pool.empty()) {
    cudaEvent_t e = h->event_pool.back();
    h->event_pool.pop_back();
    return e;
  }
  cudaEvent_t e = nullptr;
  cudaEventCreate(&e);
  return e;
}

// brackets the next kernel launch with events when profiling is on
void prof_begin(fm_handle* h, const char* name) {
  if (!h->profile) return;
  h->open_name = name;
  h->open_ev = take_event(h);
  cudaEventRecord(h->open_ev, h->stream);
}

void prof_end(fm_handle* h) {
  if (!h->profile || !h->open_ev) return;
  cudaEvent_t b = take_event(h);
  cudaEventRecord(b, h->stream);
  h->pending.push_back({h->open_name, h->open_ev, b});
  h->open_ev = nullptr;
}

uint32_t* err_word(fm_handle* h) { return reinterpret_cast<uint32_t*>(h->ws); }
fm::GridSync* grid_sync(fm_handle* h) { return reinterpret_cast<fm::GridSync*>(h->ws + 64); }
unsigned int* arrive_count(fm_handle* h) { return reinterpret_cast<unsigned int*>(h->ws + 72); }
// routing-kernel phase timers: 4 x u64 ns + a launch count, accumulated on the device
unsigned long long* phase_ns(fm_handle* h) { return reinterpret_cast<unsigned long long*>(h->ws + 128); }

template <class T>
T* at(fm_handle* h, size_t off) {
  return reinterpret_cast<T*>(h->ws + off);
}

bool quant_ok(int K, int gs, int bits) {
  return bits == 4 && (gs == 32 || gs == 64 || gs == 128) && K > 0 && K % gs == 0;
}

int launch_route(fm_handle* h, RouteArgs& ra, int64_t items, bool sigmoid = false) {
  const int max_blocks = (sigmoid ? h->route_sig_blocks_per_sm : h->route_blocks_per_sm) * h->num_sms;
  const int64_t nchunks = (ra.T + fm::kRouteChunk - 1) / fm::kRouteChunk;
  ra.arrive = arrive_count(h);
  const bool cluster = h->route_mode == FM_ROUTE_CLUSTER || h->route_mode == FM_ROUTE_AUTO;
  if (cluster && nchunks <= fm::kRouteLastMaxChunks) {
    // one cluster of kRouteClusterCtas CTAs (hardware cluster barriers, no co-residency
    // requirement beyond the cluster itself)
    prof_begin(h, ra.do_router ? "route" : "route_given");
    if (sigmoid) fm::route_cluster_kernel_sigmoid<<<fm::kRouteClusterCtas, fm::kRouteThreads, 0, h->stream>>>(ra);
    else fm::route_cluster_kernel<<<fm::kRouteClusterCtas, fm::kRouteThreads, 0, h->stream>>>(ra);
    prof_end(h);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_err(h, e, "route_cluster_kernel launch");
    return FM_OK;
  }
  if (h->route_mode == FM_ROUTE_LAST_BLOCK && nchunks <= fm::kRouteLastMaxChunks) {
    // one warp per phase-1 item, and enough blocks that zeroing the fp32 accumulators
    // takes at most 8 float4 stores per thread; no co-residency needed (nothing waits on
    // another block)
    const int64_t zero_blocks = (ra.zero0_n + ra.zero1_n + 8191) / 8192;
    const int64_t want = std::max<int64_t>((items + 7) / 8, zero_blocks);
    const int grid = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(want, max_blocks)));
    prof_begin(h, ra.do_router ? "route" : "route_given");
    if (sigmoid) fm::route_last_kernel_sigmoid<<<grid, fm::kRouteThreads, 0, h->stream>>>(ra);
    else fm::route_last_kernel<<<grid, fm::kRouteThreads, 0, h->stream>>>(ra);
    prof_end(h);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_err(h, e, "route_last_kernel launch");
    return FM_OK;
  }
  int64_t want = std::max<int64_t>((items + 7) / 8, nchunks);
  want = std::max<int64_t>(want, std::min<int64_t>(ra.E, h->num_sms));
  // the wide instance (two CTAs per SM) when the one-CTA-per-SM grid would cap the blocks
  const int wide_blocks = (sigmoid ? h->route_sig_wide_blocks_per_sm : h->route_wide_blocks_per_sm) * h->num_sms;
  const bool wide = want > max_blocks && wide_blocks > max_blocks;
  const int grid = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(want, wide ? wide_blocks : max_blocks)));
  void* args[] = {&ra};
  prof_begin(h, ra.do_router ? "route" : "route_given");
  const void* fn = sigmoid ? (wide ? reinterpret_cast<const void*>(&fm::route_kernel_sigmoid_wide)
                                   : reinterpret_cast<const void*>(&fm::route_kernel_sigmoid))
                           : (wide ? reinterpret_cast<const void*>(&fm::route_kernel_wide)
                                   : reinterpret_cast<const void*>(&fm::route_kernel));
  cudaError_t e = cudaLaunchCooperativeKernel(fn, dim3(grid), dim3(fm::kRouteThreads), args, 0, h->stream);
  prof_end(h);
  if (e != cudaSuccess) return cuda_err(h, e, "route_kernel launch");
  return FM_OK;
}

// ---------------------------------------------------------------- TMA descriptors
PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

// 2D row-major tensor [outer, inner] with the 128-byte swizzle; a null base leaves the
// descriptor zeroed (the kernel never touches it)
bool encode_2d(CUtensorMap* m, bool u32, const void* base, uint64_t inner, uint64_t outer, uint32_t box_inner,
               uint32_t box_outer) {
  std::memset(m, 0, sizeof(*m));
  if (!base) return true;
  auto fn = tensor_map_encoder();
  if (!fn) return false;
  const cuuint64_t dims[2] = {inner, outer};
  const cuuint64_t strides[1] = {inner * (u32 ? 4u : 2u)};
  const cuuint32_t box[2] = {box_inner, box_outer};
  const cuuint32_t es[2] = {1, 1};
  return fn(m, u32 ? CU_TENSOR_MAP_DATA_TYPE_UINT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims,
            strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// codes of a [rows, K] 4-bit matrix: uint32 words, box {4 k-steps, box_rows rows}
bool encode_codes(CUtensorMap* m, const uint32_t* w, int64_t rows, int K, uint32_t box_rows) {
  return encode_2d(m, true, w, static_cast<uint64_t>(K / 8), static_cast<uint64_t>(rows), 32, box_rows);
}

// bf16 activation rows [rows, cols], 128B-swizzled boxes of 64 columns: m[0] with 32-row
// boxes, m[2] (TcMaps::act[i + 2] for m = &act[i]) with kActBigBoxRows-row boxes
bool encode_act(CUtensorMap* m, const uint16_t* x, int64_t rows, int64_t cols) {
  return encode_2d(m, false, x, static_cast<uint64_t>(cols), static_cast<uint64_t>(rows), 64, 32) &&
         encode_2d(m + 2, false, x, static_cast<uint64_t>(cols), static_cast<uint64_t>(rows), 64, fm::kActBigBoxRows);
}

// tma_gemv: the GEMV path's TMA-fed kernel (qgemv_tma.cu), whose tile table was planned
// with up to qgemv_tma_max_rows() activation rows per unit; otherwise qgemv.cu (8 rows)
template <int MODE>
int launch_gemm(fm_handle* h, const GemmArgs& ga, bool tcgen05, const fm::TcMaps* maps = nullptr,
                bool tma_gemv = false) {
  static const char* names[2][5] = {{"qgemv_gateup", "qgemv_down", "qgemv_plain", "qgemv_relu2", "qgemv_down"},
                                    {"qgemm_tc_gateup", "qgemm_tc_down", "qgemm_tc_plain", "qgemm_tc_relu2", ""}};
  if ((tcgen05 || tma_gemv) && !maps) return set_err(h, FM_EINVAL, "TMA launch without tensor maps");
  if (tcgen05 && MODE == fm::MODE_DOWN_F32) return set_err(h, FM_EUNSUPPORTED, "fp32-score down runs on the GEMV path");
  prof_begin(h, names[tcgen05 ? 1 : 0][MODE]);
  const cudaError_t e =
      tcgen05    ? fm::tc::launch(MODE, h->tc_pairs, h->stream, ga, *maps)
      : tma_gemv ? fm::launch_qgemv_tma(MODE, h->num_sms * h->gemv_tma_blocks_per_sm, h->stream, ga, *maps)
                 : fm::launch_qgemv(MODE, h->num_sms * std::max(1, h->gemv_blocks_per_sm), h->stream, ga);
  prof_end(h);
  if (e != cudaSuccess) return cuda_err(h, e, tcgen05 ? "qgemm_tc launch" : "qgemv launch");
  return FM_OK;
}

// K slices of the router's partial logits: enough items to fill the GPU, at least two
// 32-wide k-blocks per item, and at most ~4096 partials per token to sum (the top-k
// phase reads ksplit partials of every logit, 32 loads in flight per lane; at 128
// experts and 256 tokens, 31 slices instead of 7 took phase 1 from 17 to 9 us and the
// top-k phase from 15 to 17 us)
int router_ksplit(const fm_handle* h, int64_t T, int H, int E) {
  const int64_t ntt = (T + 15) / 16;
  const int64_t target = static_cast<int64_t>(h->num_sms) * 16;
  const int cap = std::min(std::min(fm::kRouterMaxKsplit, std::max(1, H / 64)), std::max(2, 4096 / (E + 1)));
  int64_t ks = std::min<int64_t>(cap, std::max<int64_t>(1, (target + ntt - 1) / ntt));
  // The grid form's wide instance (launch_route takes it when the one-CTA-per-SM grid would
  // cap the blocks) gives each item of two 16-token tiles to one warp, once: as many slices
  // as fill its warps, rounded down, so that no warp walks a second item's chain (at
  // 16384 tokens 4 slices keep 2048 of 2368 warps busy, where 3 kept 1536 and 5 needed
  // two rounds)
  const int64_t max_blocks = static_cast<int64_t>(h->route_blocks_per_sm) * h->num_sms;
  const int64_t wide_warps = static_cast<int64_t>(h->route_wide_blocks_per_sm) * h->num_sms * (fm::kRouteThreads / 32);
  const int64_t nchunks = (T + fm::kRouteChunk - 1) / fm::kRouteChunk;
  if (wide_warps > max_blocks * (fm::kRouteThreads / 32) && std::max((ntt * ks + 7) / 8, nchunks) > max_blocks)
    ks = std::min<int64_t>(cap, std::max<int64_t>(1, wide_warps / ((ntt + 1) / 2)));
  return static_cast<int>(ks);
}

// The GEMV path covers group sizes 64 and 128 (each 64-wide half of its 128-wide K
// chunks lies inside one quant group); group size 32 always runs on tcgen05.
bool use_tc(const fm_handle* h, int64_t pairs, int E, int gs) {
  if (gs != 64 && gs != 128) return true;
  if (h->path == FM_PATH_GEMV) return false;
  if (h->path == FM_PATH_TCGEN05) return true;
  return pairs >= 24LL * E;  // ~24+ activation rows per matrix on average
}

int check_moe(fm_handle* h, const fm_moe_config* c, const fm_moe_weights* w) {
  if (!c || !w) return set_err(h, FM_EINVAL, "null config or weights");
  if (c->hidden <= 0 || c->inter <= 0 || c->num_experts <= 0 || c->top_k <= 0 || c->top_k > c->num_experts)
    return set_err(h, FM_EINVAL, "bad MoE dimensions");
  if (c->num_experts > fm::kMaxExperts || c->top_k > 16)
    return set_err(h, FM_EUNSUPPORTED, "num_experts > 512 or top_k > 16");
  if (!quant_ok(c->hidden, c->group_size, c->bits) || !quant_ok(c->inter, c->group_size, c->bits))
    return set_err(h, FM_EUNSUPPORTED, "only 4-bit affine with group size 32/64/128 is implemented");
  if (c->hidden % 128 || c->inter % 128)
    return set_err(h, FM_EUNSUPPORTED, "hidden and moe_intermediate_size must be multiples of 128");
  if (c->router_quantized || c->shared_gate_quantized)
    return set_err(h, FM_EUNSUPPORTED, "quantized router / shared-expert gate not implemented");
  if (c->shared_inter < 0) return set_err(h, FM_EINVAL, "negative shared_inter");
  if (c->shared_inter > 0) {
    if (c->shared_inter % 128)
      return set_err(h, FM_EUNSUPPORTED, "shared_expert_intermediate_size must be a multiple of 128");
    if (!w->shared_gate.w || !w->shared_up.w || !w->shared_down.w || !w->shared_gate.scales ||
        !w->shared_up.scales || !w->shared_down.scales || !w->shared_expert_gate_w)
      return set_err(h, FM_EINVAL, "shared expert weights missing");
  }
  if (!w->router_w || !w->gate.w || !w->up.w || !w->down.w || !w->gate.scales || !w->up.scales ||
      !w->down.scales)
    return set_err(h, FM_EINVAL, "expert weights missing");
  return FM_OK;
}


// ---------------------------------------------------------------- expert parallelism
// Balanced contiguous expert ranges: the first E % world ranks own one expert more.
void ep_range(int E, int rank, int world, int* first, int* count) {
  const int base = E / world, rem = E % world;
  *count = base + (rank < rem ? 1 : 0);
  *first = rank * base + std::min(rank, rem);
}

// Token-side workspace (fm_ep_dispatch .. fm_ep_combine): routing state, the
// pair-position map, and the send rows.
struct EpPlan1 {
  size_t total = 0;
  size_t partial, x_perm, topk_ids, topk_score, gate_sig, row_src, chunk_counts, pair_rank, totals, offsets,
      sorted_token, sorted_score, sorted_flat, pair_pos, send;
  size_t add(size_t bytes) {
    const size_t off = total;
    total = align_up(total + bytes, 256);
    return off;
  }
};

EpPlan1 make_ep_plan1(int64_t T, int H, int E, int k, int epad, int ksplit) {
  EpPlan1 p;
  p.total = kCtrlBytes;
  const int64_t P = T * k;
  const int64_t nchunks = (T + fm::kRouteChunk - 1) / fm::kRouteChunk;
  p.partial = p.add(sizeof(float) * ksplit * T * epad);
  p.x_perm = p.add(sizeof(uint16_t) * T * H);
  p.topk_ids = p.add(sizeof(int32_t) * P);
  p.topk_score = p.add(sizeof(float) * P);
  p.gate_sig = p.add(sizeof(float) * T);
  p.row_src = p.add(sizeof(int32_t) * T);
  p.chunk_counts = p.add(sizeof(int32_t) * nchunks * E);
  p.pair_rank = p.add(sizeof(int32_t) * P);
  p.totals = p.add(sizeof(int32_t) * E);
  p.offsets = p.add(sizeof(int32_t) * (E + 1));
  p.sorted_token = p.add(sizeof(int32_t) * P);
  p.sorted_score = p.add(sizeof(float) * P);
  p.sorted_flat = p.add(sizeof(int32_t) * P);
  p.pair_pos = p.add(sizeof(int32_t) * P);
  p.send = p.add(sizeof(uint16_t) * P * H);
  return p;
}

// Owner-side workspace (fm_ep_experts): tile tables and expert intermediates for the
// R received rows plus this rank's shared-expert rows.
struct EpPlan2 {
  size_t total = 0;
  size_t tab_a, tab_b, recv_counts, recv_total, row_map, unit_score, a_sorted, a_shared, ysh;
  size_t row_dst = 0;  // peer-memory exchange only
  size_t add(size_t bytes) {
    const size_t off = total;
    total = align_up(total + bytes, 256);
    return off;
  }
};

EpPlan2 make_ep_plan2(int64_t R, int64_t T, int H, int I, int Is, int nseg, bool shared) {
  EpPlan2 p;
  p.tab_a = p.add(sizeof(TileTable));
  p.tab_b = p.add(sizeof(TileTable));
  p.recv_counts = p.add(sizeof(int32_t) * nseg);
  p.recv_total = p.add(sizeof(int32_t));
  p.row_map = p.add(sizeof(int32_t) * std::max<int64_t>(R, 1));
  p.unit_score = p.add(sizeof(float) * std::max<int64_t>(R, 1));
  p.a_sorted = p.add(sizeof(uint16_t) * R * I);
  p.a_shared = p.add(shared ? sizeof(uint16_t) * T * Is : 0);
  p.ysh = p.add(shared ? sizeof(float) * T * H : 0);  // fp32 (GEMV) or bf16 (tcgen05) rows
  return p;
}

// The same plus each received row's d destination (a row of its source rank's ret
// buffer): R is the receive capacity, the host does not learn the count.
EpPlan2 make_ep_plan2_p2p(int64_t R, int64_t T, int H, int I, int Is, int nseg, bool shared) {
  EpPlan2 p = make_ep_plan2(R, T, H, I, Is, nseg, shared);
  p.row_dst = p.add(sizeof(uint16_t*) * std::max<int64_t>(R, 1));
  return p;
}

int ensure_ep_ws(fm_handle* h, size_t bytes) {
  if (bytes <= h->ep_ws_bytes) return FM_OK;
  if (h->borrowed_ws) return set_err(h, FM_ETOOLARGE, "expert parallelism needs an allocating handle");
  cudaError_t e = cudaStreamSynchronize(h->stream);
  if (e != cudaSuccess) return cuda_err(h, e, "cudaStreamSynchronize");
  if (h->ep_ws) cudaFree(h->ep_ws);
  h->ep_ws = nullptr;
  h->ep_ws_bytes = 0;
  const size_t want = align_up(bytes + bytes / 8, 1 << 20);
  e = cudaMalloc(&h->ep_ws, want);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return set_err(h, FM_ENOMEM, std::string("expert-parallel workspace allocation failed: ") + cudaGetErrorString(e));
  }
  h->ep_ws_bytes = want;
  return FM_OK;
}

template <class T>
T* ep_at(fm_handle* h, size_t off) {
  return reinterpret_cast<T*>(h->ep_ws + off);
}

int grid_for(const fm_handle* h, int64_t work) {
  return static_cast<int>(std::max<int64_t>(1, std::min<int64_t>((work + 255) / 256, static_cast<int64_t>(h->num_sms) * 8)));
}

// Routing of an expert-parallel call over this rank's T tokens (token-side workspace p).
RouteArgs ep_route_args(fm_handle* h, const fm_moe_config* c, const fm_moe_weights* w, const uint16_t* x, int64_t T,
                        int ksplit, const EpPlan1& p) {
  const int H = c->hidden, E = c->num_experts, k = c->top_k;
  const bool shared = c->shared_inter > 0;
  RouteArgs ra;
  std::memset(&ra, 0, sizeof(ra));
  ra.x = x;
  ra.router_w = static_cast<const uint16_t*>(w->router_w);
  ra.shared_gate_w = shared ? static_cast<const uint16_t*>(w->shared_expert_gate_w) : nullptr;
  ra.router_bias = w->router_bias;
  ra.T = T;
  ra.H = H;
  ra.E = E;
  ra.k = k;
  ra.norm_topk = c->norm_topk_prob;
  ra.do_router = 1;
  ra.ksplit = ksplit;
  ra.epad = (E + 1 + 7) / 8 * 8;
  ra.partial = at<float>(h, p.partial);
  ra.x_perm = at<uint16_t>(h, p.x_perm);
  ra.x_rows = T;
  ra.topk_ids = at<int32_t>(h, p.topk_ids);
  ra.topk_score = at<float>(h, p.topk_score);
  ra.gate_sig = at<float>(h, p.gate_sig);
  ra.row_src = at<int32_t>(h, p.row_src);
  ra.chunk_counts = at<int32_t>(h, p.chunk_counts);
  ra.pair_rank = at<int32_t>(h, p.pair_rank);
  ra.totals = at<int32_t>(h, p.totals);
  ra.offsets = at<int32_t>(h, p.offsets);
  ra.sorted_token = at<int32_t>(h, p.sorted_token);
  ra.sorted_score = at<float>(h, p.sorted_score);
  ra.sorted_flat = at<int32_t>(h, p.sorted_flat);
  ra.pair_pos = at<int32_t>(h, p.pair_pos);
  ra.chunk_max = 8;
  ra.chunk_align = 8;
  ra.has_shared = shared ? 1 : 0;
  ra.gsync = grid_sync(h);
  ra.err = err_word(h);
  ra.phase_ns = phase_ns(h);
  return ra;
}

// Token-side checks of fm_ep_dispatch and fm_ep_p2p_forward.
int check_ep_route(fm_handle* h, const fm_moe_config* c, const fm_moe_weights* w, const uint16_t* x, int64_t T) {
  if (!c || !w) return set_err(h, FM_EINVAL, "null argument");
  if (c->hidden <= 0 || c->num_experts <= 0 || c->top_k <= 0 || c->top_k > c->num_experts || c->top_k > 16 ||
      c->num_experts > fm::kMaxExperts)
    return set_err(h, FM_EINVAL, "bad MoE dimensions");
  if (c->hidden % 128) return set_err(h, FM_EUNSUPPORTED, "hidden must be a multiple of 128");
  if (c->router_quantized || c->shared_gate_quantized)
    return set_err(h, FM_EUNSUPPORTED, "quantized router / shared-expert gate not implemented");
  if (!w->router_w || (c->shared_inter > 0 && !w->shared_expert_gate_w))
    return set_err(h, FM_EINVAL, "router weights missing");
  if (T < 0 || (T > 0 && !x)) return set_err(h, FM_EINVAL, "bad x / T");
  if (!aligned16(x)) return set_err(h, FM_EINVAL, "x must be 16-byte aligned");
  if (T > (1LL << 24)) return set_err(h, FM_EUNSUPPORTED, "T too large");
  return FM_OK;
}


// Unmaps the peers' regions and frees this rank's own (every rank must have finished
// its calls: the regions are written by peers during a call).
void p2p_close(fm_handle* h) {
  auto& q = h->p2p;
  if (q.region || q.open) cudaStreamSynchronize(h->stream);
  for (int r = 0; r < fm::kEpMaxWorld; ++r) {
    if (q.mapped[r] && q.peer[r]) cudaIpcCloseMemHandle(q.peer[r]);
    q.mapped[r] = false;
    q.peer[r] = nullptr;
  }
  if (q.region) cudaFree(q.region);
  q = fm_handle::P2P();
}

// Owner-side planner arguments (tile groups over the (source rank, local expert)
// segments and the shared expert's own tokens).
fm::EpPlanArgs ep_plan_args(fm_handle* h, const fm_moe_config* c, int E_local, int64_t T, bool shared, bool tcp,
                            const EpPlan2& p2) {
  fm::EpPlanArgs pa;
  std::memset(&pa, 0, sizeof(pa));
  pa.recv_counts = ep_at<int32_t>(h, p2.recv_counts);
  pa.world = h->ep_world;
  pa.E_local = E_local;
  pa.T_shared = shared ? static_cast<int>(T) : 0;
  pa.a_n = c->inter;
  pa.a_n_shared = c->shared_inter;
  pa.b_n = c->hidden;
  pa.a_rows_per_block = tcp ? 128 : 64;
  pa.b_rows_per_block = tcp ? 256 : 128;
  pa.chunk_max = tcp ? fm::tc::max_rows() : 8;
  pa.chunk_align = tcp ? 16 : 8;
  pa.b_ksplit_shared = tcp ? 1 : std::max(1, c->shared_inter / std::max(1, c->inter));
  pa.tab_a = ep_at<TileTable>(h, p2.tab_a);
  pa.tab_b = ep_at<TileTable>(h, p2.tab_b);
  pa.row_map = ep_at<int32_t>(h, p2.row_map);
  pa.unit_score = ep_at<float>(h, p2.unit_score);
  pa.recv_total = ep_at<int32_t>(h, p2.recv_total);
  pa.err = err_word(h);
  return pa;
}

// Owner-side checks of fm_ep_experts and fm_ep_p2p_forward.
int check_ep_experts(fm_handle* h, const fm_moe_config* c, const fm_moe_weights* w, bool routed, bool shared) {
  const int H = c->hidden, I = c->inter, Is = c->shared_inter;
  if (I <= 0 || I % 128 || (Is > 0 && Is % 128) || !quant_ok(H, c->group_size, c->bits) ||
      !quant_ok(I, c->group_size, c->bits))
    return set_err(h, FM_EUNSUPPORTED, "inter / shared sizes must be multiples of 128, 4-bit affine");
  if (routed && (!w->gate.w || !w->up.w || !w->down.w || !w->gate.scales || !w->up.scales || !w->down.scales))
    return set_err(h, FM_EINVAL, "local expert weights missing");
  if (shared && (!w->shared_gate.w || !w->shared_up.w || !w->shared_down.w))
    return set_err(h, FM_EINVAL, "shared expert weights missing");
  return FM_OK;
}

// Owner-side expert GEMMs of an expert-parallel call: gate/up + SwiGLU, then down into
// d_rows (bf16(d), one row per received row, in receive order) or, with d_rowptr, into
// the row each received row points at (another rank's memory), over the tile tables
// pa holds.  R rows of recv_rows may be read (the received rows, or their capacity when
// the host does not know the count).  The shared expert runs on this rank's own tokens.
int ep_gemms(fm_handle* h, const fm_moe_config* c, const fm_moe_weights* w, const uint16_t* recv_rows, int64_t R,
             int64_t T, int E_local, bool shared, bool tcp, const EpPlan1& p1, const EpPlan2& p2,
             const fm::EpPlanArgs& pa, uint16_t* d_rows, uint16_t* const* d_rowptr = nullptr) {
  const int H = c->hidden, I = c->inter, Is = c->shared_inter;
  int rc = FM_OK;
  uint16_t* x_perm = at<uint16_t>(h, p1.x_perm);
  GemmArgs ga;
  std::memset(&ga, 0, sizeof(ga));
  ga.gs = c->group_size;
  ga.err = err_word(h);
  ga.sorted_token = pa.row_map;
  ga.sorted_score = pa.unit_score;
  ga.sorted_flat = pa.row_map;
  ga.K = H;
  ga.K_shared = H;
  ga.N = I;
  ga.N_shared = Is;
  ga.w0 = w->gate.w; ga.s0 = w->gate.scales; ga.b0 = w->gate.biases;
  ga.w1 = w->up.w; ga.s1 = w->up.scales; ga.b1 = w->up.biases;
  if (shared) {
    ga.sw0 = w->shared_gate.w; ga.ss0 = w->shared_gate.scales; ga.sb0 = w->shared_gate.biases;
    ga.sw1 = w->shared_up.w; ga.ss1 = w->shared_up.scales; ga.sb1 = w->shared_up.biases;
  }
  ga.act = recv_rows;
  ga.act_ld = H;
  ga.act_shared = x_perm;
  ga.act_shared_ld = H;
  ga.out = ep_at<uint16_t>(h, p2.a_sorted);
  ga.out_ld = I;
  ga.out_shared = shared ? ep_at<uint16_t>(h, p2.a_shared) : nullptr;
  ga.out_shared_ld = Is;
  ga.tab = pa.tab_a;
  fm::TcMaps maps_gu, maps_dn;
  if (tcp) {
    const bool ok =
        encode_codes(&maps_gu.code[0], w->gate.w, static_cast<int64_t>(E_local) * I, H, 64) &&
        encode_codes(&maps_gu.code[1], w->up.w, static_cast<int64_t>(E_local) * I, H, 64) &&
        encode_codes(&maps_gu.code[2], shared ? w->shared_gate.w : nullptr, Is, H, 64) &&
        encode_codes(&maps_gu.code[3], shared ? w->shared_up.w : nullptr, Is, H, 64) &&
        encode_act(&maps_gu.act[0], R > 0 ? recv_rows : nullptr, R, H) &&
        encode_act(&maps_gu.act[1], shared ? x_perm : nullptr, T, H) &&
        encode_codes(&maps_dn.code[0], w->down.w, static_cast<int64_t>(E_local) * H, I, 128) &&
        encode_codes(&maps_dn.code[1], nullptr, 0, I, 128) &&
        encode_codes(&maps_dn.code[2], shared ? w->shared_down.w : nullptr, H, shared ? Is : I, 128) &&
        encode_codes(&maps_dn.code[3], nullptr, 0, I, 128) &&
        encode_act(&maps_dn.act[0], R > 0 ? ep_at<uint16_t>(h, p2.a_sorted) : nullptr, R, I) &&
        encode_act(&maps_dn.act[1], shared ? ep_at<uint16_t>(h, p2.a_shared) : nullptr, T, Is);
    if (!ok) return set_err(h, FM_ECUDA, "cuTensorMapEncodeTiled failed (alignment or driver entry point)");
  }
  rc = launch_gemm<fm::MODE_GATEUP>(h, ga, tcp, &maps_gu);
  if (rc) return rc;
  GemmArgs gd = ga;
  gd.K = I;
  gd.K_shared = Is;
  gd.N = H;
  gd.N_shared = H;
  gd.w0 = w->down.w; gd.s0 = w->down.scales; gd.b0 = w->down.biases;
  gd.w1 = nullptr; gd.s1 = nullptr; gd.b1 = nullptr;
  if (shared) {
    gd.sw0 = w->shared_down.w; gd.ss0 = w->shared_down.scales; gd.sb0 = w->shared_down.biases;
  }
  gd.sw1 = nullptr; gd.ss1 = nullptr; gd.sb1 = nullptr;
  gd.act = ga.out;
  gd.act_ld = I;
  gd.act_shared = ga.out_shared;
  gd.act_shared_ld = Is;
  gd.out = nullptr;
  gd.out_shared = nullptr;
  gd.y_pairs = d_rowptr ? nullptr : d_rows;
  gd.y_rowptr = d_rowptr;
  gd.y_acc = nullptr;
  gd.ysh = (shared && !tcp) ? ep_at<float>(h, p2.ysh) : nullptr;
  gd.ysh16 = (shared && tcp) ? ep_at<uint16_t>(h, p2.ysh) : nullptr;
  gd.y_ld = H;
  gd.tab = pa.tab_b;
  return launch_gemm<fm::MODE_DOWN>(h, gd, tcp, &maps_dn);
}

}  // namespace

extern "C" {

const char* fm_status_string(int s) {
  switch (s) {
    case FM_OK: return "ok";
    case FM_EINVAL: return "invalid argument";
    case FM_EUNSUPPORTED: return "unsupported";
    case FM_ECUDA: return "cuda error";
    case FM_ENCCL: return "transport error";
    case FM_ETIMEOUT: return "device wait timed out";
    case FM_EDEVICE: return "device-side check failed";
    case FM_ENOMEM: return "out of device memory";
    case FM_ETOOLARGE: return "request needs more than the fixed no-allocation scratch";
    default: return "unknown status";
  }
}

int fm_create(fm_handle** out, int device, void* stream) {
  if (!out) return FM_EINVAL;
  *out = nullptr;
  fm_handle* h = new (std::nothrow) fm_handle();
  if (!h) return FM_ENOMEM;
  h->device = device;
  h->stream = static_cast<cudaStream_t>(stream);
  cudaError_t e = cudaSetDevice(device);
  if (e == cudaSuccess) e = cudaDeviceGetAttribute(&h->num_sms, cudaDevAttrMultiProcessorCount, device);
  int cc_major = 0, cc_minor = 0;
  if (e == cudaSuccess) e = cudaDeviceGetAttribute(&cc_major, cudaDevAttrComputeCapabilityMajor, device);
  if (e == cudaSuccess) e = cudaDeviceGetAttribute(&cc_minor, cudaDevAttrComputeCapabilityMinor, device);
  if (e == cudaSuccess && !(cc_major == 10 && cc_minor == 0)) {
    delete h;
    return FM_EUNSUPPORTED;  // built for sm_100a only
  }
  if (e == cudaSuccess)
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&h->route_blocks_per_sm, fm::route_kernel, fm::kRouteThreads, 0);
  if (e == cudaSuccess)
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&h->route_sig_blocks_per_sm, fm::route_kernel_sigmoid,
                                                      fm::kRouteThreads, 0);
  if (e == cudaSuccess)
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&h->route_wide_blocks_per_sm, fm::route_kernel_wide,
                                                      fm::kRouteThreads, 0);
  if (e == cudaSuccess)
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&h->route_sig_wide_blocks_per_sm, fm::route_kernel_sigmoid_wide,
                                                      fm::kRouteThreads, 0);
  if (e == cudaSuccess) e = fm::qgemv_blocks_per_sm(&h->gemv_blocks_per_sm);
  if (e == cudaSuccess) e = fm::qgemv_tma_blocks_per_sm(&h->gemv_tma_blocks_per_sm);
  if (e == cudaSuccess) e = fm::tc::init();
  if (e == cudaSuccess) e = fm::tc::max_pairs(&h->tc_pairs);
  if (e == cudaSuccess && h->tc_pairs < 1) e = cudaErrorInvalidConfiguration;
  if (e != cudaSuccess) {
    cudaGetLastError();
    delete h;
    return FM_ECUDA;
  }
  h->gemv_blocks_per_sm = std::min(h->gemv_blocks_per_sm, 8);
  const int rc = ensure_ws(h, kCtrlBytes);
  if (rc != FM_OK) {
    delete h;
    return rc;
  }
  *out = h;
  return FM_OK;
}

int fm_destroy(fm_handle* h) {
  if (!h) return FM_EINVAL;
  cudaStreamSynchronize(h->stream);
  for (auto& p : h->pending) {
    cudaEventDestroy(p.a);
    cudaEventDestroy(p.b);
  }
  for (auto e : h->event_pool) cudaEventDestroy(e);
  p2p_close(h);
  if (h->ws) cudaFree(h->ws);
  if (h->ep_ws) cudaFree(h->ep_ws);
  delete h;
  return FM_OK;
}

int fm_set_stream(fm_handle* h, void* stream) {
  if (!h) return FM_EINVAL;
  h->stream = static_cast<cudaStream_t>(stream);
  return FM_OK;
}

const char* fm_last_error(const fm_handle* h) { return h ? h->last_error.c_str() : "null handle"; }

int fm_set_path(fm_handle* h, int path) {
  if (!h) return FM_EINVAL;
  if (path != FM_PATH_AUTO && path != FM_PATH_GEMV && path != FM_PATH_TCGEN05)
    return set_err(h, FM_EINVAL, "unknown path");
  h->path = path;
  return FM_OK;
}

int fm_last_path(const fm_handle* h) { return h ? h->last_path : 0; }

int fm_set_route_mode(fm_handle* h, int mode) {
  if (!h) return FM_EINVAL;
  if (mode != FM_ROUTE_AUTO && mode != FM_ROUTE_GRID && mode != FM_ROUTE_LAST_BLOCK && mode != FM_ROUTE_CLUSTER)
    return set_err(h, FM_EINVAL, "unknown route mode");
  h->route_mode = mode;
  return FM_OK;
}

size_t fm_workspace_bytes(const fm_handle* h) { return h ? h->ws_bytes : 0; }

int fm_profile_enable(fm_handle* h, int on) {
  if (!h) return FM_EINVAL;
  h->profile = on != 0;
  return FM_OK;
}

int fm_profile_report(fm_handle* h, fm_kernel_time* out, int capacity, int* count, int reset) {
  if (!h || (capacity > 0 && !out)) return FM_EINVAL;
  for (auto& p : h->pending) {
    float ms = 0.f;
    cudaError_t e = cudaEventSynchronize(p.b);
    if (e == cudaSuccess) e = cudaEventElapsedTime(&ms, p.a, p.b);
    if (e != cudaSuccess) return cuda_err(h, e, "kernel timing event");
    auto it = h->totals.find(p.name);
    if (it == h->totals.end()) it = h->totals.emplace(p.name, fm_handle::Total{p.name, 0, 0.0}).first;
    it->second.launches += 1;
    it->second.ms += ms;
    h->event_pool.push_back(p.a);
    h->event_pool.push_back(p.b);
  }
  h->pending.clear();
  // routing-kernel phase split (accumulated on the device since the last reset)
  unsigned long long ph[4] = {0, 0, 0, 0};
  if (h->ws) {
    cudaError_t e = cudaMemcpy(ph, phase_ns(h), sizeof(ph), cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) return cuda_err(h, e, "phase timer read");
    static const char* phase_names[4] = {"route.phase1_router", "route.phase2_topk", "route.phase3_scan",
                                         "route.phase4_scatter"};
    auto rt = h->totals.find("route");
    const int64_t nl = rt == h->totals.end() ? 0 : rt->second.launches;
    for (int i = 0; i < 4; ++i)
      if (ph[i]) h->totals[phase_names[i]] = fm_handle::Total{phase_names[i], nl, ph[i] * 1e-6};
  }
  int n = 0;
  for (auto& kv : h->totals) {
    if (n < capacity) {
      out[n].name = kv.second.name;
      out[n].launches = kv.second.launches;
      out[n].total_ms = kv.second.ms;
    }
    ++n;
  }
  if (count) *count = n;
  if (reset) {
    h->totals.clear();
    if (h->ws) cudaMemset(phase_ns(h), 0, 4 * sizeof(unsigned long long));
  }
  return FM_OK;
}

int fm_sync_status(fm_handle* h) {
  if (!h) return FM_EINVAL;
  cudaError_t e = cudaStreamSynchronize(h->stream);
  if (e != cudaSuccess) return cuda_err(h, e, "cudaStreamSynchronize");
  uint32_t word = 0;
  e = cudaMemcpy(&word, h->ws, sizeof(word), cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return cuda_err(h, e, "cudaMemcpy(error word)");
  if (word == 0) return FM_OK;
  cudaMemset(h->ws, 0, kCtrlBytes);  // clear the error word and the grid-sync counters
  if (word & fm::DEVERR_TIMEOUT) return set_err(h, FM_ETIMEOUT, "a bounded device-side wait ran out");
  if (word & fm::DEVERR_BOUNDS) return set_err(h, FM_EDEVICE, "an index failed its device-side bounds check");
  return set_err(h, FM_EDEVICE, "device-side check failed");
}

int fm_reserve(fm_handle* h, const fm_moe_config* c, int64_t max_tokens) {
  if (!h || !c || max_tokens < 0) return FM_EINVAL;
  return ensure_ws(h, reserve_need(c, max_tokens));
}

size_t fm_workspace_size(const fm_moe_config* c, int64_t max_tokens) {
  if (!c || max_tokens < 0 || c->hidden <= 0 || c->num_experts <= 0 || c->top_k <= 0 || c->inter <= 0 ||
      c->shared_inter < 0)
    return 0;
  return ws_alloc_bytes(reserve_need(c, max_tokens));
}

int fm_moe_block(fm_handle* h, const fm_moe_config* c, const fm_moe_weights* w, const uint16_t* x, int64_t T,
                 uint16_t* y, const fm_moe_outputs* outs) {
  if (!h) return FM_EINVAL;
  int rc = check_moe(h, c, w);
  if (rc) return rc;
  if (T < 0 || (T > 0 && (!x || !y))) return set_err(h, FM_EINVAL, "bad x / y / T");
  if (!aligned16(x) || !aligned16(y)) return set_err(h, FM_EINVAL, "x and y must be 16-byte aligned");
  if (T == 0) return FM_OK;
  if (T > (1LL << 24)) return set_err(h, FM_EUNSUPPORTED, "T too large");
  const int H = c->hidden, I = c->inter, E = c->num_experts, k = c->top_k;
  const bool shared = c->shared_inter > 0;
  const int epad = (E + 1 + 7) / 8 * 8;
  const int ksplit = router_ksplit(h, T, H, E);
  const int64_t P = T * k;
  const bool tcp = use_tc(h, P, E, c->group_size);
  h->last_path = tcp ? FM_PATH_TCGEN05 : FM_PATH_GEMV;
  // the GEMV path's TMA-fed kernel takes every fm_moe_block shape (K multiples of 128)
  const bool tvp = !tcp && h->gemv_tma_blocks_per_sm > 0 &&
                   fm::qgemv_tma_supports(fm::MODE_GATEUP, H, H, c->group_size) &&
                   fm::qgemv_tma_supports(fm::MODE_DOWN, I, shared ? c->shared_inter : I, c->group_size);
  Plan p = make_plan(T, T, H, E, k, epad, ksplit, I, c->shared_inter, shared, true, tcp);
  rc = ensure_ws(h, p.total);
  if (rc) return rc;

  RouteArgs ra;
  std::memset(&ra, 0, sizeof(ra));
  ra.x = x;
  ra.router_w = static_cast<const uint16_t*>(w->router_w);
  ra.shared_gate_w = shared ? static_cast<const uint16_t*>(w->shared_expert_gate_w) : nullptr;
  ra.router_bias = w->router_bias;
  ra.T = T;
  ra.H = H;
  ra.E = E;
  ra.k = k;
  ra.norm_topk = c->norm_topk_prob;
  ra.do_router = 1;
  ra.ksplit = ksplit;
  ra.epad = epad;
  ra.partial = at<float>(h, p.partial);
  ra.x_perm = at<uint16_t>(h, p.x_perm);
  ra.x_rows = T;
  // the GEMV path accumulates into fp32 combine buffers; the tcgen05 path stores
  // every output row once and needs no clearing
  ra.zero0 = tcp ? nullptr : at<float>(h, p.y_acc);
  ra.zero0_n = tcp ? 0 : T * H;
  ra.zero1 = (shared && !tcp) ? at<float>(h, p.ysh) : nullptr;
  ra.zero1_n = (shared && !tcp) ? T * H : 0;
  ra.topk_ids = at<int32_t>(h, p.topk_ids);
  ra.topk_score = at<float>(h, p.topk_score);
  ra.gate_sig = at<float>(h, p.gate_sig);
  ra.row_src = at<int32_t>(h, p.row_src);
  ra.chunk_counts = at<int32_t>(h, p.chunk_counts);
  ra.pair_rank = at<int32_t>(h, p.pair_rank);
  ra.totals = at<int32_t>(h, p.totals);
  ra.offsets = at<int32_t>(h, p.offsets);
  ra.sorted_token = at<int32_t>(h, p.sorted_token);
  ra.sorted_score = at<float>(h, p.sorted_score);
  ra.sorted_flat = at<int32_t>(h, p.sorted_flat);
  ra.pair_pos = tcp ? at<int32_t>(h, p.pair_pos) : nullptr;
  ra.tab_a = at<TileTable>(h, p.tab_a);
  ra.tab_b = at<TileTable>(h, p.tab_b);
  ra.a_rows_per_block = tcp ? 128 : 64;
  ra.a_n = I;
  ra.a_n_shared = c->shared_inter;
  ra.b_n = H;
  ra.b_rows_per_block = tcp ? 256 : 128;
  // GEMV: one 8-row MMA column tile per unit (qgemv.cu), or four (qgemv_tma.cu)
  ra.chunk_max = tcp ? fm::tc::max_rows() : (tvp ? fm::qgemv_tma_max_rows() : 8);
  ra.chunk_align = tcp ? 16 : 8;
  ra.b_ksplit_shared = tcp ? 1 : std::max(1, c->shared_inter / std::max(1, I));
  ra.has_shared = shared ? 1 : 0;
  if (outs) {
    ra.out_topk_ids = outs->topk_ids;
    ra.out_topk_scores = outs->topk_scores;
    ra.out_sorted_token = outs->sorted_token;
    ra.out_offsets = outs->expert_offsets;
  }
  ra.gsync = grid_sync(h);
  ra.err = err_word(h);
  ra.phase_ns = phase_ns(h);
  const int64_t items = ((T + 15) / 16) * ksplit;
  rc = launch_route(h, ra, items);
  if (rc) return rc;

  GemmArgs ga;
  std::memset(&ga, 0, sizeof(ga));
  ga.gs = c->group_size;
  ga.err = err_word(h);
  ga.sorted_token = ra.sorted_token;
  ga.sorted_score = ra.sorted_score;
  ga.sorted_flat = ra.sorted_flat;
  // gate / up
  ga.K = H;
  ga.K_shared = H;
  ga.N = I;
  ga.N_shared = c->shared_inter;
  ga.w0 = w->gate.w; ga.s0 = w->gate.scales; ga.b0 = w->gate.biases;
  ga.w1 = w->up.w; ga.s1 = w->up.scales; ga.b1 = w->up.biases;
  if (shared) {
    ga.sw0 = w->shared_gate.w; ga.ss0 = w->shared_gate.scales; ga.sb0 = w->shared_gate.biases;
    ga.sw1 = w->shared_up.w; ga.ss1 = w->shared_up.scales; ga.sb1 = w->shared_up.biases;
  }
  ga.act = ra.x_perm;
  ga.act_shared = ra.x_perm;
  ga.act_ld = H;
  ga.act_shared_ld = H;
  ga.out = at<uint16_t>(h, p.a_sorted);
  ga.out_ld = I;
  ga.out_shared = shared ? at<uint16_t>(h, p.a_shared) : nullptr;
  ga.out_shared_ld = c->shared_inter;
  ga.tab = ra.tab_a;
  fm::TcMaps maps_gu, maps_dn;
  if (tcp || tvp) {
    const int Is = c->shared_inter;
    bool ok = encode_codes(&maps_gu.code[0], w->gate.w, static_cast<int64_t>(E) * I, H, 64) &&
              encode_codes(&maps_gu.code[1], w->up.w, static_cast<int64_t>(E) * I, H, 64) &&
              encode_codes(&maps_gu.code[2], shared ? w->shared_gate.w : nullptr, Is, H, 64) &&
              encode_codes(&maps_gu.code[3], shared ? w->shared_up.w : nullptr, Is, H, 64) &&
              encode_act(&maps_gu.act[0], ra.x_perm, T, H) &&
              encode_act(&maps_gu.act[1], shared ? ra.x_perm : nullptr, T, H) &&
              encode_codes(&maps_dn.code[0], w->down.w, static_cast<int64_t>(E) * H, I, 128) &&
              encode_codes(&maps_dn.code[1], nullptr, 0, I, 128) &&
              encode_codes(&maps_dn.code[2], shared ? w->shared_down.w : nullptr, H, shared ? Is : I, 128) &&
              encode_codes(&maps_dn.code[3], nullptr, 0, I, 128) &&
              encode_act(&maps_dn.act[0], at<uint16_t>(h, p.a_sorted), P, I) &&
              encode_act(&maps_dn.act[1], shared ? at<uint16_t>(h, p.a_shared) : nullptr, T, Is);
    if (!ok) return set_err(h, FM_ECUDA, "cuTensorMapEncodeTiled failed (alignment or driver entry point)");
  }
  rc = launch_gemm<fm::MODE_GATEUP>(h, ga, tcp, &maps_gu, tvp);
  if (rc) return rc;
  // down (+ combine)
  GemmArgs gd = ga;
  gd.K = I;
  gd.K_shared = c->shared_inter;
  gd.N = H;
  gd.N_shared = H;
  gd.w0 = w->down.w; gd.s0 = w->down.scales; gd.b0 = w->down.biases;
  gd.w1 = nullptr; gd.s1 = nullptr; gd.b1 = nullptr;
  if (shared) {
    gd.sw0 = w->shared_down.w; gd.ss0 = w->shared_down.scales; gd.sb0 = w->shared_down.biases;
  }
  gd.sw1 = nullptr; gd.ss1 = nullptr; gd.sb1 = nullptr;
  gd.act = ga.out;
  gd.act_ld = I;
  gd.act_shared = ga.out_shared;
  gd.act_shared_ld = c->shared_inter;
  gd.out = nullptr;
  gd.out_shared = nullptr;
  gd.y_acc = tcp ? nullptr : at<float>(h, p.y_acc);
  gd.ysh = (shared && !tcp) ? at<float>(h, p.ysh) : nullptr;
  gd.y_pairs = tcp ? at<uint16_t>(h, p.y_pairs) : nullptr;
  gd.ysh16 = (shared && tcp) ? at<uint16_t>(h, p.ysh16) : nullptr;
  gd.y_ld = H;
  gd.tab = ra.tab_b;
  rc = launch_gemm<fm::MODE_DOWN>(h, gd, tcp, &maps_dn, tvp);
  if (rc) return rc;
  // finalize: combine rounding + gated shared expert
  prof_begin(h, "finalize");
  if (tcp) {
    const int64_t n8 = T * H / 8;
    const int fb = static_cast<int>(std::min<int64_t>((n8 + 255) / 256, static_cast<int64_t>(h->num_sms) * 8));
    fm::launch_finalize_pairs(fb, h->stream, gd.y_pairs, ra.pair_pos, k, gd.ysh16, ra.gate_sig, T, H, y);
  } else {
    const int64_t n4 = T * H / 4;
    const int fb = static_cast<int>(std::min<int64_t>((n4 + 255) / 256, static_cast<int64_t>(h->num_sms) * 8));
    fm::finalize_kernel<<<fb, 256, 0, h->stream>>>(gd.y_acc, gd.ysh, ra.gate_sig, T, H, y);
  }
  prof_end(h);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_err(h, e, "finalize launch");
  return FM_OK;
}

// The Nemotron-H / DeepSeek-style block and other variants (fm_moe_variant): the same
// routing / sort / tile-plan kernel with sigmoid scoring when asked, then the GEMV expert
// kernels (relu^2 fc1 or SwiGLU gate/up, then down with fp32 or bf16 score products) and
// the fixed combine with the shared expert gated or not.
int fm_moe_block_variant(fm_handle* h, const fm_moe_config* c, const fm_moe_variant* v, const fm_moe_weights* w,
                         const uint16_t* x, int64_t T, uint16_t* y, const fm_moe_outputs* outs) {
  if (!h) return FM_EINVAL;
  if (!v) return fm_moe_block(h, c, w, x, T, y, outs);
  if (v->score_func != FM_SCORE_SOFTMAX && v->score_func != FM_SCORE_SIGMOID)
    return set_err(h, FM_EINVAL, "score_func must be FM_SCORE_SOFTMAX or FM_SCORE_SIGMOID");
  if (v->expert_act != FM_ACT_SWIGLU && v->expert_act != FM_ACT_RELU2)
    return set_err(h, FM_EINVAL, "expert_act must be FM_ACT_SWIGLU or FM_ACT_RELU2");
  const bool sig = v->score_func == FM_SCORE_SIGMOID, relu2 = v->expert_act == FM_ACT_RELU2;
  const bool ungated = v->shared_ungated != 0;
  if (!sig && !relu2 && !ungated) return fm_moe_block(h, c, w, x, T, y, outs);
  if (!c || !w) return set_err(h, FM_EINVAL, "null config or weights");
  const int H = c->hidden, I = c->inter, E = c->num_experts, k = c->top_k, Is = c->shared_inter;
  if (H <= 0 || I <= 0 || E <= 0 || k <= 0 || k > E || Is < 0) return set_err(h, FM_EINVAL, "bad MoE dimensions");
  if (E > fm::kMaxExperts || k > 16) return set_err(h, FM_EUNSUPPORTED, "num_experts > 512 or top_k > 16");
  // the GEMV expert path reads K in 128-wide chunks plus at most one 64-wide half
  // (group size 64), so the expert widths (the down matrices' K) need only be multiples of 64
  if (H % 128 || I % 64 || Is % 64)
    return set_err(h, FM_EUNSUPPORTED, "hidden must be a multiple of 128, the intermediate sizes of 64");
  if (!quant_ok(H, c->group_size, c->bits) || !quant_ok(I, c->group_size, c->bits) ||
      (Is > 0 && !quant_ok(Is, c->group_size, c->bits)) || (c->group_size != 64 && c->group_size != 128))
    return set_err(h, FM_EUNSUPPORTED, "variants run 4-bit affine weights with group size 64 or 128");
  if (c->router_quantized || (Is > 0 && !ungated && c->shared_gate_quantized))
    return set_err(h, FM_EUNSUPPORTED, "quantized router / shared-expert gate not implemented");
  const int n_group = v->n_group > 0 ? v->n_group : 1;
  if (sig && (n_group > 32 || E % n_group || (n_group > 1 && E / n_group < 2) || v->topk_group < 0 ||
              v->topk_group > n_group || (n_group > 1 && v->topk_group < 1)))
    return set_err(h, FM_EINVAL, "n_group must divide E (groups of >= 2, at most 32), 1 <= topk_group <= n_group");
  if (sig && w && w->router_bias)
    return set_err(h, FM_EINVAL, "router_bias applies to softmax routing; sigmoid routing takes correction_bias");
  const fm_qweight& e1 = relu2 ? w->up : w->gate;
  if (!w->router_w || !e1.w || !e1.scales || !w->down.w || !w->down.scales || (!relu2 && (!w->up.w || !w->up.scales)))
    return set_err(h, FM_EINVAL, "expert weights missing");
  if (Is > 0) {
    if (!w->shared_up.w || !w->shared_up.scales || !w->shared_down.w || !w->shared_down.scales ||
        (!relu2 && (!w->shared_gate.w || !w->shared_gate.scales)) || (!ungated && !w->shared_expert_gate_w))
      return set_err(h, FM_EINVAL, "shared expert weights missing");
  }
  if (T < 0 || (T > 0 && (!x || !y))) return set_err(h, FM_EINVAL, "bad x / y / T");
  if (!aligned16(x) || !aligned16(y)) return set_err(h, FM_EINVAL, "x and y must be 16-byte aligned");
  // A down K (I or Is) of 128 n + 64 runs the GEMV's half-chunk instance, which stages a
  // work unit's scales / biases in shared memory by aligned 4-byte copies: at most 62
  // groups per row and unit, 4-byte aligned scale / bias arrays
  const int ksplit_sh = std::max(1, Is / std::max(1, I));
  if ((I % 128) || (Is % 128)) {
    auto a4 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 3) == 0; };
    const int unit_sh = ((Is + 127) / 128 + ksplit_sh - 1) / ksplit_sh;  // 128-wide chunks per shared unit
    if (I / 64 > 62 || 2 * unit_sh > 62)
      return set_err(h, FM_EUNSUPPORTED, "expert widths of 128 n + 64 are implemented up to 3968");
    if (!a4(w->down.scales) || !a4(w->down.biases) || (Is > 0 && (!a4(w->shared_down.scales) || !a4(w->shared_down.biases))))
      return set_err(h, FM_EINVAL, "down scales / biases must be 4-byte aligned");
  }
  if (T == 0) return FM_OK;
  if (T > (1LL << 24)) return set_err(h, FM_EUNSUPPORTED, "T too large");
  const bool shared = Is > 0;
  const int epad = (E + 1 + 7) / 8 * 8;
  const int ksplit = router_ksplit(h, T, H, E);
  // The tcgen05 expert path (relu^2 epilogue, bf16(d) per pair, combine with the scores
  // in fp32 for sigmoid routing) runs when the handle's path is FM_PATH_TCGEN05; the
  // automatic choice keeps the GEMV path for the variants.
  const bool tcp = h->path == FM_PATH_TCGEN05 && I % 128 == 0 && Is % 128 == 0;
  h->last_path = tcp ? FM_PATH_TCGEN05 : FM_PATH_GEMV;
  const int64_t P = T * k;
  Plan p = make_plan(T, T, H, E, k, epad, ksplit, I, Is, shared, true, tcp);
  int rc = ensure_ws(h, p.total);
  if (rc) return rc;

  RouteArgs ra;
  std::memset(&ra, 0, sizeof(ra));
  ra.x = x;
  ra.router_w = static_cast<const uint16_t*>(w->router_w);
  ra.shared_gate_w = (shared && !ungated) ? static_cast<const uint16_t*>(w->shared_expert_gate_w) : nullptr;
  ra.router_bias = w->router_bias;
  ra.T = T;
  ra.H = H;
  ra.E = E;
  ra.k = k;
  ra.norm_topk = c->norm_topk_prob;
  ra.do_router = 1;
  ra.ksplit = ksplit;
  ra.epad = epad;
  ra.partial = at<float>(h, p.partial);
  ra.x_perm = at<uint16_t>(h, p.x_perm);
  ra.x_rows = T;
  ra.zero0 = tcp ? nullptr : at<float>(h, p.y_acc);
  ra.zero0_n = tcp ? 0 : T * H;
  ra.zero1 = (shared && !tcp) ? at<float>(h, p.ysh) : nullptr;
  ra.zero1_n = (shared && !tcp) ? T * H : 0;
  ra.pair_pos = tcp ? at<int32_t>(h, p.pair_pos) : nullptr;
  ra.topk_ids = at<int32_t>(h, p.topk_ids);
  ra.topk_score = at<float>(h, p.topk_score);
  ra.gate_sig = at<float>(h, p.gate_sig);
  ra.row_src = at<int32_t>(h, p.row_src);
  ra.chunk_counts = at<int32_t>(h, p.chunk_counts);
  ra.pair_rank = at<int32_t>(h, p.pair_rank);
  ra.totals = at<int32_t>(h, p.totals);
  ra.offsets = at<int32_t>(h, p.offsets);
  ra.sorted_token = at<int32_t>(h, p.sorted_token);
  ra.sorted_score = at<float>(h, p.sorted_score);
  ra.sorted_flat = at<int32_t>(h, p.sorted_flat);
  ra.tab_a = at<TileTable>(h, p.tab_a);
  ra.tab_b = at<TileTable>(h, p.tab_b);
  // GEMV: relu^2 is one matrix of 4 warps x 32 rows, gate/up 64 rows of each; tcgen05:
  // 256 rows of one matrix per CTA pair, or 128 of gate and up each
  ra.a_rows_per_block = tcp ? (relu2 ? 256 : 128) : (relu2 ? 128 : 64);
  ra.a_n = I;
  ra.a_n_shared = Is;
  ra.b_n = H;
  ra.b_rows_per_block = tcp ? 256 : 128;
  ra.chunk_max = tcp ? fm::tc::max_rows() : 8;
  ra.chunk_align = tcp ? 16 : 8;
  ra.b_ksplit_shared = tcp ? 1 : ksplit_sh;
  ra.has_shared = shared ? 1 : 0;
  if (outs) {
    ra.out_topk_ids = outs->topk_ids;
    ra.out_topk_scores = outs->topk_scores;
    ra.out_sorted_token = outs->sorted_token;
    ra.out_offsets = outs->expert_offsets;
  }
  ra.n_group = n_group;
  ra.topk_group = v->topk_group > 0 ? v->topk_group : n_group;
  ra.routed_scale = (sig && v->routed_scaling_factor != 0.f) ? v->routed_scaling_factor : 1.f;
  ra.corr_bias = sig ? v->correction_bias : nullptr;
  ra.out_scores_f32 = v->topk_scores_f32;
  ra.shared_ungated = (shared && ungated) ? 1 : 0;
  ra.gsync = grid_sync(h);
  ra.err = err_word(h);
  ra.phase_ns = phase_ns(h);
  rc = launch_route(h, ra, ((T + 15) / 16) * ksplit, sig);
  if (rc) return rc;

  GemmArgs ga;
  std::memset(&ga, 0, sizeof(ga));
  ga.gs = c->group_size;
  ga.err = err_word(h);
  ga.sorted_token = ra.sorted_token;
  ga.sorted_score = ra.sorted_score;
  ga.sorted_flat = ra.sorted_flat;
  ga.K = H;
  ga.K_shared = H;
  ga.N = I;
  ga.N_shared = Is;
  if (relu2) {  // fc1 = up; shared: up only
    ga.w0 = w->up.w; ga.s0 = w->up.scales; ga.b0 = w->up.biases;
    if (shared) {
      ga.sw0 = w->shared_up.w; ga.ss0 = w->shared_up.scales; ga.sb0 = w->shared_up.biases;
    }
  } else {
    ga.w0 = w->gate.w; ga.s0 = w->gate.scales; ga.b0 = w->gate.biases;
    ga.w1 = w->up.w; ga.s1 = w->up.scales; ga.b1 = w->up.biases;
    if (shared) {
      ga.sw0 = w->shared_gate.w; ga.ss0 = w->shared_gate.scales; ga.sb0 = w->shared_gate.biases;
      ga.sw1 = w->shared_up.w; ga.ss1 = w->shared_up.scales; ga.sb1 = w->shared_up.biases;
    }
  }
  ga.act = ra.x_perm;
  ga.act_shared = ra.x_perm;
  ga.act_ld = H;
  ga.act_shared_ld = H;
  ga.out = at<uint16_t>(h, p.a_sorted);
  ga.out_ld = I;
  ga.out_shared = shared ? at<uint16_t>(h, p.a_shared) : nullptr;
  ga.out_shared_ld = Is;
  ga.tab = ra.tab_a;
  fm::TcMaps maps_a, maps_dn;
  if (tcp) {
    // relu^2: one 128-row code box of fc1 per CTA; gate/up: 64 rows of each
    const int box = relu2 ? 128 : 64;
    bool ok = encode_codes(&maps_a.code[0], relu2 ? w->up.w : w->gate.w, static_cast<int64_t>(E) * I, H, box) &&
              encode_codes(&maps_a.code[1], relu2 ? nullptr : w->up.w, relu2 ? 0 : static_cast<int64_t>(E) * I, H, box) &&
              encode_codes(&maps_a.code[2], shared ? (relu2 ? w->shared_up.w : w->shared_gate.w) : nullptr, Is, H, box) &&
              encode_codes(&maps_a.code[3], (shared && !relu2) ? w->shared_up.w : nullptr, Is, H, box) &&
              encode_act(&maps_a.act[0], ra.x_perm, T, H) &&
              encode_act(&maps_a.act[1], shared ? ra.x_perm : nullptr, T, H) &&
              encode_codes(&maps_dn.code[0], w->down.w, static_cast<int64_t>(E) * H, I, 128) &&
              encode_codes(&maps_dn.code[1], nullptr, 0, I, 128) &&
              encode_codes(&maps_dn.code[2], shared ? w->shared_down.w : nullptr, H, shared ? Is : I, 128) &&
              encode_codes(&maps_dn.code[3], nullptr, 0, I, 128) &&
              encode_act(&maps_dn.act[0], at<uint16_t>(h, p.a_sorted), P, I) &&
              encode_act(&maps_dn.act[1], shared ? at<uint16_t>(h, p.a_shared) : nullptr, T, Is);
    if (!ok) return set_err(h, FM_ECUDA, "cuTensorMapEncodeTiled failed (alignment or driver entry point)");
  }
  rc = relu2 ? launch_gemm<fm::MODE_RELU2>(h, ga, tcp, &maps_a) : launch_gemm<fm::MODE_GATEUP>(h, ga, tcp, &maps_a);
  if (rc) return rc;
  GemmArgs gd = ga;
  gd.K = I;
  gd.K_shared = Is;
  gd.N = H;
  gd.N_shared = H;
  gd.w0 = w->down.w; gd.s0 = w->down.scales; gd.b0 = w->down.biases;
  gd.w1 = nullptr; gd.s1 = nullptr; gd.b1 = nullptr;
  gd.sw0 = shared ? w->shared_down.w : nullptr;
  gd.ss0 = shared ? w->shared_down.scales : nullptr;
  gd.sb0 = shared ? w->shared_down.biases : nullptr;
  gd.sw1 = nullptr; gd.ss1 = nullptr; gd.sb1 = nullptr;
  gd.act = ga.out;
  gd.act_ld = I;
  gd.act_shared = ga.out_shared;
  gd.act_shared_ld = Is;
  gd.out = nullptr;
  gd.out_shared = nullptr;
  gd.y_acc = tcp ? nullptr : at<float>(h, p.y_acc);
  gd.ysh = (shared && !tcp) ? at<float>(h, p.ysh) : nullptr;
  gd.y_pairs = tcp ? at<uint16_t>(h, p.y_pairs) : nullptr;
  gd.ysh16 = (shared && tcp) ? at<uint16_t>(h, p.ysh16) : nullptr;
  gd.unit_score = (tcp && sig) ? 1 : 0;  // tcgen05 + sigmoid scores: bf16(d) per pair, scaled in the combine
  gd.y_ld = H;
  gd.tab = ra.tab_b;
  if (tcp)
    rc = launch_gemm<fm::MODE_DOWN>(h, gd, true, &maps_dn);
  else
    rc = sig ? launch_gemm<fm::MODE_DOWN_F32>(h, gd, false) : launch_gemm<fm::MODE_DOWN>(h, gd, false);
  if (rc) return rc;
  prof_begin(h, "finalize");
  if (tcp) {
    const int64_t n8 = T * H / 8;
    const int fb = static_cast<int>(std::min<int64_t>((n8 + 255) / 256, static_cast<int64_t>(h->num_sms) * 8));
    if (sig)
      fm::finalize_pairs_f32_kernel<<<fb, 256, 0, h->stream>>>(gd.y_pairs, ra.pair_pos, ra.topk_score, k, gd.ysh16,
                                                               ra.gate_sig, T, H, y);
    else
      fm::launch_finalize_pairs(fb, h->stream, gd.y_pairs, ra.pair_pos, k, gd.ysh16, ra.gate_sig, T, H, y);
  } else {
    const int64_t n4 = T * H / 4;
    const int fb = static_cast<int>(std::min<int64_t>((n4 + 255) / 256, static_cast<int64_t>(h->num_sms) * 8));
    fm::finalize_kernel<<<fb, 256, 0, h->stream>>>(gd.y_acc, gd.ysh, ra.gate_sig, T, H, y);
  }
  prof_end(h);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_err(h, e, "finalize launch");
  return FM_OK;
}

}  // extern "C"

namespace {

// gather_qmm / quantized_matmul.  direct: one matrix, rows in order (fm_linear) -- the
// row layout and tile table come from dense_prep_kernel instead of the routing kernel.
int gather_qmm_impl(fm_handle* h, const uint16_t* x, int64_t x_batches, int M, int K, const uint32_t* w,
                    const uint16_t* scales, const uint16_t* biases, int E, int N, const uint32_t* lhs_indices,
                    const uint32_t* rhs_indices, int64_t B, int transpose, int group_size, int bits, uint16_t* out,
                    bool direct) {
  if (!h) return FM_EINVAL;
  if (!transpose) return set_err(h, FM_EUNSUPPORTED, "transpose=false is not implemented");
  if (!quant_ok(K, group_size, bits)) return set_err(h, FM_EUNSUPPORTED, "only 4-bit affine, group 32/64/128");
  if (x_batches <= 0 || M <= 0 || E <= 0 || N <= 0 || B < 0) return set_err(h, FM_EINVAL, "bad sizes");
  if (E > fm::kMaxExperts) return set_err(h, FM_EUNSUPPORTED, "more than 512 experts");
  if (!lhs_indices && B % x_batches != 0) return set_err(h, FM_EINVAL, "x batch does not broadcast against rhs");
  if (B == 0) return FM_OK;
  if (!x || !w || !scales || !out || (!rhs_indices && E != 1)) return set_err(h, FM_EINVAL, "null pointer");
  if (!aligned16(x) || !aligned16(out)) return set_err(h, FM_EINVAL, "x and out must be 16-byte aligned");
  if (K % 64 || N % 16) return set_err(h, FM_EUNSUPPORTED, "K must be a multiple of 64 and N of 16");
  const int64_t rows = B * M;
  if (rows > (1LL << 24)) return set_err(h, FM_EUNSUPPORTED, "too many rows");
  bool tcp = use_tc(h, rows, E, group_size);
  if (K % 128) tcp = true;  // the GEMV path works in 128-wide K chunks
  h->last_path = tcp ? FM_PATH_TCGEN05 : FM_PATH_GEMV;
  const bool tvp = !tcp && h->gemv_tma_blocks_per_sm > 0 && fm::qgemv_tma_supports(fm::MODE_PLAIN, K, K, group_size);
  Plan p = make_plan(rows, x_batches * M, K, E, 1, 8, 1, 0, 0, false, false, tcp);
  int rc = ensure_ws(h, p.total);
  if (rc) return rc;

  RouteArgs ra;
  std::memset(&ra, 0, sizeof(ra));
  ra.x = x;
  ra.T = rows;
  ra.H = K;
  ra.E = E;
  ra.k = 1;
  ra.do_router = 0;
  ra.ksplit = 1;
  ra.epad = 8;
  ra.given_ids = rhs_indices;
  ra.given_lhs = lhs_indices;
  ra.x_batches = x_batches;
  ra.batches = B;
  ra.M = M;
  ra.x_perm = at<uint16_t>(h, p.x_perm);
  ra.x_rows = x_batches * M;
  ra.topk_ids = at<int32_t>(h, p.topk_ids);
  ra.topk_score = at<float>(h, p.topk_score);
  ra.gate_sig = at<float>(h, p.gate_sig);
  ra.row_src = at<int32_t>(h, p.row_src);
  ra.chunk_counts = at<int32_t>(h, p.chunk_counts);
  ra.pair_rank = at<int32_t>(h, p.pair_rank);
  ra.totals = at<int32_t>(h, p.totals);
  ra.offsets = at<int32_t>(h, p.offsets);
  ra.sorted_token = at<int32_t>(h, p.sorted_token);
  ra.sorted_score = at<float>(h, p.sorted_score);
  ra.sorted_flat = at<int32_t>(h, p.sorted_flat);
  ra.tab_a = at<TileTable>(h, p.tab_a);
  ra.tab_b = nullptr;
  ra.a_rows_per_block = tcp ? 256 : 128;
  ra.a_n = N;
  ra.a_n_shared = 0;
  ra.chunk_max = tcp ? fm::tc::max_rows() : (tvp ? fm::qgemv_tma_max_rows() : 8);
  ra.chunk_align = tcp ? 16 : 8;
  ra.b_ksplit_shared = 1;
  ra.gsync = grid_sync(h);
  ra.err = err_word(h);
  if (direct) {
    const int64_t n = ra.x_rows * (K / 8);
    const int grid = static_cast<int>(std::max<int64_t>(
        1, std::min<int64_t>((std::max<int64_t>(n, rows) + 255) / 256, static_cast<int64_t>(h->num_sms) * 8)));
    prof_begin(h, "dense_prep");
    fm::dense_prep_kernel<<<grid, 256, 0, h->stream>>>(ra);
    prof_end(h);
    const cudaError_t le = cudaGetLastError();
    if (le != cudaSuccess) return cuda_err(h, le, "dense_prep launch");
  } else {
    const int64_t items = (ra.x_rows * (K / 8) + 255) / 256 * 8;
    rc = launch_route(h, ra, items);
    if (rc) return rc;
  }

  GemmArgs ga;
  std::memset(&ga, 0, sizeof(ga));
  ga.K = K;
  ga.K_shared = K;
  ga.N = N;
  ga.N_shared = N;
  ga.gs = group_size;
  ga.w0 = w; ga.s0 = scales; ga.b0 = biases;
  ga.act = ra.x_perm;
  ga.act_ld = K;
  ga.sorted_token = ra.sorted_token;
  ga.sorted_score = ra.sorted_score;
  ga.sorted_flat = ra.sorted_flat;
  ga.out = out;
  ga.out_ld = N;
  ga.tab = ra.tab_a;
  ga.err = err_word(h);
  fm::TcMaps maps;
  if (tcp || tvp) {
    const bool ok = encode_codes(&maps.code[0], w, static_cast<int64_t>(E) * N, K, 128) &&
                    encode_codes(&maps.code[1], nullptr, 0, K, 128) && encode_codes(&maps.code[2], nullptr, 0, K, 128) &&
                    encode_codes(&maps.code[3], nullptr, 0, K, 128) &&
                    encode_act(&maps.act[0], ra.x_perm, ra.x_rows, K) &&
                    encode_act(&maps.act[1], nullptr, 0, K);
    if (!ok) return set_err(h, FM_ECUDA, "cuTensorMapEncodeTiled failed (alignment or driver entry point)");
  }
  return launch_gemm<fm::MODE_PLAIN>(h, ga, tcp, &maps, tvp);
}

}  // namespace

extern "C" {

int fm_gather_qmm(fm_handle* h, const uint16_t* x, int64_t x_batches, int M, int K, const uint32_t* w,
                  const uint16_t* scales, const uint16_t* biases, int E, int N, const uint32_t* lhs_indices,
                  const uint32_t* rhs_indices, int64_t B, int transpose, int group_size, int bits,
                  int sorted_indices, uint16_t* out) {
  (void)sorted_indices;  // a hint in MLX; the expert-major order is rebuilt either way
  return gather_qmm_impl(h, x, x_batches, M, K, w, scales, biases, E, N, lhs_indices, rhs_indices, B, transpose,
                         group_size, bits, out, false);
}

int fm_linear(fm_handle* h, const uint16_t* x, int64_t M, int K, const uint32_t* w, const uint16_t* scales,
              const uint16_t* biases, int N, int group_size, int bits, uint16_t* out) {
  if (!h) return FM_EINVAL;
  if (M < 0) return set_err(h, FM_EINVAL, "negative M");
  if (M == 0) return FM_OK;
  if (M > (1LL << 24)) return set_err(h, FM_EUNSUPPORTED, "too many rows");
  return gather_qmm_impl(h, x, 1, static_cast<int>(M), K, w, scales, biases, 1, N, nullptr, nullptr, 1, 1,
                         group_size, bits, out, true);
}


// ---------------------------------------------------------------- expert parallelism
int fm_ep_range(int num_experts, int rank, int world, int* first, int* count) {
  if (num_experts <= 0 || world <= 0 || rank < 0 || rank >= world || !first || !count) return FM_EINVAL;
  ep_range(num_experts, rank, world, first, count);
  return FM_OK;
}

int fm_ep_set(fm_handle* h, int rank, int world) {
  if (!h) return FM_EINVAL;
  if (world <= 0 || rank < 0 || rank >= world) return set_err(h, FM_EINVAL, "bad expert-parallel rank / world");
  h->ep_rank = rank;
  h->ep_world = world;
  h->ep_T = -1;
  h->ep_stage = 0;
  return FM_OK;
}

int fm_ep_dispatch(fm_handle* h, const fm_moe_config* c, const fm_moe_weights* w, const uint16_t* x, int64_t T,
                   int32_t* expert_counts, const uint16_t** send_rows) {
  if (!h) return FM_EINVAL;
  if (!expert_counts || !send_rows) return set_err(h, FM_EINVAL, "null argument");
  int rc = check_ep_route(h, c, w, x, T);
  if (rc) return rc;
  const int H = c->hidden, E = c->num_experts, k = c->top_k;
  const int epad = (E + 1 + 7) / 8 * 8;
  const int ksplit = router_ksplit(h, std::max<int64_t>(T, 1), H, E);
  const int64_t P = T * k;
  const EpPlan1 p = make_ep_plan1(T, H, E, k, epad, ksplit);
  rc = ensure_ws(h, p.total);
  if (rc) return rc;
  *send_rows = at<uint16_t>(h, p.send);
  h->ep_T = T;
  h->ep_stage = 1;
  if (T == 0) {
    std::memset(expert_counts, 0, sizeof(int32_t) * E);
    return FM_OK;
  }
  RouteArgs ra = ep_route_args(h, c, w, x, T, ksplit, p);
  rc = launch_route(h, ra, ((T + 15) / 16) * ksplit);
  if (rc) return rc;
  prof_begin(h, "ep_gather");
  fm::ep_gather_kernel<<<grid_for(h, P * (H / 8)), 256, 0, h->stream>>>(ra.x_perm, ra.sorted_token, P, H,
                                                                        at<uint16_t>(h, p.send));
  prof_end(h);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_err(h, e, "ep_gather launch");
  std::vector<int32_t> off(static_cast<size_t>(E) + 1);
  e = cudaMemcpyAsync(off.data(), ra.offsets, sizeof(int32_t) * (E + 1), cudaMemcpyDeviceToHost, h->stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(h->stream);
  if (e != cudaSuccess) return cuda_err(h, e, "expert counts");
  uint32_t dev_err = 0;
  e = cudaMemcpy(&dev_err, h->ws, sizeof(dev_err), cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return cuda_err(h, e, "device error word");
  if (dev_err) return set_err(h, FM_EDEVICE, "device-side check failed in routing");
  for (int i = 0; i < E; ++i) expert_counts[i] = off[i + 1] - off[i];
  return FM_OK;
}

int fm_ep_experts(fm_handle* h, const fm_moe_config* c, const fm_moe_weights* w, const uint16_t* recv_rows,
                  const int32_t* recv_counts, uint16_t* d_rows) {
  if (!h) return FM_EINVAL;
  if (h->ep_stage != 1) return set_err(h, FM_EINVAL, "fm_ep_experts must follow fm_ep_dispatch");
  if (!c || !w || !recv_counts) return set_err(h, FM_EINVAL, "null argument");
  int first = 0, E_local = 0;
  ep_range(c->num_experts, h->ep_rank, h->ep_world, &first, &E_local);
  const int nseg = h->ep_world * E_local;
  if (nseg + 1 > fm::kMaxGroups) return set_err(h, FM_EUNSUPPORTED, "too many (rank, expert) segments");
  int64_t R = 0;
  for (int i = 0; i < nseg; ++i) {
    if (recv_counts[i] < 0) return set_err(h, FM_EINVAL, "negative receive count");
    R += recv_counts[i];
  }
  if (R > 0 && (!recv_rows || !d_rows)) return set_err(h, FM_EINVAL, "null receive / result rows");
  if (!aligned16(recv_rows) || !aligned16(d_rows)) return set_err(h, FM_EINVAL, "rows must be 16-byte aligned");
  const int64_t T = h->ep_T;
  const int H = c->hidden, I = c->inter, E = c->num_experts, k = c->top_k, Is = c->shared_inter;
  const bool shared = Is > 0 && T > 0;
  int rc = check_ep_experts(h, c, w, R > 0, shared);
  if (rc) return rc;
  const bool tcp = use_tc(h, R + (shared ? T : 0), E_local + (shared ? 1 : 0), c->group_size);
  h->last_path = tcp ? FM_PATH_TCGEN05 : FM_PATH_GEMV;
  const EpPlan2 p2 = make_ep_plan2(R, std::max<int64_t>(T, 0), H, I, Is, nseg, shared);
  rc = ensure_ep_ws(h, p2.total);
  if (rc) return rc;
  const EpPlan1 p1 = make_ep_plan1(std::max<int64_t>(T, 0), H, E, k, (E + 1 + 7) / 8 * 8,
                                   router_ksplit(h, std::max<int64_t>(T, 1), H, E));
  h->ep_ysh_bf16 = tcp;
  h->ep_shared = shared;
  h->ep_R = R;
  h->ep_stage = 2;
  cudaError_t e = cudaMemcpyAsync(ep_at<int32_t>(h, p2.recv_counts), recv_counts, sizeof(int32_t) * nseg,
                                  cudaMemcpyHostToDevice, h->stream);
  if (e != cudaSuccess) return cuda_err(h, e, "receive counts");
  if (shared && !tcp) {
    e = cudaMemsetAsync(ep_at<float>(h, p2.ysh), 0, sizeof(float) * T * H, h->stream);
    if (e != cudaSuccess) return cuda_err(h, e, "cudaMemsetAsync");
  }
  const fm::EpPlanArgs pa = ep_plan_args(h, c, E_local, T, shared, tcp, p2);
  prof_begin(h, "ep_plan");
  fm::ep_plan_kernel<<<1, fm::kRouteThreads, 0, h->stream>>>(pa);
  prof_end(h);
  e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_err(h, e, "ep_plan launch");
  if (R == 0 && !shared) return FM_OK;

  return ep_gemms(h, c, w, recv_rows, R, T, E_local, shared, tcp, p1, p2, pa, d_rows);
}

int fm_ep_combine(fm_handle* h, const fm_moe_config* c, const uint16_t* ret_rows, uint16_t* y) {
  if (!h) return FM_EINVAL;
  if (h->ep_stage != 2) return set_err(h, FM_EINVAL, "fm_ep_combine must follow fm_ep_experts");
  if (!c) return set_err(h, FM_EINVAL, "null config");
  const int64_t T = h->ep_T;
  h->ep_stage = 0;
  if (T == 0) return FM_OK;
  if (!y || !ret_rows) return set_err(h, FM_EINVAL, "null rows");
  if (!aligned16(ret_rows) || !aligned16(y)) return set_err(h, FM_EINVAL, "rows must be 16-byte aligned");
  const int H = c->hidden, E = c->num_experts, k = c->top_k;
  const EpPlan1 p1 = make_ep_plan1(T, H, E, k, (E + 1 + 7) / 8 * 8, router_ksplit(h, std::max<int64_t>(T, 1), H, E));
  const int Is = c->shared_inter, I = c->inter;
  int first = 0, E_local = 0;
  ep_range(E, h->ep_rank, h->ep_world, &first, &E_local);
  const EpPlan2 p2 = make_ep_plan2(h->ep_R, T, H, I, Is, h->ep_world * E_local, h->ep_shared);
  const bool shared = h->ep_shared;
  prof_begin(h, "ep_combine");
  fm::finalize_ep_kernel<<<grid_for(h, T * (H / 8)), 256, 0, h->stream>>>(
      ret_rows, at<int32_t>(h, p1.pair_pos), at<float>(h, p1.topk_score), k,
      (shared && !h->ep_ysh_bf16) ? ep_at<float>(h, p2.ysh) : nullptr,
      (shared && h->ep_ysh_bf16) ? ep_at<uint16_t>(h, p2.ysh) : nullptr, at<float>(h, p1.gate_sig), T, H, y);
  prof_end(h);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_err(h, e, "ep_combine launch");
  return FM_OK;
}

// ---------------------------------------------------------------- expert parallelism over peer memory
// Region layout (identical on every rank of the group; offsets in bytes):
//   [0, 256)      local control: the grid completion counter of the exchange kernels
//   off_flags     u32 [3][W]      epoch of the last post per (kind, source rank)
//   off_counts    i32 [W][E]      pairs of every source rank per global expert
//   off_recv      bf16 [cap_recv][H]  rows received as an owner
//   off_ret       bf16 [cap_ret][H]   d rows returned to this rank as a token owner
int fm_ep_p2p_alloc(fm_handle* h, const fm_moe_config* c, int64_t max_tokens, void* ipc_handle_out) {
  if (!h) return FM_EINVAL;
  if (!c || !ipc_handle_out || max_tokens <= 0) return set_err(h, FM_EINVAL, "null argument or max_tokens <= 0");
  if (h->borrowed_ws) return set_err(h, FM_ETOOLARGE, "expert parallelism needs an allocating handle");
  const int W = h->ep_world, E = c->num_experts, H = c->hidden, k = c->top_k;
  if (W > fm::kEpMaxWorld) return set_err(h, FM_EUNSUPPORTED, "peer-memory exchange supports up to 8 ranks");
  if (H <= 0 || H % 128 || E <= 0 || k <= 0 || k > E || E > fm::kMaxExperts)
    return set_err(h, FM_EINVAL, "bad MoE dimensions");
  if (max_tokens > (1LL << 24)) return set_err(h, FM_EUNSUPPORTED, "max_tokens too large");
  p2p_close(h);
  auto& q = h->p2p;
  const int64_t e_local_max = (E + W - 1) / W;
  q.world = W;
  q.E = E;
  q.H = H;
  q.k = k;
  q.max_tokens = max_tokens;
  q.cap_recv = static_cast<int64_t>(W) * max_tokens * std::min<int64_t>(k, e_local_max);
  q.cap_ret = max_tokens * k;
  size_t off = 256;
  q.off_flags = static_cast<int64_t>(off);
  off = align_up(off + sizeof(uint32_t) * 3 * W, 256);
  q.off_counts = static_cast<int64_t>(off);
  off = align_up(off + sizeof(int32_t) * static_cast<size_t>(W) * E, 256);
  q.off_recv = static_cast<int64_t>(off);
  off = align_up(off + sizeof(uint16_t) * static_cast<size_t>(q.cap_recv) * H, 256);
  q.off_ret = static_cast<int64_t>(off);
  off = align_up(off + sizeof(uint16_t) * static_cast<size_t>(q.cap_ret) * H, 256);
  q.bytes = off;
  cudaError_t e = cudaMalloc(&q.region, q.bytes);
  if (e != cudaSuccess) {
    cudaGetLastError();
    q = fm_handle::P2P();
    return set_err(h, FM_ENOMEM, std::string("peer-exchange region allocation failed: ") + cudaGetErrorString(e));
  }
  e = cudaMemsetAsync(q.region, 0, static_cast<size_t>(q.off_recv), h->stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(h->stream);
  cudaIpcMemHandle_t ipc;
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(&ipc, q.region);
  int per_sm = 0;
  if (e == cudaSuccess) e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fm::ep_dispatch_kernel, 256, 0);
  if (e != cudaSuccess) {
    p2p_close(h);
    return cuda_err(h, e, "peer-exchange region setup");
  }
  q.coop_blocks = h->num_sms * std::max(1, std::min(per_sm, 4));
  q.peer[h->ep_rank] = q.region;
  std::memcpy(ipc_handle_out, &ipc, sizeof(ipc));
  return FM_OK;
}

int fm_ep_p2p_open(fm_handle* h, const void* ipc_handles) {
  if (!h) return FM_EINVAL;
  auto& q = h->p2p;
  if (!q.region) return set_err(h, FM_EINVAL, "fm_ep_p2p_open must follow fm_ep_p2p_alloc");
  if (q.open) return set_err(h, FM_EINVAL, "peer regions already open");
  if (!ipc_handles && q.world > 1) return set_err(h, FM_EINVAL, "null handles");
  for (int r = 0; r < q.world; ++r) {
    if (r == h->ep_rank) continue;
    cudaIpcMemHandle_t ipc;
    std::memcpy(&ipc, static_cast<const uint8_t*>(ipc_handles) + static_cast<size_t>(r) * sizeof(ipc), sizeof(ipc));
    void* ptr = nullptr;
    const cudaError_t e = cudaIpcOpenMemHandle(&ptr, ipc, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) {
      for (int s = 0; s < r; ++s)
        if (q.mapped[s]) {
          cudaIpcCloseMemHandle(q.peer[s]);
          q.mapped[s] = false;
          q.peer[s] = nullptr;
        }
      return cuda_err(h, e, "cudaIpcOpenMemHandle");
    }
    q.peer[r] = static_cast<uint8_t*>(ptr);
    q.mapped[r] = true;
  }
  q.open = true;
  return FM_OK;
}

int fm_ep_p2p_close(fm_handle* h) {
  if (!h) return FM_EINVAL;
  p2p_close(h);
  return FM_OK;
}

int fm_ep_p2p_forward(fm_handle* h, const fm_moe_config* c, const fm_moe_weights* w, const uint16_t* x, int64_t T,
                      uint16_t* y) {
  if (!h) return FM_EINVAL;
  auto& q = h->p2p;
  if (!q.open) return set_err(h, FM_EINVAL, "peer regions not open (fm_ep_p2p_alloc, fm_ep_p2p_open)");
  int rc = check_ep_route(h, c, w, x, T);
  if (rc) return rc;
  const int H = c->hidden, I = c->inter, E = c->num_experts, k = c->top_k, Is = c->shared_inter;
  if (E != q.E || H != q.H || k != q.k || h->ep_world != q.world)
    return set_err(h, FM_EINVAL, "config differs from the one the peer regions were sized for");
  if (T > q.max_tokens) return set_err(h, FM_ETOOLARGE, "T exceeds the max_tokens of fm_ep_p2p_alloc");
  if (T > 0 && !y) return set_err(h, FM_EINVAL, "null y");
  if (!aligned16(y)) return set_err(h, FM_EINVAL, "y must be 16-byte aligned");
  int first = 0, E_local = 0;
  ep_range(E, h->ep_rank, h->ep_world, &first, &E_local);
  const int nseg = h->ep_world * E_local;
  if (nseg + 1 > fm::kMaxGroups) return set_err(h, FM_EUNSUPPORTED, "too many (rank, expert) segments");
  const bool shared = Is > 0 && T > 0;
  const bool routed = E_local > 0;
  rc = check_ep_experts(h, c, w, routed, shared);
  if (rc) return rc;
  // the receive count is not known on the host: decide the path on this rank's own pairs
  const bool tcp = use_tc(h, T * k + (shared ? T : 0), E_local + (shared ? 1 : 0), c->group_size);
  h->last_path = tcp ? FM_PATH_TCGEN05 : FM_PATH_GEMV;
  const int ksplit = router_ksplit(h, std::max<int64_t>(T, 1), H, E);
  const EpPlan1 p1 = make_ep_plan1(T, H, E, k, (E + 1 + 7) / 8 * 8, ksplit);
  rc = ensure_ws(h, p1.total);
  if (rc) return rc;
  const EpPlan2 p2 = make_ep_plan2_p2p(q.cap_recv, T, H, I, Is, nseg, shared);
  rc = ensure_ep_ws(h, p2.total);
  if (rc) return rc;
  if (++q.epoch == 0) q.epoch = 1;
  cudaError_t e = cudaMemsetAsync(q.region, 0, 256, h->stream);
  if (e != cudaSuccess) return cuda_err(h, e, "cudaMemsetAsync");
  RouteArgs ra = ep_route_args(h, c, w, x, T, ksplit, p1);
  if (T > 0) {
    rc = launch_route(h, ra, ((T + 15) / 16) * ksplit);
    if (rc) return rc;
  } else {
    e = cudaMemsetAsync(ra.offsets, 0, sizeof(int32_t) * (E + 1), h->stream);
    if (e != cudaSuccess) return cuda_err(h, e, "cudaMemsetAsync");
  }
  if (shared && !tcp) {
    e = cudaMemsetAsync(ep_at<float>(h, p2.ysh), 0, sizeof(float) * T * H, h->stream);
    if (e != cudaSuccess) return cuda_err(h, e, "cudaMemsetAsync");
  }
  fm::EpPlanArgs pa = ep_plan_args(h, c, E_local, T, shared, tcp, p2);
  pa.src_rot = h->ep_rank;  // see ep_plan_body: owners start their stores at different sources
  fm::EpP2PArgs a;
  std::memset(&a, 0, sizeof(a));
  for (int r = 0; r < q.world; ++r) a.peer[r] = q.peer[r];
  a.rank = h->ep_rank;
  a.world = q.world;
  a.E = E;
  a.H = H;
  a.k = k;
  a.epoch = q.epoch;
  a.off_flags = q.off_flags;
  a.off_counts = q.off_counts;
  a.off_recv = q.off_recv;
  a.off_ret = q.off_ret;
  a.cap_recv = q.cap_recv;
  a.cap_ret = q.cap_ret;
  a.offsets = ra.offsets;
  a.sorted_token = ra.sorted_token;
  a.x_perm = ra.x_perm;
  a.P = T * k;
  a.row_dst = ep_at<uint16_t*>(h, p2.row_dst);
  a.done_counter = reinterpret_cast<int32_t*>(q.region);
  a.err = err_word(h);

  prof_begin(h, "ep_p2p_dispatch");
  {
    const int64_t want = (a.P * (H / 8) + 255) / 256;
    const int grid = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(want, q.coop_blocks)));
    void* args[] = {&a};
    e = cudaLaunchCooperativeKernel(reinterpret_cast<const void*>(fm::ep_dispatch_kernel), dim3(grid), dim3(256),
                                    args, 0, h->stream);
  }
  prof_end(h);
  if (e != cudaSuccess) return cuda_err(h, e, "ep_dispatch launch");
  prof_begin(h, "ep_p2p_plan");
  fm::ep_p2p_plan_kernel<<<1, fm::kRouteThreads, 0, h->stream>>>(a, pa);
  prof_end(h);
  e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_err(h, e, "ep_plan launch");
  if (routed || shared) {
    uint16_t* recv = reinterpret_cast<uint16_t*>(q.region + q.off_recv);
    rc = ep_gemms(h, c, w, recv, routed ? q.cap_recv : 0, T, E_local, shared, tcp, p1, p2, pa,
                  nullptr, a.row_dst);
    if (rc) return rc;
  }
  prof_begin(h, "ep_p2p_release");
  fm::ep_release_kernel<<<1, 32, 0, h->stream>>>(a, 2);
  prof_end(h);
  e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_err(h, e, "ep_release launch");
  prof_begin(h, "ep_p2p_combine");
  fm::ep_combine_p2p_kernel<<<grid_for(h, T * (H / 8)), 256, 0, h->stream>>>(
      a, ra.pair_pos, ra.topk_score, k, (shared && !tcp) ? ep_at<float>(h, p2.ysh) : nullptr,
      (shared && tcp) ? ep_at<uint16_t>(h, p2.ysh) : nullptr, ra.gate_sig, T, y);
  prof_end(h);
  e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_err(h, e, "ep_combine launch");
  return FM_OK;
}

int fm_quantized_matmul(fm_handle* h, const uint16_t* x, int64_t M, int K, const uint32_t* w,
                        const uint16_t* scales, const uint16_t* biases, int N, int transpose, int group_size,
                        int bits, uint16_t* out) {
  if (!h) return FM_EINVAL;
  if (M < 0) return set_err(h, FM_EINVAL, "negative M");
  if (M == 0) return FM_OK;
  if (M > (1LL << 24)) return set_err(h, FM_EUNSUPPORTED, "too many rows");
  // one expert, one batch of M rows: gather_qmm with E = 1 and no indices
  return fm_gather_qmm(h, x, 1, static_cast<int>(M), K, w, scales, biases, 1, N, nullptr, nullptr, 1, transpose,
                       group_size, bits, 1, out);
}

// ---------------------------------------------------------------- decoder ops (decoder.cu)

int fm_dequantize(fm_handle* h, const uint32_t* w, const uint16_t* scales, const uint16_t* biases, int64_t N, int K,
                  int group_size, int bits, uint16_t* out) {
  if (!h) return FM_EINVAL;
  if (!quant_ok(K, group_size, bits) || K % 8) return set_err(h, FM_EUNSUPPORTED, "only 4-bit affine, group 32/64/128");
  if (N < 0) return set_err(h, FM_EINVAL, "negative N");
  if (N == 0) return FM_OK;
  if (!w || !scales || !out) return set_err(h, FM_EINVAL, "null pointer");
  if (!aligned16(out) || (reinterpret_cast<uintptr_t>(w) & 3)) return set_err(h, FM_EINVAL, "misaligned pointer");
  prof_begin(h, "dequantize");
  const cudaError_t e = fm::launch_dequant(w, scales, biases, N, K, group_size, out, h->num_sms, h->stream);
  prof_end(h);
  return e == cudaSuccess ? FM_OK : cuda_err(h, e, "dequantize launch");
}

int fm_embed(fm_handle* h, const uint16_t* table, int64_t V, int H, const int32_t* ids, int64_t T, uint16_t* y) {
  if (!h) return FM_EINVAL;
  if (V <= 0 || H <= 0 || H % 8 || T < 0) return set_err(h, FM_EINVAL, "bad sizes (H % 8 == 0)");
  if (T == 0) return FM_OK;
  if (!table || !ids || !y) return set_err(h, FM_EINVAL, "null pointer");
  if (!aligned16(table) || !aligned16(y)) return set_err(h, FM_EINVAL, "table and y must be 16-byte aligned");
  prof_begin(h, "embed");
  const cudaError_t e = fm::launch_embed(table, V, H, ids, T, y, err_word(h), h->num_sms, h->stream);
  prof_end(h);
  return e == cudaSuccess ? FM_OK : cuda_err(h, e, "embed launch");
}

int fm_rms_norm(fm_handle* h, const uint16_t* x, const uint16_t* residual, const uint16_t* weight, int64_t T, int H,
                float eps, uint16_t* h_out, uint16_t* y) {
  if (!h) return FM_EINVAL;
  if (H <= 0 || H % 8 || T < 0 || !(eps >= 0.f)) return set_err(h, FM_EINVAL, "bad sizes (H % 8 == 0) or eps");
  if (T == 0) return FM_OK;
  if (T > 0x7fffffffLL) return set_err(h, FM_EUNSUPPORTED, "too many rows");
  if (!x || !weight || !y) return set_err(h, FM_EINVAL, "null pointer");
  if (!aligned16(x) || !aligned16(weight) || !aligned16(y) || (residual && !aligned16(residual)) ||
      (h_out && !aligned16(h_out)))
    return set_err(h, FM_EINVAL, "rows must be 16-byte aligned");
  if (y == x || y == residual) return set_err(h, FM_EINVAL, "y may not alias x or residual");
  prof_begin(h, "rms_norm");
  const cudaError_t e = fm::launch_rms_norm(x, residual, weight, T, H, eps, h_out, y, h->stream);
  prof_end(h);
  return e == cudaSuccess ? FM_OK : cuda_err(h, e, "rms_norm launch");
}

int fm_attention(fm_handle* h, const fm_attn_config* cfg, uint16_t* q, const uint16_t* k, const uint16_t* v,
                 const uint16_t* q_bias, const uint16_t* k_bias, const uint16_t* v_bias, const uint16_t* q_norm,
                 const uint16_t* k_norm, uint16_t* cache_k, uint16_t* cache_v, int B, int L, int offset,
                 uint16_t* out) {
  if (!h) return FM_EINVAL;
  if (!cfg) return set_err(h, FM_EINVAL, "null config");
  const int nh = cfg->n_heads, nkv = cfg->n_kv_heads, d = cfg->head_dim;
  if (nh <= 0 || nkv <= 0 || nh % nkv || cfg->max_len <= 0 || !(cfg->rope_theta > 0.f))
    return set_err(h, FM_EINVAL, "bad attention config");
  if (d != 64 && d != 128) return set_err(h, FM_EUNSUPPORTED, "head_dim must be 64 or 128");
  if ((q_norm || k_norm) && !(cfg->norm_eps >= 0.f)) return set_err(h, FM_EINVAL, "bad QK-norm eps");
  if (cfg->qkv_ld < 0 || cfg->qkv_ld % 8 || (cfg->qkv_ld > 0 && cfg->qkv_ld < nh * d))
    return set_err(h, FM_EINVAL, "qkv_ld must be 0 or a multiple of 8 of at least n_heads * head_dim");
  if (B < 0 || L < 0 || offset < 0) return set_err(h, FM_EINVAL, "negative B, L or offset");
  if (B == 0 || L == 0) return FM_OK;
  if (static_cast<int64_t>(offset) + L > cfg->max_len) return set_err(h, FM_EINVAL, "offset + L exceeds max_len");
  if (static_cast<int64_t>(B) * L > 0x7fffffffLL / (nh + 2 * nkv) || nh > 65535 || B > 65535)
    return set_err(h, FM_EUNSUPPORTED, "too many tokens or heads");
  if (!q || !k || !v || !cache_k || !cache_v || !out) return set_err(h, FM_EINVAL, "null pointer");
  if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(cache_k) || !aligned16(cache_v) ||
      !aligned16(out))
    return set_err(h, FM_EINVAL, "q, k, v, caches and out must be 16-byte aligned");
  if (out == q) return set_err(h, FM_EINVAL, "out may not alias q");
  if (!h->attn_ready) {
    const cudaError_t ie = fm::attn_init();
    if (ie != cudaSuccess) return cuda_err(h, ie, "attention kernel set-up");
    h->attn_ready = true;
  }
  fm::AttnArgs a;
  std::memset(&a, 0, sizeof(a));
  a.q = q;
  a.k = k;
  a.v = v;
  a.q_bias = q_bias;
  a.k_bias = k_bias;
  a.v_bias = v_bias;
  a.q_norm = q_norm;
  a.k_norm = k_norm;
  a.norm_eps = cfg->norm_eps;
  a.cache_k = cache_k;
  a.cache_v = cache_v;
  a.out = out;
  a.q_ld = cfg->qkv_ld > 0 ? cfg->qkv_ld : static_cast<int64_t>(nh) * d;
  a.kv_ld = cfg->qkv_ld > 0 ? cfg->qkv_ld : static_cast<int64_t>(nkv) * d;
  a.out_ld = static_cast<int64_t>(nh) * d;
  a.B = B;
  a.L = L;
  a.offset = offset;
  a.nh = nh;
  a.nkv = nkv;
  a.head_dim = d;
  a.max_len = cfg->max_len;
  a.scale = cfg->scale != 0.f ? cfg->scale : 1.0f / std::sqrt(static_cast<float>(d));
  a.log2_theta = std::log2(static_cast<double>(cfg->rope_theta));
  prof_begin(h, "attention");
  const cudaError_t e = fm::launch_attention(a, h->stream);
  prof_end(h);
  return e == cudaSuccess ? FM_OK : cuda_err(h, e, "attention launch");
}

int fm_swiglu(fm_handle* h, const uint16_t* gate, const uint16_t* up, int64_t n, uint16_t* out) {
  if (!h) return FM_EINVAL;
  if (n < 0) return set_err(h, FM_EINVAL, "negative n");
  if (n == 0) return FM_OK;
  if (!gate || !up || !out) return set_err(h, FM_EINVAL, "null pointer");
  prof_begin(h, "swiglu");
  const cudaError_t e = fm::launch_swiglu(gate, up, n, out, h->num_sms, h->stream);
  prof_end(h);
  return e == cudaSuccess ? FM_OK : cuda_err(h, e, "swiglu launch");
}

int fm_argmax(fm_handle* h, const uint16_t* logits, int64_t T, int64_t V, int32_t* ids) {
  if (!h) return FM_EINVAL;
  if (T < 0 || V <= 0 || V > 0x7fffffffLL) return set_err(h, FM_EINVAL, "bad sizes");
  if (T == 0) return FM_OK;
  if (T > 0x7fffffffLL) return set_err(h, FM_EUNSUPPORTED, "too many rows");
  if (!logits || !ids) return set_err(h, FM_EINVAL, "null pointer");
  prof_begin(h, "argmax");
  const cudaError_t e = fm::launch_argmax(logits, T, V, ids, h->stream);
  prof_end(h);
  return e == cudaSuccess ? FM_OK : cuda_err(h, e, "argmax launch");
}

}  // extern "C"

// ---------------------------------------------------------------- no-allocation entry point
//
// fm_moe_block_noalloc runs the same kernels as fm_moe_block, but its scratch (the
// routing tables, the expert-sorted activations and the fp32 combine buffers) lives in
// the fixed array below instead of a handle-owned cudaMalloc workspace.  Every GPU
// that loads this library holds the array until the process exits.  All calls on a
// device share it and it keeps the last call's contents: each call clears the control
// block (error word, grid-barrier counters) on its stream before use, and calls whose
// execution overlaps on the GPU race on the array.

namespace {

constexpr size_t kNoAllocScratchBytes = size_t(16) << 20;  // 16 MiB per device
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

struct NoAllocDevice {
  bool ready = false;
  int status = FM_OK;
  uint8_t* scratch = nullptr;  // device address of g_noalloc_scratch on this device
  int num_sms = 0;
  int route_blocks_per_sm = 0;
  int route_wide_blocks_per_sm = 0;
  int gemv_blocks_per_sm = 0;
  int gemv_tma_blocks_per_sm = 0;  // TMA-fed GEMV (qgemv_tma.cu); 0: not available
  int tc_pairs = 0;
};
constexpr int kNoAllocMaxDevices = 64;
NoAllocDevice g_noalloc_dev[kNoAllocMaxDevices];
std::mutex g_noalloc_mu;

// One-time set-up for `device`, which must be current: resolve the array's device
// address (host code only ever sees a host-side stand-in for its name), query the
// launch parameters fm_create would, and clear the control block.
int noalloc_setup(int device, NoAllocDevice& d) {
  void* p = nullptr;
  cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
  int cc_major = 0, cc_minor = 0;
  if (e == cudaSuccess) e = cudaDeviceGetAttribute(&d.num_sms, cudaDevAttrMultiProcessorCount, device);
  if (e == cudaSuccess) e = cudaDeviceGetAttribute(&cc_major, cudaDevAttrComputeCapabilityMajor, device);
  if (e == cudaSuccess) e = cudaDeviceGetAttribute(&cc_minor, cudaDevAttrComputeCapabilityMinor, device);
  if (e == cudaSuccess && !(cc_major == 10 && cc_minor == 0)) return FM_EUNSUPPORTED;
  if (e == cudaSuccess)
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&d.route_blocks_per_sm, fm::route_kernel, fm::kRouteThreads, 0);
  if (e == cudaSuccess)
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&d.route_wide_blocks_per_sm, fm::route_kernel_wide,
                                                      fm::kRouteThreads, 0);
  if (e == cudaSuccess) e = fm::qgemv_blocks_per_sm(&d.gemv_blocks_per_sm);
  if (e == cudaSuccess) e = fm::qgemv_tma_blocks_per_sm(&d.gemv_tma_blocks_per_sm);
  if (e == cudaSuccess) e = fm::tc::init();
  if (e == cudaSuccess) e = fm::tc::max_pairs(&d.tc_pairs);
  if (e == cudaSuccess && d.tc_pairs < 1) e = cudaErrorInvalidConfiguration;
  if (e == cudaSuccess) e = cudaMemset(p, 0, kCtrlBytes);
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  if (e != cudaSuccess) {
    cudaGetLastError();
    return FM_ECUDA;
  }
  d.scratch = static_cast<uint8_t*>(p);
  d.gemv_blocks_per_sm = std::min(d.gemv_blocks_per_sm, 8);
  return FM_OK;
}

}  // namespace

extern "C" int fm_moe_block_noalloc(int device, void* stream, const fm_moe_config* c, const fm_moe_weights* w,
                                    const uint16_t* x, int64_t T, uint16_t* y) {
  if (device < 0 || device >= kNoAllocMaxDevices || !c || T < 0) return FM_EINVAL;
  int prev = -1;
  if (cudaGetDevice(&prev) != cudaSuccess) return FM_ECUDA;
  if (prev != device && cudaSetDevice(device) != cudaSuccess) {
    cudaGetLastError();
    return FM_ECUDA;
  }
  NoAllocDevice& d = g_noalloc_dev[device];
  int rc = FM_OK;
  {
    std::lock_guard<std::mutex> lock(g_noalloc_mu);
    if (!d.ready) {
      // the set-up synchronizes the device, which would invalidate a capture in progress
      cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
      if (cudaStreamIsCapturing(static_cast<cudaStream_t>(stream), &cap) != cudaSuccess) {
        cudaGetLastError();
        rc = FM_ECUDA;
      } else if (cap != cudaStreamCaptureStatusNone) {
        rc = FM_EINVAL;
      } else {
        rc = noalloc_setup(device, d);
        // an unsupported device stays unsupported; a failed CUDA call is retried next call
        d.ready = rc == FM_OK || rc == FM_EUNSUPPORTED;
        d.status = rc;
      }
    } else {
      rc = d.status;
    }
  }
  if (rc == FM_OK) {
    fm_handle h;  // borrows the fixed scratch; never grows or frees it
    h.device = device;
    h.stream = static_cast<cudaStream_t>(stream);
    h.num_sms = d.num_sms;
    h.route_blocks_per_sm = d.route_blocks_per_sm;
    h.route_wide_blocks_per_sm = d.route_wide_blocks_per_sm;
    h.gemv_blocks_per_sm = d.gemv_blocks_per_sm;
    h.gemv_tma_blocks_per_sm = d.gemv_tma_blocks_per_sm;
    h.tc_pairs = d.tc_pairs;
    h.ws = d.scratch;
    h.ws_bytes = kNoAllocScratchBytes;
    h.borrowed_ws = true;
    const int epad = (c->num_experts + 1 + 7) / 8 * 8;
    const size_t need = make_plan(T, T, c->hidden, c->num_experts, c->top_k, epad, router_ksplit(&h, T, c->hidden, c->num_experts),
                                  c->inter, c->shared_inter, c->shared_inter > 0, true,
                                  use_tc(&h, T * c->top_k, c->num_experts, c->group_size))
                            .total;
    if (need > kNoAllocScratchBytes) {
      rc = FM_ETOOLARGE;
    } else if (cudaMemsetAsync(d.scratch, 0, kCtrlBytes, h.stream) != cudaSuccess) {
      cudaGetLastError();
      rc = FM_ECUDA;
    } else {
      rc = fm_moe_block(&h, c, w, x, T, y, nullptr);
    }
  }
  if (prev != device) cudaSetDevice(prev);
  return rc;
}
