// fm_internal.cuh -- data structures shared by the libflashmoe kernels and host code.
#pragma once

#include <cuda.h>
#include <stdint.h>

#include "fm_common.cuh"

namespace fm {

constexpr int kMaxExperts = 512;
constexpr int kMaxGroups = kMaxExperts + 1;  // routed experts + the shared expert

// One weight matrix set (an expert, or the shared expert) and the activation rows it
// multiplies, cut into output-row blocks x token chunks x K splits.  Written on the
// device by the routing kernel (the row counts are only known there).
struct TileGroup {
  int32_t expert;      // expert id, -1 = shared expert
  int32_t row_begin;   // first activation row in the expert-major pair order
  int32_t rows;        // activation rows of this group
  int32_t chunk_rows;  // rows per token chunk
  int32_t chunks;      // token chunks
  int32_t nblocks;     // output-row blocks
  int32_t ksplit;      // K splits (GEMV path only; partial sums are added atomically)
  int32_t tile_begin;  // first tile id of the group
};

struct TileTable {
  int32_t num_groups;
  int32_t num_tiles;
  int32_t pad[6];
  TileGroup g[kMaxGroups];
};

struct TileInfo {
  int group;
  int expert;  // -1 shared
  int rb;      // output-row block
  int ks;      // K split index
  int ksplit;
  int row0;    // first activation row of the chunk
  int nrows;   // activation rows in the chunk
};

// tile `tile` of group G (index lo)
FM_DEV TileInfo tile_in_group(const TileGroup& G, int lo, int tile) {
  int local = tile - G.tile_begin;
  TileInfo t;
  t.group = lo;
  t.expert = G.expert;
  t.ksplit = G.ksplit;
  t.ks = local % G.ksplit;
  local /= G.ksplit;
  const int ch = local % G.chunks;
  t.rb = local / G.chunks;
  t.row0 = G.row_begin + ch * G.chunk_rows;
  t.nrows = min(G.chunk_rows, G.rows - ch * G.chunk_rows);
  return t;
}

FM_DEV TileInfo tile_of_group(const TileTable* tab, int lo, int tile) { return tile_in_group(tab->g[lo], lo, tile); }

FM_DEV TileInfo decode_tile(const TileTable* tab, int tile) {
  int lo = 0, hi = tab->num_groups - 1;
  while (lo < hi) {  // largest group with tile_begin <= tile
    const int mid = (lo + hi + 1) >> 1;
    if (tab->g[mid].tile_begin <= tile) lo = mid; else hi = mid - 1;
  }
  return tile_of_group(tab, lo, tile);
}

// same, searching a shared-memory copy of the groups' tile_begin values
FM_DEV TileInfo decode_tile(const TileTable* tab, const int* tile_begin, int ngroups, int tile) {
  int lo = 0, hi = ngroups - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (tile_begin[mid] <= tile) lo = mid; else hi = mid - 1;
  }
  return tile_of_group(tab, lo, tile);
}

// MODE_RELU2: one ungated matrix (fc1) per expert with relu^2, written like gate/up's
// activation rows for the down matrix (GEMV and tcgen05); MODE_DOWN_F32: down with fp32
// routing scores, the product d * score kept in fp32 (the sigmoid-routed variant's
// combine; GEMV only: the tcgen05 path stores bf16(d) per pair and combines separately).
enum GemmMode : int { MODE_GATEUP = 0, MODE_DOWN = 1, MODE_PLAIN = 2, MODE_RELU2 = 3, MODE_DOWN_F32 = 4 };

// Arguments of the expert-product kernels (GEMV and tcgen05 paths).
struct GemmArgs {
  int K;          // reduction length of routed matrices (H for gate/up, I for down)
  int K_shared;   // reduction length of the shared matrices
  int N;          // output rows of a routed matrix (I for gate/up, H for down)
  int N_shared;   // output rows of a shared matrix
  int gs;         // quantization group size
  int unit_score; // tcgen05 down: store bf16(d) per routed pair (the scores are applied by the combine)
  // routed matrices, stacked [E, N, K/8]; gate/up mode: 0 = gate, 1 = up
  const uint32_t* w0; const uint16_t* s0; const uint16_t* b0;
  const uint32_t* w1; const uint16_t* s1; const uint16_t* b1;
  // shared-expert matrices [N_shared, K_shared/8]
  const uint32_t* sw0; const uint16_t* ss0; const uint16_t* sb0;
  const uint32_t* sw1; const uint16_t* ss1; const uint16_t* sb1;
  // activation rows (B operand), stored with the within-8 pair permutation
  const uint16_t* act;         // routed rows: x_perm (gate/up, plain) or a_sorted (down)
  const uint16_t* act_shared;  // shared rows: x_perm (gate/up) or a_shared (down)
  int64_t act_ld;
  int64_t act_shared_ld;
  // pair metadata in expert-major order
  const int32_t* sorted_token;  // token (gate/up, down) or source x row (plain)
  const float* sorted_score;
  const int32_t* sorted_flat;   // original pair / output row index
  // outputs
  uint16_t* out;          // gate/up: a_sorted [P, N]; plain: out [rows, N]
  uint16_t* out_shared;   // gate/up: a_shared [T, N_shared]
  int64_t out_ld;
  int64_t out_shared_ld;
  float* y_acc;           // down (GEMV): [T, H] fp32, sum_k bf16(d*score)
  float* ysh;             // down (GEMV): [T, H] fp32 shared-expert sums
  uint16_t* y_pairs;      // down (tcgen05): [P, H] bf16(bf16(d)*score), expert-major rows
  uint16_t* const* y_rowptr;  // down, instead of y_pairs: destination of each pair's row
                              // (another rank's memory over NVLink, expert parallelism)
  uint16_t* ysh16;        // down (tcgen05): [T, H] bf16 shared-expert rows
  int64_t y_ld;
  const TileTable* tab;
  uint32_t* err;
};

// TMA descriptors of one tcgen05 expert-product launch (host-encoded per call).
//   code[0..3]: packed 4-bit weight codes as uint32 [rows, K/8], 128B swizzle, box
//               {32 words = 4 k-steps, 64 rows (gate/up) | 128 rows (down, plain)}:
//               gate/up: routed gate, routed up, shared gate, shared up;
//               down / plain: routed, (unused), shared, (unused)
//   act[0]:     routed activation rows, bf16 [rows, K], 128B swizzle, box {64, 32}
//               (read by TMA only where the rows are contiguous: down; gate/up and
//               plain gather their token rows with cp.async)
//   act[1]:     shared-expert activation rows, box {64, 32}
//   act[2], act[3]: the same two tensors with boxes of {64, kActBigBoxRows} rows, so
//               a tile half of more than 64 rows takes one TMA per k-step, not 3-4
constexpr int kActBigBoxRows = 128;
struct alignas(64) TcMaps {
  CUtensorMap code[4];
  CUtensorMap act[4];
};

// Arguments of the routing kernel.
struct RouteArgs {
  // router mode inputs
  const uint16_t* x;            // [rows, H] bf16
  const uint16_t* router_w;     // [E, H] bf16
  const uint16_t* shared_gate_w;  // [1, H] bf16 or NULL
  const uint16_t* router_bias;  // [E] bf16 or NULL
  int64_t T;                    // tokens (router mode) / rows (given mode)
  int H;                        // row length of x
  int E;
  int k;
  int norm_topk;
  int do_router;                // 1: router + top-k; 0: experts given
  int ksplit;                   // router K slices (phase 1)
  int epad;                     // padded logit width (multiple of 8, >= E + has shared gate)
  // given mode (gather_qmm / quantized_matmul)
  const uint32_t* given_ids;    // expert of batch b (NULL: all expert 0)
  const uint32_t* given_lhs;    // x batch of batch b (NULL: broadcast)
  int64_t x_batches;
  int64_t batches;              // B
  int M;                        // rows per batch
  // workspace
  float* partial;               // [ksplit, T, epad]
  uint16_t* x_perm;             // [x_rows, H]
  int64_t x_rows;               // rows of x to permute
  float* zero0; int64_t zero0_n;  // buffers cleared in phase 1 (fp32 counts)
  float* zero1; int64_t zero1_n;
  int32_t* topk_ids;            // [T, k]
  float* topk_score;            // [T, k]
  float* gate_sig;              // [T]
  int32_t* row_src;             // [T] source x row (given mode)
  int32_t* chunk_counts;        // [nchunks, E]
  int32_t* pair_rank;           // [T, k]
  int32_t* totals;              // [E]
  int32_t* offsets;             // [E + 1]
  int32_t* sorted_token;        // [T*k]
  float* sorted_score;          // [T*k]
  int32_t* sorted_flat;         // [T*k]
  int32_t* pair_pos;            // [T*k] expert-major position of pair (t, j), or NULL
  // tile tables
  TileTable* tab_a;             // gate/up (or plain)
  TileTable* tab_b;             // down (NULL in plain mode)
  int a_rows_per_block;         // GEMV: 64 gate/up, 128 plain; tcgen05 pairs: 128, 256
  int a_n;                      // routed output rows of table a
  int a_n_shared;               // shared output rows of table a (0 = no shared group)
  int b_n;                      // output rows of table b (H)
  int b_rows_per_block;         // GEMV 128, tcgen05 pairs 256
  int chunk_max;                // token rows per chunk cap (8 GEMV, 256 tcgen05)
  int chunk_align;              // chunk size granularity (8 GEMV, 16 tcgen05)
  int b_ksplit_shared;          // K splits of the shared down group (GEMV)
  int has_shared;
  // user-visible outputs (nullable)
  int32_t* out_topk_ids;
  uint16_t* out_topk_scores;
  int32_t* out_sorted_token;
  int32_t* out_offsets;
  // sigmoid-routed variant (route_kernel_sigmoid): scores sigmoid(logit) [+ correction
  // bias for selection], group-limited top-k, fp32 renormalised and scaled scores
  int n_group, topk_group;
  float routed_scale;
  const float* corr_bias;       // [E] fp32 or NULL
  float* out_scores_f32;        // [T, k] fp32 scores as used (nullable, either routing)
  int shared_ungated;           // the shared expert is added without a gate (gate_sig = 1)
  GridSync* gsync;
  unsigned int* arrive;  // arrival counter of the last-block routing kernel (0 between launches)
  uint32_t* err;
  unsigned long long* phase_ns;  // [4] accumulated per-phase time of block 0 (profiling)
};

// Arguments of the expert-parallel plan kernel.
struct EpPlanArgs {
  const int32_t* recv_counts;  // [world, E_local] rows received per (source rank, local expert)
  int world;
  int E_local;
  int src_rot;                 // first source rank in the table's group order (then +1, ...)
  int T_shared;                // this rank's tokens for its shared-expert group (0: none)
  int a_n, a_n_shared, b_n;    // output rows of the routed / shared matrices per table
  int a_rows_per_block, b_rows_per_block;
  int chunk_max, chunk_align;
  int b_ksplit_shared;
  TileTable* tab_a;
  TileTable* tab_b;
  int32_t* row_map;            // [R] identity (received row p is activation row p)
  float* unit_score;           // [R] 1.0
  int32_t* recv_total;         // R
  uint32_t* err;
};

constexpr int kEpMaxWorld = 8;  // ranks of one peer-memory expert-parallel group

// Arguments of the expert-parallel exchange kernels over peer memory (layout: ep.cu).
struct EpP2PArgs {
  uint8_t* peer[kEpMaxWorld];  // region base of every rank, mapped here (peer[rank] = own)
  int rank, world;
  int E, H, k;
  uint32_t epoch;
  int64_t off_flags, off_counts, off_recv, off_ret;  // byte offsets in a region
  int64_t cap_recv, cap_ret;                         // rows of recv / ret
  // dispatch (token side)
  const int32_t* offsets;       // [E + 1] expert offsets of this rank's pairs
  const int32_t* sorted_token;  // [P] token of each pair, expert-major
  const uint16_t* x_perm;       // [T, H]
  int64_t P;
  // owner side
  uint16_t** row_dst;           // [cap_recv] where each received row's d goes: its source
                                // rank's ret buffer, at its position in that rank's send order
  int32_t* done_counter;        // grid completion counter, 0 between launches
  uint32_t* err;
};

// The attention step of a decoder layer (decoder.cu): q / k / v projections in, the KV
// cache updated, the attention rows out.  Activations are token-major [B * L, n * d].
struct AttnArgs {
  uint16_t* q;              // [B*L, q_ld] projections; rotated in place
  const uint16_t* k;        // [B*L, kv_ld]
  const uint16_t* v;        // [B*L, kv_ld]
  const uint16_t* q_bias;   // [nh * d] or null
  const uint16_t* k_bias;   // [nkv * d] or null
  const uint16_t* v_bias;   // [nkv * d] or null
  const uint16_t* q_norm;   // [d] per-head RMSNorm weight of q (QK-norm) or null
  const uint16_t* k_norm;   // [d] the same for k
  uint16_t* cache_k;        // [B, nkv, max_len, d]
  uint16_t* cache_v;
  uint16_t* out;            // [B*L, out_ld]
  int64_t q_ld, kv_ld, out_ld;
  int B, L, offset, nh, nkv, head_dim, max_len;
  float scale;              // softmax scale (1/sqrt(d) by default)
  float norm_eps;           // QK-norm eps
  double log2_theta;        // log2 of the RoPE base
};

constexpr int kRouteThreads = 256;  // 8 warps
constexpr int kRouteChunk = 16;     // tokens per counting chunk (one bitmask word)
constexpr int kRouterMaxKsplit = 32;  // K slices of the router partial logits
constexpr int kRouteLastMaxChunks = 8;  // batches the small-batch routing forms take (<= 128 tokens)
constexpr int kRouteClusterCtas = 8;    // CTAs of the cluster routing kernel (one portable cluster)

}  // namespace fm
