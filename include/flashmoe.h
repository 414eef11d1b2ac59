/*
 * flashmoe.h -- C ABI of libflashmoe, the B200 (sm_100a) MoE-block library.
 *
 * libflashmoe replaces, for FlashMLX's mixture-of-experts layers, the MLX operators
 * the reference's model forward calls (server/src/model.cpp):
 *
 *   fm_quantized_matmul  <- mx::quantized_matmul(x, w, scales, biases, transpose=true,
 *                           group_size, bits)        model.cpp:476-480, 531-535, 741-747
 *   fm_gather_qmm        <- mx::gather_qmm(x, w, scales, biases, lhs_indices, rhs_indices,
 *                           transpose=true, group_size, bits, "affine", sorted_indices)
 *                                                    model.cpp:703-721
 *   fm_moe_block         <- LlamaModel::moe_block (router, softmax, top-k, switch_mlp,
 *                           weighted combine, sigmoid-gated shared expert)
 *                                                    model.cpp:750-807 (+673-748)
 *
 * Conventions
 *   - bf16 tensors are passed as uint16_t bit patterns; all pointers are device
 *     pointers unless stated otherwise; every tensor is dense row-major.
 *   - Quantized weights use MLX's affine layout: w [.., N, K*bits/32] uint32 with
 *     element j of a row at bits bits*(j % (32/bits)) of word j/(32/bits) (low first),
 *     scales / biases [.., N, K/group_size] bf16, w_hat = scale * q + bias.
 *   - Calls are asynchronous on the handle's stream.  They return a status for the
 *     argument checks and launch; faults detected on the device (bounded waits that
 *     ran out, failed bounds checks) surface at the next fm_sync_status().
 *   - No C++ exception crosses this boundary.  The library never calls exit/abort.
 *   - One handle per host thread / stream.  A handle owns a device workspace that
 *     grows on demand; fm_reserve() sizes it up front so hot calls never allocate.
 */
#ifndef FLASHMOE_H_
#define FLASHMOE_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define FM_ABI_VERSION 1

#if defined(__GNUC__)
#define FM_API __attribute__((visibility("default")))
#else
#define FM_API
#endif

typedef enum fm_status {
  FM_OK = 0,
  FM_EINVAL = 1,        /* bad argument (null pointer, negative size, index range) */
  FM_EUNSUPPORTED = 2,  /* valid for MLX but not implemented here (bits, group size, shape) */
  FM_ECUDA = 3,         /* a CUDA runtime call failed; fm_last_error() has the text */
  FM_ENCCL = 4,         /* expert-parallel transport failure */
  FM_ETIMEOUT = 5,      /* a bounded device-side wait ran out */
  FM_EDEVICE = 6,       /* a kernel reported a failed device-side check */
  FM_ENOMEM = 7,        /* workspace allocation failed */
  FM_ETOOLARGE = 8      /* fm_moe_block_noalloc: the call needs more than its fixed scratch */
} fm_status;

typedef struct fm_handle fm_handle;

/* One affine-quantized matrix (possibly stacked over experts). */
typedef struct fm_qweight {
  const uint32_t* w;       /* [.., N, K*bits/32] */
  const uint16_t* scales;  /* [.., N, K/group_size] bf16 */
  const uint16_t* biases;  /* [.., N, K/group_size] bf16, NULL = zero */
} fm_qweight;

/* ModelConfig's MoE fields (server/include/flashmlx/model.h:40-45) plus the
 * quantization parameters (model.h:35-36). */
typedef struct fm_moe_config {
  int hidden;                /* H (hidden_size) */
  int inter;                 /* I (moe_intermediate_size) */
  int num_experts;           /* E */
  int top_k;                 /* k (num_experts_per_tok) */
  int group_size;            /* quant_group_size (64) */
  int bits;                  /* quant_bits (4) */
  int norm_topk_prob;        /* renormalise the k scores to sum 1 */
  int shared_inter;          /* shared_expert_intermediate_size, 0 = no shared expert */
  int router_quantized;      /* router weight quantized (model.cpp:757-760) */
  int shared_gate_quantized; /* shared_expert_gate quantized (model.cpp:792-797) */
} fm_moe_config;

/* MoEWeights (model.h:56-72): stacked expert weights of one layer. */
typedef struct fm_moe_weights {
  const void* router_w;       /* [E, H] bf16, or [E, H*bits/32] uint32 when quantized */
  const uint16_t* router_s;   /* quantized router only */
  const uint16_t* router_b;
  fm_qweight gate;            /* [E, I, H] */
  fm_qweight up;              /* [E, I, H] */
  fm_qweight down;            /* [E, H, I] */
  fm_qweight shared_gate;     /* [Is, H] */
  fm_qweight shared_up;       /* [Is, H] */
  fm_qweight shared_down;     /* [H, Is] */
  const void* shared_expert_gate_w; /* [1, H] bf16 (or packed when quantized) */
  const uint16_t* shared_expert_gate_s;
  const uint16_t* shared_expert_gate_b;
  const uint16_t* router_bias; /* [E] bf16 added to the logits, NULL in the reference
                                  model; used by the benchmark to skew expert load */
} fm_moe_weights;

/* Optional outputs of fm_moe_block (each pointer may be NULL). */
typedef struct fm_moe_outputs {
  int32_t* topk_ids;       /* [T, k] expert ids, descending score, ties -> lower id */
  uint16_t* topk_scores;   /* [T, k] bf16 routing weights (after optional renorm) */
  int32_t* sorted_token;   /* [T*k] token of each pair in stable expert-major order */
  int32_t* expert_offsets; /* [E+1] start of each expert's segment in that order */
} fm_moe_outputs;

/* Routing / expert variant of an MoE block.  All zero (or cfg-only calls through
 * fm_moe_block) is the reference's LlamaModel block: softmax routing, SwiGLU gate/up/down
 * experts, a sigmoid-gated shared expert.  The Nemotron-H / DeepSeek-style block of
 * NemotronHModel::moe_block (nemotron_h.cpp:1010-1106) is score_func = FM_SCORE_SIGMOID,
 * expert_act = FM_ACT_RELU2, shared_ungated = 1:
 *   orig = sigmoid(fp32(bf16 logits)), sel = orig + correction_bias; with n_group > 1 each
 *   of the n_group equal expert groups scores the sum of its two best sel and the
 *   n_group - topk_group lowest groups get sel = 0; the top-k of sel take their orig as
 *   scores, divided by (their sum + 1e-20) when norm_topk_prob and k > 1, times
 *   routed_scaling_factor, in fp32; experts h = fc2(relu2(fc1(x))) with fc1 passed as
 *   weights.up and fc2 as weights.down (weights.gate unused); y = bf16(sum_k h_k * s_k)
 *   in fp32, plus bf16(shared_down(relu2(shared_up(x)))) unweighted when the layer has a
 *   shared expert (shared_inter > 0; weights.shared_gate and shared_expert_gate_w unused). */
#define FM_SCORE_SOFTMAX 0
#define FM_SCORE_SIGMOID 1
#define FM_ACT_SWIGLU 0
#define FM_ACT_RELU2 1

typedef struct fm_moe_variant {
  int score_func;               /* FM_SCORE_SOFTMAX | FM_SCORE_SIGMOID */
  int n_group;                  /* sigmoid: expert groups for group-limited top-k (<= 32); 0 or 1 = off */
  int topk_group;               /* sigmoid: groups kept */
  float routed_scaling_factor;  /* sigmoid: multiplies the scores; 0 reads as 1 */
  int expert_act;               /* FM_ACT_SWIGLU | FM_ACT_RELU2 */
  int shared_ungated;           /* 1: the shared expert's output is added without the sigmoid gate */
  const float* correction_bias; /* sigmoid: [E] fp32 e_score_correction_bias (selection only), or NULL */
  float* topk_scores_f32;       /* optional [T, k] fp32 scores as applied (device) */
} fm_moe_variant;

/* Handle lifecycle -------------------------------------------------------- */

/* Creates a handle on `device`, issuing work on `stream` (a cudaStream_t, NULL =
 * legacy default stream).  Replaces no reference interface: MLX binds its device
 * and stream implicitly (mx::default_device / default_stream). */
FM_API int fm_create(fm_handle** out, int device, void* stream);
FM_API int fm_destroy(fm_handle* h);
FM_API int fm_set_stream(fm_handle* h, void* stream);
FM_API const char* fm_last_error(const fm_handle* h);
FM_API const char* fm_status_string(int status);

/* Synchronizes the stream and folds device-side error bits into a status.
 * The MLX analogue is the sync at mx::eval (scheduler.cpp:204). */
FM_API int fm_sync_status(fm_handle* h);

/* Pre-sizes the workspace for fm_moe_block calls of up to max_tokens tokens. */
FM_API int fm_reserve(fm_handle* h, const fm_moe_config* cfg, int64_t max_tokens);
FM_API size_t fm_workspace_bytes(const fm_handle* h);
/* The device workspace fm_reserve(h, cfg, max_tokens) makes a handle hold, computed on
 * the host without a handle or a device (for a caller budgeting device memory before
 * creating handles); 0 for an invalid config or max_tokens < 0. */
FM_API size_t fm_workspace_size(const fm_moe_config* cfg, int64_t max_tokens);

/* Path selection for the expert products.  FM_PATH_AUTO picks the small-batch
 * dequant-GEMV for few tokens per expert and the tcgen05 grouped GEMM otherwise. */
enum { FM_PATH_AUTO = 0, FM_PATH_GEMV = 1, FM_PATH_TCGEN05 = 2 };
FM_API int fm_set_path(fm_handle* h, int path);
/* The expert-product path (FM_PATH_GEMV or FM_PATH_TCGEN05) that the handle's last
 * fm_moe_block / fm_moe_block_variant / fm_quantized_matmul / fm_gather_qmm / fm_linear /
 * expert-parallel call took, 0 before the first.  The two paths follow MLX's two
 * arithmetic forms of a 4-bit product: the GEMV keeps the dequantized weights exact
 * (s * sum(q x) + b * sum(x) in fp32, MLX's qmv), the tcgen05 GEMM rounds each weight
 * s * q + b to bf16 (MLX's qmm tiles).  No reference counterpart (MLX picks its kernel
 * internally). */
FM_API int fm_last_path(const fm_handle* h);

/* Form of the routing kernel (router, top-k, sort and tile plan; the reference's
 * op chain of model.cpp:757-775 and 682-700).  FM_ROUTE_GRID: one cooperative kernel
 * whose four phases are separated by grid barriers.  FM_ROUTE_LAST_BLOCK: for batches
 * of at most 128 tokens (rows, for fm_gather_qmm), the router GEMV over the whole grid
 * and top-k, sort and planning in the one block that finishes it last, with no grid
 * barrier.  FM_ROUTE_CLUSTER: for batches of at most 128 tokens, one cluster of 8 CTAs
 * (router GEMV and top-k over the cluster, sort and planning in its first CTA, hardware
 * cluster barriers between them).  Larger batches take the grid form in every mode.
 * FM_ROUTE_AUTO (the default) is FM_ROUTE_CLUSTER.  All forms give identical results. */
enum { FM_ROUTE_AUTO = 0, FM_ROUTE_GRID = 1, FM_ROUTE_LAST_BLOCK = 2, FM_ROUTE_CLUSTER = 3 };
FM_API int fm_set_route_mode(fm_handle* h, int mode);

/* Kernel timing ------------------------------------------------------------------
 * With profiling on, every kernel the handle launches is bracketed by CUDA events on
 * the handle's stream; fm_profile_report() synchronizes and returns, per kernel
 * name, the launch count and the summed device time since the last reset.  The
 * reference's analogue is the ad-hoc std::chrono graph-build timers of
 * model.cpp:1163-1259 / scheduler.cpp:532-658. */
typedef struct fm_kernel_time {
  const char* name;     /* static string, e.g. "qgemm_tc_gateup" */
  int64_t launches;
  double total_ms;
} fm_kernel_time;
FM_API int fm_profile_enable(fm_handle* h, int on);
FM_API int fm_profile_report(fm_handle* h, fm_kernel_time* out, int capacity, int* count, int reset);

/* Operators ------------------------------------------------------------------
 * Activation and output pointers (x, y, out) must be 16-byte aligned (the kernels
 * move rows in 16-byte units); FM_EINVAL otherwise.  Weight codes, scales and
 * biases must be 16-byte aligned for the tcgen05 path's TMA descriptors (FM_ECUDA
 * from the descriptor encoder otherwise). */

/* out[M, N] = x[M, K] @ w_hat^T.  Replaces mx::quantized_matmul with transpose=true
 * (model.cpp:478-479, 509-511, 531-535, 741-747, 759-760, 793-796).
 * transpose=0 returns FM_EUNSUPPORTED (the reference never calls it). */
FM_API int fm_quantized_matmul(fm_handle* h, const uint16_t* x, int64_t M, int K, const uint32_t* w,
                        const uint16_t* scales, const uint16_t* biases, int N, int transpose,
                        int group_size, int bits, uint16_t* out);

/* out[B, M, N]: out[i] = x[lhs(i)] @ w_hat[rhs_indices[i]]^T, x [x_batches, M, K],
 * w [E, N, K*bits/32].  lhs_indices == NULL broadcasts x against rhs: lhs(i) =
 * i * x_batches / B (x [T,1,1,K] against rhs [T,k] gives lhs(i) = i / k).
 * sorted_indices is MLX's hint that rhs is ascending (model.cpp:703-721); results
 * do not depend on it.  Replaces mx::gather_qmm (model.cpp:703-721). */
FM_API int fm_gather_qmm(fm_handle* h, const uint16_t* x, int64_t x_batches, int M, int K, const uint32_t* w,
                  const uint16_t* scales, const uint16_t* biases, int E, int N,
                  const uint32_t* lhs_indices, const uint32_t* rhs_indices, int64_t B, int transpose,
                  int group_size, int bits, int sorted_indices, uint16_t* out);

/* out[M, N] = x[M, K] @ w_hat^T for a dense layer (the quantized_matmul of
 * LlamaModel::linear_fast, model.cpp:476-480, with transpose=true): the same result as
 * fm_quantized_matmul, but the rows are laid out and tiled by one plain kernel instead of
 * the routing kernel (no grid barriers; one launch fewer per call on the decode path). */
FM_API int fm_linear(fm_handle* h, const uint16_t* x, int64_t M, int K, const uint32_t* w, const uint16_t* scales,
                     const uint16_t* biases, int N, int group_size, int bits, uint16_t* out);

/* y[T, H] = moe_block(x[T, H]).  Replaces LlamaModel::moe_block (model.cpp:750-807):
 * router logits (bf16), softmax (fp32 inside, bf16 out), top-k, optional renorm,
 * gate/up/down expert products with silu(g)*u, bf16(d*score) summed over k, plus
 * bf16(sigmoid(x.wg) * shared(x)) when the layer has a shared expert. */
/* fm_moe_block for a variant of the block (fm_moe_variant above; NULL = fm_moe_block).
 * The default variant runs fm_moe_block itself; the others run the GEMV expert path at
 * every batch size (correct at any size, not tuned for prefill).  No reference
 * interface is replaced: NemotronHModel::moe_block (nemotron_h.cpp:1010-1106) is what
 * a caller would switch. */
FM_API int fm_moe_block_variant(fm_handle* h, const fm_moe_config* cfg, const fm_moe_variant* v,
                                const fm_moe_weights* w, const uint16_t* x, int64_t T, uint16_t* y,
                                const fm_moe_outputs* outs);

FM_API int fm_moe_block(fm_handle* h, const fm_moe_config* cfg, const fm_moe_weights* w, const uint16_t* x,
                 int64_t T, uint16_t* y, const fm_moe_outputs* outs);

/* fm_moe_block without a handle and without any device allocation.  No counterpart in
 * the reference (MLX allocates its own buffers).  It is for callers that cannot let a
 * library allocate device memory: runtimes whose memory planner or caching allocator
 * owns all device memory after start-up, and hot paths where cudaMalloc / cudaFree,
 * which synchronize the device, are not acceptable.  Same arguments and results as
 * fm_moe_block on `device` / `stream` (a cudaStream_t), but every call uses one fixed
 * 16 MiB scratch array per GPU that the library holds from load until process exit;
 * calls that need more (the routing tables, sorted activations and combine buffers
 * grow with T) return FM_ETOOLARGE before launching anything.  For the
 * Qwen1.5-MoE-shaped layer that is a few hundred tokens, i.e. decode batches.
 * The first call on a device resolves the array's device address, queries launch
 * parameters and synchronizes the device once; make that first call before any stream
 * capture (a first call on a capturing stream returns FM_EINVAL and leaves the capture
 * intact).  If that set-up fails on a CUDA call (FM_ECUDA), the next call tries it
 * again; a device that is not a B200 (FM_EUNSUPPORTED) stays refused for the life of
 * the process.  All calls share the
 * array: calls whose execution overlaps on the GPU (other streams, other threads) race
 * and must be serialized by the caller.  Device-side failures (a bounded wait that ran
 * out) are not reported by this entry point; fm_moe_block + fm_sync_status report them. */
FM_API int fm_moe_block_noalloc(int device, void* stream, const fm_moe_config* cfg, const fm_moe_weights* w,
                                const uint16_t* x, int64_t T, uint16_t* y);

/* Decoder ops -------------------------------------------------------------------
 * The rest of the reference's decoder layer (LlamaModel::transformer_block,
 * model.cpp:813-839, with attention 542-643), so a whole layer runs on this library.
 * Activations are token-major bf16 rows, 16-byte aligned; T = B * L tokens, token
 * t = b * L + l.  Same stream ordering and status codes as the operators above. */

/* out[N, K] = dequantize(w, scales, biases) in bf16 (bf16(fma(s, q, b))).  Replaces
 * mx::dequantize, used at load for the embedding table (model.cpp:216-230). */
FM_API int fm_dequantize(fm_handle* h, const uint32_t* w, const uint16_t* scales, const uint16_t* biases, int64_t N,
                         int K, int group_size, int bits, uint16_t* out);

/* y[t] = table[ids[t]] ([V, H] bf16 table).  Replaces mx::take(table, ids, 0)
 * (model.cpp:490-496).  An id outside [0, V) gives a zero row and FM_EDEVICE at the next
 * fm_sync_status. */
FM_API int fm_embed(fm_handle* h, const uint16_t* table, int64_t V, int H, const int32_t* ids, int64_t T,
                    uint16_t* y);

/* y = rms_norm(h) * weight with h = x + residual (residual NULL: h = x), both [T, H];
 * h is also written to h_out when it is not NULL (h_out may be x).  Replaces mx::add
 * (model.cpp:824, 838) followed by mx::fast::rms_norm (486-488): h = bf16(x + r),
 * n = 1/sqrt(mean_fp32(h^2) + eps), y = bf16(bf16(h * n) * weight).  H % 8 == 0. */
FM_API int fm_rms_norm(fm_handle* h, const uint16_t* x, const uint16_t* residual, const uint16_t* weight, int64_t T,
                       int H, float eps, uint16_t* h_out, uint16_t* y);

typedef struct fm_attn_config {
  int n_heads;       /* num_attention_heads */
  int n_kv_heads;    /* num_key_value_heads (divides n_heads) */
  int head_dim;      /* 64 or 128 */
  int max_len;       /* positions per (sequence, kv head) in the cache */
  float rope_theta;  /* RoPE base (traditional = false, scale 1) */
  float scale;       /* softmax scale; 0 = 1/sqrt(head_dim) */
  float norm_eps;    /* eps of the per-head q / k RMSNorm (QK-norm), when its weights are given */
  int qkv_ld;        /* elements from one token's row of q, k and v to the next when the three
                        share one buffer (the output of a fused q|k|v projection; a multiple
                        of 8); 0 = separate packed buffers */
} fm_attn_config;

/* The attention step of a layer after its q/k/v projections (model.cpp:560-635): bias
 * adds (biases may be NULL), the per-head RMSNorm of q and k over head_dim when q_norm /
 * k_norm [head_dim] are given (QK-norm, model.cpp:573-581), RoPE at positions offset + l,
 * k / v written into the caches
 * [B, n_kv_heads, max_len, head_dim] at [offset, offset + L) (mx::slice_update), and
 * scaled dot-product attention of the L queries over positions [0, offset + l] (causal;
 * mx::fast::scaled_dot_product_attention) into out [T, n_heads*head_dim].  q [T,
 * n_heads*head_dim] is overwritten with its rotated rows; k, v are [T,
 * n_kv_heads*head_dim] (with qkv_ld > 0: rows qkv_ld apart, e.g. q, k, v at columns 0,
 * n_heads*head_dim and (n_heads + n_kv_heads)*head_dim of one [T, qkv_ld] buffer).  Every sequence of the batch is at the same offset, as in the
 * reference (model.cpp:594-606). */
FM_API int fm_attention(fm_handle* h, const fm_attn_config* cfg, uint16_t* q, const uint16_t* k, const uint16_t* v,
                        const uint16_t* q_bias, const uint16_t* k_bias, const uint16_t* v_bias, const uint16_t* q_norm,
                        const uint16_t* k_norm, uint16_t* cache_k, uint16_t* cache_v, int B, int L, int offset,
                        uint16_t* out);

/* out = swiglu(gate, up) elementwise over n values: silu(g) * u with bf16 rounding after
 * every op, the compiled swiglu of model.cpp:14-25, for dense MLP layers (model.cpp:645-656). */
FM_API int fm_swiglu(fm_handle* h, const uint16_t* gate, const uint16_t* up, int64_t n, uint16_t* out);

/* ids[t] = argmax over logits[t, 0:V) (bf16), the first index among equal maxima.
 * Replaces sample_token at temperature 0, mx::argmax(logits, -1) (sampling.cpp:5-7). */
FM_API int fm_argmax(fm_handle* h, const uint16_t* logits, int64_t T, int64_t V, int32_t* ids);

/* Expert parallelism ------------------------------------------------------------
 * No reference counterpart: the reference runs the whole MoE layer in one process
 * (model.cpp:750-807).  These calls split fm_moe_block into the three stages of an
 * expert-parallel layer so that the caller's collectives (NCCL all-to-all over NVLink)
 * move the rows between them.  Rank r of world W owns the contiguous experts
 * [first, first + count) given by fm_ep_range (the first E % W ranks one more).
 *
 *   fm_ep_dispatch   route this rank's T tokens (router, softmax, top-k, stable
 *                    expert-major order); fills expert_counts[E] (host, the call
 *                    synchronizes the stream) and points *send_rows at the T*k token rows
 *                    (device, H bf16 each, within-8 pair order) in expert-major order, so
 *                    the rows for each owner are contiguous.  Valid until the next dispatch.
 *   fm_ep_experts    owner side: recv_rows holds the rows received from every source rank
 *                    in source order, each source's rows in expert-major order;
 *                    recv_counts[W * count] (host) gives the rows per (source, local
 *                    expert).  w holds the router / shared tensors and the stacked weights
 *                    of the local experts only.  Writes bf16(d) per received row to d_rows
 *                    (same order) and runs this rank's shared expert over its own tokens.
 *   fm_ep_combine    token side: ret_rows holds the d rows returned by the owners in the
 *                    order fm_ep_dispatch sent them; y = the MoE block output (sum over j
 *                    of bf16(d * score) in order j = 0..k-1, plus the gated shared expert).
 * The three calls on one handle form one layer and must come in this order. */
FM_API int fm_ep_range(int num_experts, int rank, int world, int* first, int* count);
FM_API int fm_ep_set(fm_handle* h, int rank, int world);
FM_API int fm_ep_dispatch(fm_handle* h, const fm_moe_config* cfg, const fm_moe_weights* w, const uint16_t* x,
                          int64_t T, int32_t* expert_counts, const uint16_t** send_rows);
FM_API int fm_ep_experts(fm_handle* h, const fm_moe_config* cfg, const fm_moe_weights* w, const uint16_t* recv_rows,
                         const int32_t* recv_counts, uint16_t* d_rows);
FM_API int fm_ep_combine(fm_handle* h, const fm_moe_config* cfg, const uint16_t* ret_rows, uint16_t* y);

/* Expert parallelism over peer memory: the same layer with no host synchronization and
 * no collective library.  Every rank of the group (one process per GPU of one NVLink
 * domain, at most 8) owns a device region of identical layout, exported by CUDA IPC;
 * the kernels write the routed rows straight into their owners' regions and the d rows
 * back into their token ranks' regions, and order the steps with epoch flags in the
 * regions (bounded device-side waits: a rank that does not take part makes the others'
 * calls fail with FM_ETIMEOUT at fm_sync_status, after which the group must close and
 * reallocate its regions).
 *
 *   fm_ep_p2p_alloc    after fm_ep_set: allocate this rank's region for up to max_tokens
 *                      tokens per call with cfg's hidden / experts / top_k (identical on
 *                      every rank) and write its 64-byte CUDA IPC handle to ipc_handle_out.
 *   fm_ep_p2p_open     ipc_handles = the W handles in rank order (this rank's own slot is
 *                      ignored): map every peer's region.  Call after every rank's alloc.
 *   fm_ep_p2p_forward  one layer on this rank's T tokens (T <= max_tokens, may be 0): y =
 *                      the MoE block output, as fm_moe_block over the whole model's
 *                      experts.  Asynchronous on the handle's stream; every rank of the
 *                      group must make the same sequence of calls.
 *   fm_ep_p2p_close    unmap the peers' regions and free this rank's (also done by
 *                      fm_destroy).  Call on every rank only after every rank's last
 *                      forward completed (a barrier after a stream synchronize). */
FM_API int fm_ep_p2p_alloc(fm_handle* h, const fm_moe_config* cfg, int64_t max_tokens, void* ipc_handle_out);
FM_API int fm_ep_p2p_open(fm_handle* h, const void* ipc_handles);
FM_API int fm_ep_p2p_forward(fm_handle* h, const fm_moe_config* cfg, const fm_moe_weights* w, const uint16_t* x,
                             int64_t T, uint16_t* y);
FM_API int fm_ep_p2p_close(fm_handle* h);

#ifdef __cplusplus
}
#endif

#endif /* FLASHMOE_H_ */
