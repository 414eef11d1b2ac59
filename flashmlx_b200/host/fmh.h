/* fmh.h -- C interface of the C++ host layer's decoder (libflashmoe_host.so), for
 * callers that are not C++ (the Python tests and bench bind it with ctypes).
 *
 * The decoder is the reference's LlamaModel forward (server/src/model.cpp: embed
 * 490-496, transformer_block 813-839, attention 542-643, moe_block 750-807, lm_head
 * 499-520) with greedy sampling (sampling.cpp:5-7), every op a libflashmoe call on one
 * stream.  Weights are device pointers in MLX's layout; the caller owns them (or
 * fmh_decoder_open loads and owns them).  All entry points return an fm_status. */
#ifndef FLASHMOE_HOST_H_
#define FLASHMOE_HOST_H_

#include <stdint.h>

#include "flashmoe.h"

#ifdef __cplusplus
extern "C" {
#endif

typedef struct fmh_decoder fmh_decoder;

typedef struct fmh_decoder_config {
  int hidden;               /* hidden_size */
  int layers;               /* num_hidden_layers */
  int n_heads;              /* num_attention_heads */
  int n_kv_heads;           /* num_key_value_heads */
  int head_dim;             /* 64 or 128 */
  int vocab;                /* vocab_size */
  int intermediate;         /* intermediate_size of dense MLP layers */
  float rope_theta;
  float rms_eps;
  int group_size;           /* quantization of every projection (4-bit affine) */
  int bits;
  int tie_word_embeddings;  /* lm_head = the quantized embedding */
  fm_moe_config moe;        /* the MoE layers' shape */
} fmh_decoder_config;

typedef struct fmh_layer {
  const uint16_t* in_norm;    /* input_layernorm.weight [H] */
  const uint16_t* post_norm;  /* post_attention_layernorm.weight [H] */
  fm_qweight q, k, v, o;      /* self_attn.{q,k,v,o}_proj */
  const uint16_t* q_bias;     /* self_attn.{q,k,v}_proj.bias, NULL if absent */
  const uint16_t* k_bias;
  const uint16_t* v_bias;
  const uint16_t* q_norm;     /* self_attn.{q,k}_norm.weight [head_dim] (QK-norm), NULL if absent */
  const uint16_t* k_norm;
  int is_moe;                 /* layer_is_moe_ (model.cpp:253-266) */
  fm_moe_weights moe;         /* the stacked MoE weights when is_moe */
  fm_qweight gate, up, down;  /* the dense MLP otherwise */
} fmh_layer;

typedef struct fmh_weights {
  const uint16_t* embed_table;  /* [V, H] bf16 (the dequantized embed_tokens) */
  fm_qweight embed_q;           /* the quantized embed_tokens (lm_head when tied) */
  const uint16_t* norm;         /* norm.weight [H] */
  fm_qweight lm_head;           /* lm_head.* when not tied */
  const fmh_layer* layers;      /* [layers] */
} fmh_weights;

/* A decoder over caller-owned device weights, with KV caches for max_batch sequences of
 * max_len positions; the weight tables are copied, the weights are not. */
int fmh_decoder_create(const fmh_decoder_config* cfg, const fmh_weights* w, int device, int max_batch, int max_len,
                       void* stream, fmh_decoder** out);
/* The same over an MLX-format model directory, loaded and uploaded (owned by the decoder). */
int fmh_decoder_open(const char* model_dir, int device, int max_batch, int max_len, void* stream, fmh_decoder** out);
void fmh_decoder_close(fmh_decoder* d);
const char* fmh_last_error(const fmh_decoder* d);

/* One forward over ids [B, L] (device int32) at the current cache offset: fills the caches
 * at [offset, offset + L), writes the greedy next token of each sequence to next_ids [B]
 * (device) and advances the offset by L.  Asynchronous on the decoder's stream. */
int fmh_decoder_forward(fmh_decoder* d, const int32_t* ids, int B, int L, int32_t* next_ids);
/* logits [B, vocab] bf16 (device) of the last forward's final positions */
const uint16_t* fmh_decoder_logits(const fmh_decoder* d);
/* copies the first B rows of those logits to dst (device), ordered on the decoder's stream */
int fmh_decoder_copy_logits(fmh_decoder* d, uint16_t* dst, int B);
int fmh_decoder_offset(const fmh_decoder* d);
/* starts new sequences (offset 0) */
int fmh_decoder_reset(fmh_decoder* d);
/* waits for the stream; FM_EDEVICE etc. as fm_sync_status */
int fmh_decoder_sync(fmh_decoder* d);
/* the libflashmoe handle the decoder's calls run on (fm_profile_enable / _report) */
fm_handle* fmh_decoder_handle(fmh_decoder* d);
/* Greedy generation from host buffers: prompt [B, L] -> out [B, steps] (the first token
 * from the prompt's forward, then steps - 1 single-token forwards).  Resets first. */
int fmh_decoder_generate(fmh_decoder* d, const int32_t* prompt, int B, int L, int steps, int32_t* out);

#ifdef __cplusplus
}
#endif

#endif /* FLASHMOE_HOST_H_ */
