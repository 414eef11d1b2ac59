// decoder.cpp -- see decoder.hpp.
#include "decoder.hpp"

#include <cmath>
#include <stdexcept>

#include "checkpoint.hpp"
#include "moe_model.hpp"

namespace flashmoe {

namespace {

std::runtime_error err(const std::string& what) { return std::runtime_error(what); }

}  // namespace

Decoder::Decoder(const fmh_decoder_config& cfg, const fmh_weights& w, int device, int max_batch, int max_len,
                 void* stream)
    : cfg_(cfg), w_(w), device_(device), max_batch_(max_batch), max_len_(max_len),
      stream_(static_cast<cudaStream_t>(stream)), bufs_(device) {
  if (!w.layers && cfg.layers > 0) throw Error(FM_EINVAL, "null layer table");
  layers_.assign(w.layers, w.layers + cfg.layers);
  w_.layers = layers_.data();
  validate();
  cuda_check(cudaSetDevice(device_), "cudaSetDevice");
  handle_ = Handle(device_, stream);
  attn_.n_heads = cfg_.n_heads;
  attn_.n_kv_heads = cfg_.n_kv_heads;
  attn_.head_dim = cfg_.head_dim;
  attn_.max_len = max_len_;
  attn_.rope_theta = cfg_.rope_theta;
  attn_.scale = 0.f;
  attn_.norm_eps = cfg_.rms_eps;  // QK-norm uses the model's rms_norm_eps (model.cpp:486-488)
  const int64_t tokens = static_cast<int64_t>(max_batch_) * max_len_;
  const int64_t H = cfg_.hidden, QD = static_cast<int64_t>(cfg_.n_heads) * cfg_.head_dim,
                KVD = static_cast<int64_t>(cfg_.n_kv_heads) * cfg_.head_dim;
  auto bf = [&](int64_t n) { return static_cast<uint16_t*>(bufs_.alloc(static_cast<size_t>(n) * 2)); };
  // Each layer's q, k and v projections as one [QD + 2 KVD, H] matrix (their rows, scales
  // and biases concatenated): one fm_linear per layer instead of three, q, k and v side by
  // side in each output row.  The rows of a quantized linear do not interact and the
  // direct path never splits K, so the fused output equals the three projections' bit
  // for bit.  A layer whose three matrices disagree on having biases stays separate.
  const int64_t W = QD + 2 * KVD, kw = H / 8, gpr = H / cfg_.group_size;
  const bool fusable = cfg_.group_size > 0 && H % cfg_.group_size == 0 && H % 8 == 0;
  bool any_fused = false, any_split = false;
  qkv_.assign(cfg_.layers, fm_qweight{nullptr, nullptr, nullptr});
  for (int li = 0; li < cfg_.layers; ++li) {
    const fmh_layer& l = layers_[li];
    const bool nb = !l.q.biases;
    if (!fusable || !l.q.scales || !l.k.scales || !l.v.scales || !l.k.biases != nb || !l.v.biases != nb) {
      any_split = true;
      continue;
    }
    // q, k and v already side by side (codes, scales and biases each one [QD + 2 KVD]-row
    // block, as open() uploads them): used in place, no copy
    const bool adjacent = l.k.w == l.q.w + QD * kw && l.v.w == l.k.w + KVD * kw &&
                          l.k.scales == l.q.scales + QD * gpr && l.v.scales == l.k.scales + KVD * gpr &&
                          (nb || (l.k.biases == l.q.biases + QD * gpr && l.v.biases == l.k.biases + KVD * gpr));
    if (adjacent) {
      qkv_[li] = fm_qweight{l.q.w, l.q.scales, l.q.biases};
      any_fused = true;
      continue;
    }
    auto* w = static_cast<uint32_t*>(bufs_.alloc(static_cast<size_t>(W * kw) * 4));
    uint16_t* sc = bf(W * gpr);
    uint16_t* bi = nb ? nullptr : bf(W * gpr);
    const fm_qweight* parts[3] = {&l.q, &l.k, &l.v};
    const int64_t rows[3] = {QD, KVD, KVD};
    int64_t r0 = 0;
    for (int i = 0; i < 3; ++i) {
      cuda_check(cudaMemcpyAsync(w + r0 * kw, parts[i]->w, static_cast<size_t>(rows[i] * kw) * 4,
                                 cudaMemcpyDeviceToDevice, stream_), "cudaMemcpyAsync qkv codes");
      cuda_check(cudaMemcpyAsync(sc + r0 * gpr, parts[i]->scales, static_cast<size_t>(rows[i] * gpr) * 2,
                                 cudaMemcpyDeviceToDevice, stream_), "cudaMemcpyAsync qkv scales");
      if (bi)
        cuda_check(cudaMemcpyAsync(bi + r0 * gpr, parts[i]->biases, static_cast<size_t>(rows[i] * gpr) * 2,
                                   cudaMemcpyDeviceToDevice, stream_), "cudaMemcpyAsync qkv biases");
      r0 += rows[i];
    }
    qkv_[li] = fm_qweight{w, sc, bi};
    any_fused = true;
  }
  attn_qkv_ = attn_;
  attn_qkv_.qkv_ld = static_cast<int>(W);
  x_ = bf(tokens * H);
  normed_ = bf(tokens * H);
  o_ = bf(tokens * H);
  mlp_ = bf(tokens * H);
  attn_out_ = bf(tokens * QD);
  if (any_fused) qkv_out_ = bf(tokens * W);
  if (any_split) {
    q_ = bf(tokens * QD);
    k_ = bf(tokens * KVD);
    v_ = bf(tokens * KVD);
  }
  bool dense = false, moe = false;
  for (const auto& l : layers_) (l.is_moe ? moe : dense) = true;
  if (dense) {
    gate_ = bf(tokens * cfg_.intermediate);
    up_ = bf(tokens * cfg_.intermediate);
  }
  last_ = bf(static_cast<int64_t>(max_batch_) * H);
  logits_ = bf(static_cast<int64_t>(max_batch_) * cfg_.vocab);
  tok_ = static_cast<int32_t*>(bufs_.alloc(sizeof(int32_t) * 2 * static_cast<size_t>(tokens)));
  gen_ = static_cast<int32_t*>(bufs_.alloc(sizeof(int32_t) * static_cast<size_t>(tokens)));
  gen_cap_ = tokens;
  const int64_t cache = static_cast<int64_t>(max_batch_) * cfg_.n_kv_heads * max_len_ * cfg_.head_dim;
  for (int l = 0; l < cfg_.layers; ++l) {
    cache_k_.push_back(bf(cache));
    cache_v_.push_back(bf(cache));
  }
  if (moe) handle_.reserve(cfg_.moe, tokens);
}

Decoder::~Decoder() {
  if (handle_) fm_sync_status(handle_.get());  // nothing may still read the buffers or weights
}

void Decoder::validate() const {
  const fmh_decoder_config& c = cfg_;
  if (c.hidden <= 0 || c.layers <= 0 || c.n_heads <= 0 || c.n_kv_heads <= 0 || c.n_heads % c.n_kv_heads ||
      c.vocab <= 0 || !(c.rms_eps >= 0.f) || !(c.rope_theta > 0.f))
    throw Error(FM_EINVAL, "bad decoder config");
  if (c.head_dim != 64 && c.head_dim != 128) throw Error(FM_EUNSUPPORTED, "head_dim must be 64 or 128");
  if (c.bits != 4) throw Error(FM_EUNSUPPORTED, "only 4-bit affine projections are implemented");
  if (max_batch_ <= 0 || max_len_ <= 0) throw Error(FM_EINVAL, "max_batch and max_len must be positive");
  if (!w_.embed_table || !w_.norm) throw Error(FM_EINVAL, "embedding table or final norm missing");
  if (c.tie_word_embeddings ? !w_.embed_q.w : !w_.lm_head.w) throw Error(FM_EINVAL, "lm_head weights missing");
  for (int i = 0; i < c.layers; ++i) {
    const fmh_layer& l = layers_[i];
    if (!l.in_norm || !l.post_norm || !l.q.w || !l.k.w || !l.v.w || !l.o.w)
      throw Error(FM_EINVAL, "layer " + std::to_string(i) + ": attention weights or norms missing");
    if (!l.is_moe && (!l.gate.w || !l.up.w || !l.down.w || c.intermediate <= 0))
      throw Error(FM_EINVAL, "layer " + std::to_string(i) + ": dense MLP weights missing");
    if (l.is_moe && c.moe.hidden != c.hidden) throw Error(FM_EINVAL, "MoE hidden size differs from the model's");
  }
}

// the dense projections (q, k, v, o, dense MLP, lm_head): LlamaModel::linear_fast
void Decoder::qmm(const uint16_t* x, int64_t M, int K, const fm_qweight& w, int N, uint16_t* out) {
  handle_.check(fm_linear(handle_.get(), x, M, K, w.w, w.scales, w.biases, N, cfg_.group_size, cfg_.bits, out));
}

void Decoder::forward(const int32_t* ids, int B, int L, int32_t* next_ids) {
  if (B <= 0 || L <= 0 || B > max_batch_) throw Error(FM_EINVAL, "B must be in [1, max_batch], L positive");
  if (static_cast<int64_t>(offset_) + L > max_len_) throw Error(FM_EINVAL, "offset + L exceeds max_len");
  if (!ids || !next_ids) throw Error(FM_EINVAL, "null ids");
  fm_handle* h = handle_.get();
  const int64_t T = static_cast<int64_t>(B) * L;
  const int H = cfg_.hidden, QD = cfg_.n_heads * cfg_.head_dim, KVD = cfg_.n_kv_heads * cfg_.head_dim;
  const float eps = cfg_.rms_eps;
  handle_.check(fm_embed(h, w_.embed_table, cfg_.vocab, H, ids, T, x_));
  handle_.check(fm_rms_norm(h, x_, nullptr, layers_[0].in_norm, T, H, eps, nullptr, normed_));
  for (int li = 0; li < cfg_.layers; ++li) {
    const fmh_layer& l = layers_[li];
    if (qkv_[li].w) {
      qmm(normed_, T, H, qkv_[li], QD + 2 * KVD, qkv_out_);
      handle_.check(fm_attention(h, &attn_qkv_, qkv_out_, qkv_out_ + QD, qkv_out_ + QD + KVD, l.q_bias, l.k_bias,
                                 l.v_bias, l.q_norm, l.k_norm, cache_k_[li], cache_v_[li], B, L, offset_, attn_out_));
    } else {
      qmm(normed_, T, H, l.q, QD, q_);
      qmm(normed_, T, H, l.k, KVD, k_);
      qmm(normed_, T, H, l.v, KVD, v_);
      handle_.check(fm_attention(h, &attn_, q_, k_, v_, l.q_bias, l.k_bias, l.v_bias, l.q_norm, l.k_norm,
                                 cache_k_[li], cache_v_[li], B, L, offset_, attn_out_));
    }
    qmm(attn_out_, T, QD, l.o, H, o_);
    // h = x + attention; normed = rms_norm(h, post_attention_layernorm)
    handle_.check(fm_rms_norm(h, x_, o_, l.post_norm, T, H, eps, x_, normed_));
    if (l.is_moe) {
      handle_.check(fm_moe_block(h, &cfg_.moe, &l.moe, normed_, T, mlp_, nullptr));
    } else {
      const int I = cfg_.intermediate;
      qmm(normed_, T, H, l.gate, I, gate_);
      qmm(normed_, T, H, l.up, I, up_);
      handle_.check(fm_swiglu(h, gate_, up_, T * I, gate_));
      qmm(gate_, T, I, l.down, H, mlp_);
    }
    // x = h + mlp; normed = rms_norm(x) with the next layer's input norm (or the final norm)
    const uint16_t* next_w = li + 1 < cfg_.layers ? layers_[li + 1].in_norm : w_.norm;
    handle_.check(fm_rms_norm(h, x_, mlp_, next_w, T, H, eps, x_, normed_));
  }
  // each sequence's last position: rows b * L + L - 1
  cuda_check(cudaMemcpy2DAsync(last_, static_cast<size_t>(H) * 2, normed_ + static_cast<int64_t>(L - 1) * H,
                               static_cast<size_t>(L) * H * 2, static_cast<size_t>(H) * 2, B, cudaMemcpyDeviceToDevice,
                               stream_),
             "cudaMemcpy2DAsync");
  qmm(last_, B, H, cfg_.tie_word_embeddings ? w_.embed_q : w_.lm_head, cfg_.vocab, logits_);
  handle_.check(fm_argmax(h, logits_, B, cfg_.vocab, next_ids));
  offset_ += L;
}

void Decoder::copy_logits(uint16_t* dst, int B) const {
  if (B > max_batch_) throw Error(FM_EINVAL, "B exceeds max_batch");
  cuda_check(cudaMemcpyAsync(dst, logits_, sizeof(uint16_t) * static_cast<size_t>(B) * cfg_.vocab,
                             cudaMemcpyDeviceToDevice, stream_),
             "cudaMemcpyAsync logits");
}

std::vector<int32_t> Decoder::generate(const int32_t* prompt, int B, int L, int steps) {
  if (steps <= 0) return {};
  if (static_cast<int64_t>(L) + steps - 1 > max_len_) throw Error(FM_EINVAL, "prompt + steps exceed max_len");
  if (static_cast<int64_t>(steps) * B > gen_cap_) throw Error(FM_EINVAL, "too many steps");
  reset();
  int32_t* in = tok_;
  int32_t* nxt = tok_ + static_cast<int64_t>(max_batch_) * max_len_;
  cuda_check(cudaMemcpyAsync(in, prompt, sizeof(int32_t) * B * static_cast<size_t>(L), cudaMemcpyHostToDevice,
                             stream_),
             "cudaMemcpyAsync prompt");
  forward(in, B, L, nxt);
  cuda_check(cudaMemcpyAsync(gen_, nxt, sizeof(int32_t) * B, cudaMemcpyDeviceToDevice, stream_), "cudaMemcpyAsync");
  for (int s = 1; s < steps; ++s) {
    std::swap(in, nxt);
    forward(in, B, 1, nxt);
    cuda_check(cudaMemcpyAsync(gen_ + static_cast<int64_t>(s) * B, nxt, sizeof(int32_t) * B, cudaMemcpyDeviceToDevice,
                               stream_),
               "cudaMemcpyAsync");
  }
  std::vector<int32_t> by_step(static_cast<size_t>(steps) * B), out(by_step.size());
  cuda_check(cudaMemcpyAsync(by_step.data(), gen_, by_step.size() * sizeof(int32_t), cudaMemcpyDeviceToHost, stream_),
             "cudaMemcpyAsync tokens");
  sync();
  for (int s = 0; s < steps; ++s)
    for (int b = 0; b < B; ++b) out[static_cast<size_t>(b) * steps + s] = by_step[static_cast<size_t>(s) * B + b];
  return out;
}

// ---------------------------------------------------------------- loading a model directory
DecoderPlan plan_decoder(const Checkpoint& ck) {
  const ModelConfig& c = ck.config();
  if (c.sigmoid_routed()) throw err("Nemotron-H (hybrid) models are not decoded by this class");
  if (c.quant_bits != 4) throw err("only 4-bit affine checkpoints are implemented");
  DecoderPlan p;
  fmh_decoder_config& cfg = p.cfg;
  cfg.hidden = c.hidden_size;
  cfg.layers = c.num_hidden_layers;
  cfg.n_heads = c.num_attention_heads;
  cfg.n_kv_heads = c.num_key_value_heads;
  cfg.head_dim = c.attn_head_dim();
  cfg.vocab = c.vocab_size;
  cfg.intermediate = c.intermediate_size;
  cfg.rope_theta = c.rope_theta;
  cfg.rms_eps = c.rms_norm_eps;
  cfg.group_size = c.quant_group_size;
  cfg.bits = c.quant_bits;
  cfg.tie_word_embeddings = c.tie_word_embeddings ? 1 : 0;
  cfg.moe = c.moe_config();
  const int64_t H = cfg.hidden, QD = static_cast<int64_t>(cfg.n_heads) * cfg.head_dim,
                KVD = static_cast<int64_t>(cfg.n_kv_heads) * cfg.head_dim;
  const int per_word = 32 / cfg.bits;
  auto qview = [&](const std::string& prefix, int64_t n, int64_t k) {
    QView q;
    q.w = &ck.get(prefix + ".weight", "U32");
    q.s = &ck.get(prefix + ".scales", "BF16");
    if (q.w->shape != std::vector<int64_t>{n, k / per_word} ||
        q.s->shape != std::vector<int64_t>{n, k / cfg.group_size})
      throw err(prefix + ": shape differs from the config's (" + std::to_string(n) + ", " + std::to_string(k) + ")");
    if (ck.has(prefix + ".biases")) {
      q.b = &ck.get(prefix + ".biases", "BF16");
      if (q.b->shape != q.s->shape) throw err(prefix + ".biases: shape differs from the scales'");
    }
    return q;
  };
  auto vview = [&](const std::string& key, int64_t n) {
    const TensorView* t = &ck.get(key, "BF16");
    if (t->numel() != n) throw err(key + ": " + std::to_string(t->numel()) + " values, expected " + std::to_string(n));
    return t;
  };
  auto vview_opt = [&](const std::string& key, int64_t n) -> const TensorView* {
    return ck.has(key) ? vview(key, n) : nullptr;
  };
  if (ck.has("embed_tokens.scales")) {
    p.embed = qview("embed_tokens", cfg.vocab, H);
  } else {
    if (cfg.tie_word_embeddings) throw err("a tied bf16 embedding (bf16 lm_head) is not implemented");
    p.embed_bf16 = vview("embed_tokens.weight", static_cast<int64_t>(cfg.vocab) * H);
  }
  p.norm = vview("norm.weight", H);
  if (!cfg.tie_word_embeddings) p.lm_head = qview("lm_head", cfg.vocab, H);
  p.layers.resize(cfg.layers);
  for (int i = 0; i < cfg.layers; ++i) {
    const std::string pre = "layers." + std::to_string(i);
    LayerPlan& l = p.layers[i];
    l.in_norm = vview(pre + ".input_layernorm.weight", H);
    l.post_norm = vview(pre + ".post_attention_layernorm.weight", H);
    l.q = qview(pre + ".self_attn.q_proj", QD, H);
    l.k = qview(pre + ".self_attn.k_proj", KVD, H);
    l.v = qview(pre + ".self_attn.v_proj", KVD, H);
    l.o = qview(pre + ".self_attn.o_proj", H, QD);
    l.q_bias = vview_opt(pre + ".self_attn.q_proj.bias", QD);
    l.k_bias = vview_opt(pre + ".self_attn.k_proj.bias", KVD);
    l.v_bias = vview_opt(pre + ".self_attn.v_proj.bias", KVD);
    l.q_norm = vview_opt(pre + ".self_attn.q_norm.weight", cfg.head_dim);
    l.k_norm = vview_opt(pre + ".self_attn.k_norm.weight", cfg.head_dim);
    l.is_moe = ck.has(pre + ".mlp.gate.weight");
    if (!l.is_moe) {
      l.gate = qview(pre + ".mlp.gate_proj", cfg.intermediate, H);
      l.up = qview(pre + ".mlp.up_proj", cfg.intermediate, H);
      l.down = qview(pre + ".mlp.down_proj", H, cfg.intermediate);
    }
  }
  return p;
}

std::unique_ptr<Decoder> Decoder::open(const std::string& model_dir, int device, int max_batch, int max_len,
                                       void* stream) {
  Checkpoint ck(model_dir);
  const DecoderPlan p = plan_decoder(ck);
  const fmh_decoder_config& cfg = p.cfg;
  cuda_check(cudaSetDevice(device), "cudaSetDevice");
  auto store = std::make_unique<DeviceStore>(device);
  auto up = [&](const TensorView* t) -> const void* { return t ? store->upload(t->data, t->nbytes) : nullptr; };
  auto uq = [&](const QView& q) {
    fm_qweight r{};
    r.w = static_cast<const uint32_t*>(up(q.w));
    r.scales = static_cast<const uint16_t*>(up(q.s));
    r.biases = static_cast<const uint16_t*>(up(q.b));
    return r;
  };
  // q, k and v of a layer in one allocation each for codes, scales and biases (q's rows,
  // then k's, then v's), which the decoder takes as its fused q|k|v projection without a
  // second copy; a layer whose three matrices differ in having scales or biases is
  // uploaded matrix by matrix
  auto uq3 = [&](const QView& q, const QView& k, const QView& v, fm_qweight& oq, fm_qweight& ok, fm_qweight& ov) {
    const bool all = q.w && k.w && v.w && q.s && k.s && v.s && !q.b == !k.b && !q.b == !v.b;
    if (!all) {
      oq = uq(q);
      ok = uq(k);
      ov = uq(v);
      return;
    }
    auto cat = [&](const TensorView* a, const TensorView* b, const TensorView* c, const void* (&out)[3]) {
      auto* base = static_cast<uint8_t*>(store->alloc(a->nbytes + b->nbytes + c->nbytes));
      const TensorView* parts[3] = {a, b, c};
      size_t off = 0;
      for (int i = 0; i < 3; ++i) {
        if (parts[i]->nbytes)
          cuda_check(cudaMemcpy(base + off, parts[i]->data, parts[i]->nbytes, cudaMemcpyHostToDevice), "cudaMemcpy");
        out[i] = base + off;
        off += parts[i]->nbytes;
      }
    };
    const void* pw[3];
    const void* ps[3];
    const void* pb[3] = {nullptr, nullptr, nullptr};
    cat(q.w, k.w, v.w, pw);
    cat(q.s, k.s, v.s, ps);
    if (q.b) cat(q.b, k.b, v.b, pb);
    fm_qweight* outs[3] = {&oq, &ok, &ov};
    for (int i = 0; i < 3; ++i)
      *outs[i] = fm_qweight{static_cast<const uint32_t*>(pw[i]), static_cast<const uint16_t*>(ps[i]),
                            static_cast<const uint16_t*>(pb[i])};
  };
  fmh_weights w{};
  if (p.embed.w) {  // a quantized table is dequantized once on the device (model.cpp:216-230)
    w.embed_q = uq(p.embed);
    uint16_t* table = static_cast<uint16_t*>(store->alloc(static_cast<size_t>(cfg.vocab) * cfg.hidden * 2));
    Handle tmp(device, stream);
    tmp.check(fm_dequantize(tmp.get(), w.embed_q.w, w.embed_q.scales, w.embed_q.biases, cfg.vocab, cfg.hidden,
                            cfg.group_size, cfg.bits, table));
    tmp.sync();
    w.embed_table = table;
  } else {
    w.embed_table = static_cast<const uint16_t*>(up(p.embed_bf16));
  }
  w.norm = static_cast<const uint16_t*>(up(p.norm));
  if (!cfg.tie_word_embeddings) w.lm_head = uq(p.lm_head);
  std::vector<fmh_layer> layers(cfg.layers);
  for (int i = 0; i < cfg.layers; ++i) {
    const LayerPlan& lp = p.layers[i];
    fmh_layer& l = layers[i];
    l.in_norm = static_cast<const uint16_t*>(up(lp.in_norm));
    l.post_norm = static_cast<const uint16_t*>(up(lp.post_norm));
    uq3(lp.q, lp.k, lp.v, l.q, l.k, l.v);
    l.o = uq(lp.o);
    l.q_bias = static_cast<const uint16_t*>(up(lp.q_bias));
    l.k_bias = static_cast<const uint16_t*>(up(lp.k_bias));
    l.v_bias = static_cast<const uint16_t*>(up(lp.v_bias));
    l.q_norm = static_cast<const uint16_t*>(up(lp.q_norm));
    l.k_norm = static_cast<const uint16_t*>(up(lp.k_norm));
    l.is_moe = lp.is_moe ? 1 : 0;
    if (lp.is_moe) {
      l.moe = upload_moe_layer(*store, ck.moe_layer(i), nullptr);
    } else {
      l.gate = uq(lp.gate);
      l.up = uq(lp.up);
      l.down = uq(lp.down);
    }
  }
  w.layers = layers.data();
  auto d = std::make_unique<Decoder>(cfg, w, device, max_batch, max_len, stream);
  d->owned_ = std::move(store);
  return d;
}

}  // namespace flashmoe

// ---------------------------------------------------------------- C interface (fmh.h)
struct fmh_decoder {
  std::unique_ptr<flashmoe::Decoder> d;
  std::string last_error;
};

namespace {

template <class F>
int guarded(fmh_decoder* d, F&& f) {
  try {
    f();
    return FM_OK;
  } catch (const flashmoe::Error& e) {
    if (d) d->last_error = e.what();
    return e.status();
  } catch (const std::exception& e) {
    if (d) d->last_error = e.what();
    return FM_EINVAL;
  }
}

}  // namespace

extern "C" {

int fmh_decoder_create(const fmh_decoder_config* cfg, const fmh_weights* w, int device, int max_batch, int max_len,
                       void* stream, fmh_decoder** out) {
  if (!cfg || !w || !out) return FM_EINVAL;
  *out = nullptr;
  auto box = std::make_unique<fmh_decoder>();
  const int rc = guarded(box.get(), [&] {
    box->d = std::make_unique<flashmoe::Decoder>(*cfg, *w, device, max_batch, max_len, stream);
  });
  if (rc == FM_OK) *out = box.release();
  return rc;
}

int fmh_decoder_open(const char* model_dir, int device, int max_batch, int max_len, void* stream, fmh_decoder** out) {
  if (!model_dir || !out) return FM_EINVAL;
  *out = nullptr;
  auto box = std::make_unique<fmh_decoder>();
  const int rc = guarded(box.get(), [&] { box->d = flashmoe::Decoder::open(model_dir, device, max_batch, max_len, stream); });
  if (rc == FM_OK) *out = box.release();
  return rc;
}

void fmh_decoder_close(fmh_decoder* d) { delete d; }

const char* fmh_last_error(const fmh_decoder* d) { return d ? d->last_error.c_str() : "null decoder"; }

int fmh_decoder_forward(fmh_decoder* d, const int32_t* ids, int B, int L, int32_t* next_ids) {
  if (!d || !d->d) return FM_EINVAL;
  return guarded(d, [&] { d->d->forward(ids, B, L, next_ids); });
}

const uint16_t* fmh_decoder_logits(const fmh_decoder* d) { return d && d->d ? d->d->logits() : nullptr; }

int fmh_decoder_copy_logits(fmh_decoder* d, uint16_t* dst, int B) {
  if (!d || !d->d || !dst || B < 0) return FM_EINVAL;
  return guarded(d, [&] { d->d->copy_logits(dst, B); });
}

int fmh_decoder_offset(const fmh_decoder* d) { return d && d->d ? d->d->offset() : -1; }

int fmh_decoder_reset(fmh_decoder* d) {
  if (!d || !d->d) return FM_EINVAL;
  d->d->reset();
  return FM_OK;
}

int fmh_decoder_sync(fmh_decoder* d) {
  if (!d || !d->d) return FM_EINVAL;
  return guarded(d, [&] { d->d->sync(); });
}

fm_handle* fmh_decoder_handle(fmh_decoder* d) { return d && d->d ? d->d->handle().get() : nullptr; }

int fmh_decoder_generate(fmh_decoder* d, const int32_t* prompt, int B, int L, int steps, int32_t* out) {
  if (!d || !d->d || !prompt || !out) return FM_EINVAL;
  return guarded(d, [&] {
    const std::vector<int32_t> toks = d->d->generate(prompt, B, L, steps);
    std::copy(toks.begin(), toks.end(), out);
  });
}

}  // extern "C"
