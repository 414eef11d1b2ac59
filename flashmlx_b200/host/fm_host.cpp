// fm_host -- command-line driver of the C++ host layer (checkpoint.hpp, moe_model.hpp).
//
//   fm_host inspect DIR                  the config and MoE layers of a model directory (JSON)
//   fm_host dump DIR LAYER OUT           one MoE layer's stacked host arrays as raw
//                                        little-endian files OUT/<name>.bin + OUT/manifest.json
//   fm_host run DIR LAYER X T Y [DEV]    y = moe_block(x, LAYER) on the GPU: X holds T x hidden
//                                        bf16 (raw), Y receives the same
//   fm_host check-decoder DIR            the decoder layout of a model directory, checked (JSON)
//   fm_host generate DIR P B L STEPS OUT [DEV]
//                                        greedy decoding with the whole model (Decoder): P
//                                        holds B x L int32 prompt tokens, OUT receives
//                                        B x STEPS int32 tokens
//
// Exit status: 0 ok; 2 usage; 3 a libflashmoe status (the status name and message on
// stderr, "fm_status <n>" on the first line); 4 any other error.
#include <cuda_runtime.h>

#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <fstream>
#include <iostream>
#include <sstream>
#include <string>
#include <vector>

#include "checkpoint.hpp"
#include "decoder.hpp"
#include "moe_model.hpp"

using namespace flashmoe;

namespace {

std::string q(const std::string& s) {
  std::string r = "\"";
  for (char c : s) {
    if (c == '"' || c == '\\') r += '\\';
    r += c;
  }
  return r + "\"";
}

std::string shape_json(const std::vector<int64_t>& s) {
  std::string r = "[";
  for (size_t i = 0; i < s.size(); ++i) r += (i ? "," : "") + std::to_string(s[i]);
  return r + "]";
}

template <typename T>
void write_raw(const std::string& path, const std::vector<T>& v) {
  std::ofstream f(path, std::ios::binary);
  if (!f) throw std::runtime_error(path + ": cannot write");
  f.write(reinterpret_cast<const char*>(v.data()), static_cast<std::streamsize>(v.size() * sizeof(T)));
  if (!f) throw std::runtime_error(path + ": write failed");
}

int inspect(const std::string& dir) {
  Checkpoint ck(dir);
  const ModelConfig& c = ck.config();
  std::ostringstream o;
  o << "{\"hidden\":" << c.hidden_size << ",\"num_layers\":" << c.num_hidden_layers << ",\"num_experts\":" << c.experts()
    << ",\"top_k\":" << c.num_experts_per_tok << ",\"inter\":" << c.moe_intermediate_size
    << ",\"shared_inter\":" << c.shared_inter() << ",\"norm_topk_prob\":" << (c.norm_topk_prob ? "true" : "false")
    << ",\"bits\":" << c.quant_bits << ",\"group_size\":" << c.quant_group_size << ",\"n_group\":" << c.n_group
    << ",\"topk_group\":" << c.topk_group << ",\"routed_scaling_factor\":" << c.routed_scaling_factor
    << ",\"sigmoid_routed\":" << (c.sigmoid_routed() ? "true" : "false") << ",\"n_heads\":" << c.num_attention_heads
    << ",\"n_kv_heads\":" << c.num_key_value_heads << ",\"head_dim\":" << c.attn_head_dim()
    << ",\"vocab\":" << c.vocab_size << ",\"intermediate\":" << c.intermediate_size
    << ",\"rms_eps\":" << c.rms_norm_eps << ",\"rope_theta\":" << c.rope_theta
    << ",\"tie_word_embeddings\":" << (c.tie_word_embeddings ? "true" : "false") << ",\"moe_layers\":[";
  const std::vector<int> layers = ck.moe_layers();
  for (size_t i = 0; i < layers.size(); ++i) o << (i ? "," : "") << layers[i];
  o << "]}";
  std::cout << o.str() << std::endl;
  return 0;
}

int dump(const std::string& dir, int layer, const std::string& out) {
  Checkpoint ck(dir);
  const HostLayer L = ck.config().sigmoid_routed() ? ck.sigmoid_moe_layer(layer) : ck.moe_layer(layer);
  std::ostringstream m;
  m << "{\"sigmoid\":" << (L.sigmoid ? "true" : "false") << ",\"arrays\":{";
  bool first = true;
  auto entry = [&](const std::string& name, const char* dtype, const std::vector<int64_t>& shape) {
    m << (first ? "" : ",") << q(name) << ":{\"dtype\":" << q(dtype) << ",\"shape\":" << shape_json(shape) << "}";
    first = false;
  };
  const int64_t E = ck.config().experts(), H = ck.config().hidden_size;
  write_raw(out + "/router_w.bin", L.router_w);
  entry("router_w", "BF16", {E, H});
  if (!L.correction_bias.empty()) {
    write_raw(out + "/correction_bias.bin", L.correction_bias);
    entry("correction_bias", "F32", {E});
  }
  auto qdump = [&](const std::string& name, const HostQ& hq) {
    write_raw(out + "/" + name + ".w.bin", hq.w);
    entry(name + ".w", "U32", hq.w_shape);
    write_raw(out + "/" + name + ".s.bin", hq.s);
    entry(name + ".s", "BF16", hq.s_shape);
    if (hq.has_biases()) {
      write_raw(out + "/" + name + ".b.bin", hq.b);
      entry(name + ".b", "BF16", hq.s_shape);
    }
  };
  if (L.sigmoid) {
    qdump("fc1", L.up);
    qdump("fc2", L.down);
    if (L.has_shared) {
      qdump("shared_up", L.shared_up);
      qdump("shared_down", L.shared_down);
    }
  } else {
    qdump("gate", L.gate);
    qdump("up", L.up);
    qdump("down", L.down);
    if (L.has_shared) {
      qdump("shared_gate", L.shared_gate);
      qdump("shared_up", L.shared_up);
      qdump("shared_down", L.shared_down);
      write_raw(out + "/shared_expert_gate_w.bin", L.shared_expert_gate_w);
      entry("shared_expert_gate_w", "BF16", {1, H});
    }
  }
  m << "}}";
  std::ofstream f(out + "/manifest.json");
  f << m.str() << std::endl;
  if (!f) throw std::runtime_error(out + "/manifest.json: write failed");
  return 0;
}

void cuda_ok(cudaError_t e, const char* what) {
  if (e != cudaSuccess) throw Error(FM_ECUDA, std::string(what) + ": " + cudaGetErrorString(e));
}

int run(const std::string& dir, int layer, const std::string& xpath, int64_t T, const std::string& ypath, int dev) {
  MoEModel model(dir, dev, nullptr, T, {layer});
  const int64_t H = model.config().hidden_size;
  std::vector<uint16_t> x(static_cast<size_t>(T * H)), y(static_cast<size_t>(T * H));
  {
    std::ifstream f(xpath, std::ios::binary);
    if (!f) throw std::runtime_error(xpath + ": cannot open");
    f.read(reinterpret_cast<char*>(x.data()), static_cast<std::streamsize>(x.size() * 2));
    if (f.gcount() != static_cast<std::streamsize>(x.size() * 2))
      throw std::runtime_error(xpath + ": holds fewer than T x hidden bf16 values");
  }
  void* dx = nullptr;
  void* dy = nullptr;
  const size_t bytes = x.size() * 2;
  cuda_ok(cudaMalloc(&dx, bytes ? bytes : 16), "cudaMalloc x");
  cuda_ok(cudaMalloc(&dy, bytes ? bytes : 16), "cudaMalloc y");
  try {
    cuda_ok(cudaMemcpy(dx, x.data(), bytes, cudaMemcpyHostToDevice), "cudaMemcpy x");
    model.moe_block(static_cast<const uint16_t*>(dx), T, static_cast<uint16_t*>(dy), layer);
    model.handle().sync();
    cuda_ok(cudaMemcpy(y.data(), dy, bytes, cudaMemcpyDeviceToHost), "cudaMemcpy y");
  } catch (...) {
    cudaFree(dx);
    cudaFree(dy);
    throw;
  }
  cudaFree(dx);
  cudaFree(dy);
  write_raw(ypath, y);
  return 0;
}

int generate(const std::string& dir, const std::string& ppath, int B, int L, int steps, const std::string& opath,
             int dev) {
  if (B <= 0 || L <= 0 || steps <= 0) throw std::runtime_error("B, L and STEPS must be positive");
  std::vector<int32_t> prompt(static_cast<size_t>(B) * L);
  {
    std::ifstream f(ppath, std::ios::binary);
    if (!f) throw std::runtime_error(ppath + ": cannot open");
    f.read(reinterpret_cast<char*>(prompt.data()), static_cast<std::streamsize>(prompt.size() * 4));
    if (f.gcount() != static_cast<std::streamsize>(prompt.size() * 4))
      throw std::runtime_error(ppath + ": holds fewer than B x L int32 tokens");
  }
  auto dec = Decoder::open(dir, dev, B, L + steps, nullptr);
  const std::vector<int32_t> out = dec->generate(prompt.data(), B, L, steps);
  write_raw(opath, out);
  return 0;
}

// the decoder layout of a model directory, checked without a device (plan_decoder)
int check_decoder(const std::string& dir) {
  Checkpoint ck(dir);
  const DecoderPlan p = plan_decoder(ck);
  std::ostringstream o;
  o << "{\"layers\":" << p.cfg.layers << ",\"moe_layers\":[";
  bool first = true;
  for (int i = 0; i < p.cfg.layers; ++i)
    if (p.layers[i].is_moe) {
      o << (first ? "" : ",") << i;
      first = false;
      (void)ck.moe_layer(i);  // the MoE layer's own checks
    }
  bool bias = p.cfg.layers > 0, qk_norm = p.cfg.layers > 0;
  for (const auto& l : p.layers) {
    bias = bias && l.q_bias && l.k_bias && l.v_bias;
    qk_norm = qk_norm && l.q_norm && l.k_norm;
  }
  o << "],\"attn_bias\":" << (bias ? "true" : "false") << ",\"qk_norm\":" << (qk_norm ? "true" : "false")
    << ",\"embed_quantized\":" << (p.embed.w ? "true" : "false")
    << ",\"tie_word_embeddings\":" << (p.cfg.tie_word_embeddings ? "true" : "false") << ",\"head_dim\":"
    << p.cfg.head_dim << ",\"vocab\":" << p.cfg.vocab << "}";
  std::cout << o.str() << std::endl;
  return 0;
}

int usage() {
  std::cerr << "usage: fm_host inspect DIR | dump DIR LAYER OUT | run DIR LAYER X T Y [DEVICE] |"
               " check-decoder DIR | generate DIR PROMPT B L STEPS OUT [DEVICE]\n";
  return 2;
}

}  // namespace

int main(int argc, char** argv) {
  if (argc < 3) return usage();
  const std::string cmd = argv[1];
  try {
    if (cmd == "inspect" && argc == 3) return inspect(argv[2]);
    if (cmd == "dump" && argc == 5) return dump(argv[2], std::atoi(argv[3]), argv[4]);
    if (cmd == "run" && (argc == 7 || argc == 8))
      return run(argv[2], std::atoi(argv[3]), argv[4], std::atoll(argv[5]), argv[6], argc == 8 ? std::atoi(argv[7]) : 0);
    if (cmd == "check-decoder" && argc == 3) return check_decoder(argv[2]);
    if (cmd == "generate" && (argc == 8 || argc == 9))
      return generate(argv[2], argv[3], std::atoi(argv[4]), std::atoi(argv[5]), std::atoi(argv[6]), argv[7],
                      argc == 9 ? std::atoi(argv[8]) : 0);
    return usage();
  } catch (const Error& e) {
    std::cerr << "fm_status " << e.status() << "\n" << e.what() << std::endl;
    return 3;
  } catch (const std::exception& e) {
    std::cerr << "error: " << e.what() << std::endl;
    return 4;
  }
}
