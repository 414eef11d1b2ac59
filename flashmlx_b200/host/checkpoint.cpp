// checkpoint.cpp -- see checkpoint.hpp.
#include "checkpoint.hpp"

#include <dirent.h>
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <cerrno>
#include <cstring>
#include <fstream>
#include <sstream>
#include <stdexcept>

#include "json.hpp"

namespace flashmoe {

namespace {

std::runtime_error err(const std::string& what) { return std::runtime_error(what); }

std::string read_file(const std::string& path) {
  std::ifstream f(path, std::ios::binary);
  if (!f) throw err(path + ": cannot open");
  std::ostringstream ss;
  ss << f.rdbuf();
  return ss.str();
}

size_t dtype_size(const std::string& dt) {
  if (dt == "BOOL" || dt == "U8" || dt == "I8") return 1;
  if (dt == "U16" || dt == "I16" || dt == "F16" || dt == "BF16") return 2;
  if (dt == "U32" || dt == "I32" || dt == "F32") return 4;
  if (dt == "U64" || dt == "I64" || dt == "F64") return 8;
  return 0;
}

std::string shape_str(const std::vector<int64_t>& s) {
  std::string r = "(";
  for (size_t i = 0; i < s.size(); ++i) r += (i ? ", " : "") + std::to_string(s[i]);
  return r + (s.size() == 1 ? ",)" : ")");
}

template <typename T>
std::vector<T> copy_out(const TensorView& t) {
  std::vector<T> v(t.nbytes / sizeof(T));
  if (t.nbytes) std::memcpy(v.data(), t.data, t.nbytes);
  return v;
}

int to_int(double v, const char* key) {
  if (!(v >= -2147483648.0 && v <= 2147483647.0) || v != static_cast<double>(static_cast<int>(v)))
    throw err(std::string("config.json: ") + key + " is not an integer");
  return static_cast<int>(v);
}

}  // namespace

int64_t TensorView::numel() const {
  int64_t n = 1;
  for (int64_t d : shape) n *= d;
  return n;
}

fm_moe_config ModelConfig::moe_config() const {
  fm_moe_config c{};
  c.hidden = hidden_size;
  c.inter = moe_intermediate_size;
  c.num_experts = experts();
  c.top_k = num_experts_per_tok;
  c.group_size = quant_group_size;
  c.bits = quant_bits;
  c.norm_topk_prob = norm_topk_prob ? 1 : 0;
  c.shared_inter = shared_inter();
  c.router_quantized = 0;
  c.shared_gate_quantized = 0;
  return c;
}

fm_moe_variant ModelConfig::variant() const {
  fm_moe_variant v{};
  v.score_func = FM_SCORE_SIGMOID;
  v.n_group = n_group;
  v.topk_group = topk_group;
  v.routed_scaling_factor = routed_scaling_factor;
  v.expert_act = FM_ACT_RELU2;
  v.shared_ungated = 1;
  v.correction_bias = nullptr;
  v.topk_scores_f32 = nullptr;
  return v;
}

ModelConfig load_config(const std::string& model_dir) {
  const json::Value c = json::parse(read_file(model_dir + "/config.json"));
  if (!c.is_object()) throw err(model_dir + "/config.json: not a JSON object");
  ModelConfig m;
  m.hidden_size = to_int(c.number_or("hidden_size", 4096), "hidden_size");
  m.intermediate_size = to_int(c.number_or("intermediate_size", 14336), "intermediate_size");
  m.num_hidden_layers = to_int(c.number_or("num_hidden_layers", 32), "num_hidden_layers");
  m.num_attention_heads = to_int(c.number_or("num_attention_heads", 32), "num_attention_heads");
  m.num_key_value_heads = to_int(c.number_or("num_key_value_heads", 8), "num_key_value_heads");
  m.head_dim = to_int(c.number_or("head_dim", 0), "head_dim");
  m.vocab_size = to_int(c.number_or("vocab_size", 128256), "vocab_size");
  m.rms_norm_eps = static_cast<float>(c.number_or("rms_norm_eps", 1e-5));
  m.rope_theta = static_cast<float>(c.number_or("rope_theta", 10000.0));
  m.tie_word_embeddings = c.bool_or("tie_word_embeddings", true);
  m.num_experts = to_int(c.number_or("num_experts", 0), "num_experts");
  m.n_routed_experts = to_int(c.number_or("n_routed_experts", 0), "n_routed_experts");
  m.num_experts_per_tok = to_int(c.number_or("num_experts_per_tok", 0), "num_experts_per_tok");
  m.moe_intermediate_size = to_int(c.number_or("moe_intermediate_size", 0), "moe_intermediate_size");
  m.shared_expert_intermediate_size =
      to_int(c.number_or("shared_expert_intermediate_size", 0), "shared_expert_intermediate_size");
  m.n_shared_experts = to_int(c.number_or("n_shared_experts", 1), "n_shared_experts");
  m.moe_shared_expert_intermediate_size =
      to_int(c.number_or("moe_shared_expert_intermediate_size", 0), "moe_shared_expert_intermediate_size");
  m.norm_topk_prob = c.bool_or("norm_topk_prob", false);
  m.n_group = to_int(c.number_or("n_group", 1), "n_group");
  m.topk_group = to_int(c.number_or("topk_group", 1), "topk_group");
  m.routed_scaling_factor = static_cast<float>(c.number_or("routed_scaling_factor", 1.0));
  m.hybrid_override_pattern = c.string_or("hybrid_override_pattern", "");
  if (const json::Value* q = c.find("quantization"); q && q->is_object()) {
    m.quant_bits = to_int(q->number_or("bits", 0), "quantization.bits");
    m.quant_group_size = to_int(q->number_or("group_size", 64), "quantization.group_size");
  }
  return m;
}

// The format: an 8-byte little-endian header length, a JSON header mapping each name to
// {dtype, shape, data_offsets [begin, end)} relative to the data that follows it.
SafetensorsFile::SafetensorsFile(const std::string& path) {
  const int fd = ::open(path.c_str(), O_RDONLY);
  if (fd < 0) throw err(path + ": cannot open: " + std::strerror(errno));
  struct stat st;
  if (::fstat(fd, &st) != 0) {
    ::close(fd);
    throw err(path + ": cannot stat");
  }
  size_ = static_cast<size_t>(st.st_size);
  if (size_ < 8) {
    ::close(fd);
    throw err(path + ": not a safetensors file (short header)");
  }
  map_ = ::mmap(nullptr, size_, PROT_READ, MAP_PRIVATE, fd, 0);
  ::close(fd);
  if (map_ == MAP_FAILED) {
    map_ = nullptr;
    throw err(path + ": mmap failed");
  }
  const uint8_t* base = static_cast<const uint8_t*>(map_);
  uint64_t n = 0;
  for (int i = 7; i >= 0; --i) n = (n << 8) | base[i];
  if (n > size_ - 8) {
    unmap();
    throw err(path + ": header length " + std::to_string(n) + " exceeds the file");
  }
  json::Value h;
  try {
    h = json::parse(reinterpret_cast<const char*>(base + 8), static_cast<size_t>(n));
  } catch (const std::exception& e) {
    unmap();
    throw err(path + ": " + e.what());
  }
  if (!h.is_object()) {
    unmap();
    throw err(path + ": header is not a JSON object");
  }
  const uint8_t* data = base + 8 + n;
  const uint64_t data_size = size_ - 8 - n;
  for (const auto& [name, info] : h.obj) {
    if (name == "__metadata__") continue;
    TensorView t;
    const json::Value* dt = info.find("dtype");
    const json::Value* shape = info.find("shape");
    const json::Value* offs = info.find("data_offsets");
    if (!dt || dt->kind != json::Value::String || !shape || shape->kind != json::Value::Array || !offs ||
        offs->kind != json::Value::Array || offs->arr.size() != 2 || offs->arr[0].kind != json::Value::Number ||
        offs->arr[1].kind != json::Value::Number || offs->arr[0].num < 0 || offs->arr[1].num < 0 ||
        offs->arr[0].num > 9.0e15 || offs->arr[1].num > 9.0e15) {
      unmap();
      throw err(path + ": " + name + ": malformed tensor record");
    }
    t.dtype = dt->str;
    const size_t es = dtype_size(t.dtype);
    if (!es) {
      unmap();
      throw err(path + ": " + name + ": unsupported dtype " + t.dtype);
    }
    uint64_t numel = 1;
    for (const auto& d : shape->arr) {
      if (d.kind != json::Value::Number || d.num < 0 || d.num > 9.0e15 || d.num != static_cast<double>(static_cast<int64_t>(d.num))) {
        unmap();
        throw err(path + ": " + name + ": bad shape");
      }
      t.shape.push_back(static_cast<int64_t>(d.num));
      numel *= static_cast<uint64_t>(d.num);
    }
    const uint64_t beg = static_cast<uint64_t>(offs->arr[0].num), end = static_cast<uint64_t>(offs->arr[1].num);
    if (!(beg <= end && end <= data_size) || end - beg != numel * es) {
      unmap();
      throw err(path + ": " + name + ": data_offsets " + std::to_string(beg) + ".." + std::to_string(end) +
                " do not hold " + t.dtype + shape_str(t.shape));
    }
    t.data = data + beg;
    t.nbytes = static_cast<size_t>(end - beg);
    tensors_.emplace(name, std::move(t));
  }
}

void SafetensorsFile::unmap() {
  if (map_) ::munmap(map_, size_);
  map_ = nullptr;
}

SafetensorsFile::~SafetensorsFile() { unmap(); }

Checkpoint::Checkpoint(const std::string& model_dir) : dir_(model_dir), config_(load_config(model_dir)) {
  std::vector<std::string> names;
  if (DIR* d = ::opendir(model_dir.c_str())) {
    while (dirent* e = ::readdir(d)) {
      const std::string n = e->d_name;
      if (n.size() > 12 && n.compare(n.size() - 12, 12, ".safetensors") == 0) names.push_back(n);
    }
    ::closedir(d);
  }
  if (names.empty()) throw err("no .safetensors files in " + model_dir);
  std::sort(names.begin(), names.end());
  for (const auto& n : names) {
    files_.push_back(std::make_unique<SafetensorsFile>(model_dir + "/" + n));
    for (const auto& [key, t] : files_.back()->tensors()) {
      std::string k = key;
      for (const char* pre : {"model.", "backbone."}) {
        const size_t len = std::strlen(pre);
        if (k.compare(0, len, pre) == 0) {
          k = k.substr(len);
          break;
        }
      }
      tensors_[k] = &t;  // a later file overrides an earlier one
    }
  }
}

const TensorView& Checkpoint::get(const std::string& key, const char* dtype) const {
  auto it = tensors_.find(key);
  if (it == tensors_.end()) throw err(dir_ + ": tensor " + key + " missing");
  if (dtype && it->second->dtype != dtype)
    throw err(key + ": " + it->second->dtype + ", expected " + dtype);
  return *it->second;
}

std::vector<int> Checkpoint::moe_layers() const {
  std::vector<int> out;
  const ModelConfig& c = config_;
  if (c.sigmoid_routed()) {
    if (static_cast<int>(c.hybrid_override_pattern.size()) != c.num_hidden_layers)
      throw err("hybrid_override_pattern length differs from num_hidden_layers");
    for (int i = 0; i < c.num_hidden_layers; ++i)
      if (c.hybrid_override_pattern[i] == 'E') out.push_back(i);
    return out;
  }
  for (int i = 0; i < c.num_hidden_layers; ++i)
    if (has("layers." + std::to_string(i) + ".mlp.gate.weight")) out.push_back(i);
  return out;
}

HostQ Checkpoint::qmatrix(const std::string& prefix) const {
  HostQ q;
  const TensorView& w = get(prefix + ".weight", "U32");
  const TensorView& s = get(prefix + ".scales", "BF16");
  q.w = copy_out<uint32_t>(w);
  q.s = copy_out<uint16_t>(s);
  q.w_shape = w.shape;
  q.s_shape = s.shape;
  if (has(prefix + ".biases")) {
    const TensorView& b = get(prefix + ".biases", "BF16");
    if (b.shape != s.shape) throw err(prefix + ".biases: shape " + shape_str(b.shape) + " differs from the scales'");
    q.b = copy_out<uint16_t>(b);
  }
  return q;
}

HostQ Checkpoint::stacked(const std::string& mlp, const std::string& proj) const {
  const std::string pre = mlp + ".switch_mlp." + proj;
  if (has(pre + ".weight")) return qmatrix(pre);  // mlx-lm layout: already [E, ...]
  const int E = config_.experts();
  HostQ out;
  for (int e = 0; e < E; ++e) {
    const std::string p = mlp + ".experts." + std::to_string(e) + "." + proj;
    HostQ q = qmatrix(p);
    if (e == 0) {
      out.w_shape = q.w_shape;
      out.s_shape = q.s_shape;
      out.w_shape.insert(out.w_shape.begin(), E);
      out.s_shape.insert(out.s_shape.begin(), E);
      out.w.reserve(q.w.size() * E);
      out.s.reserve(q.s.size() * E);
      if (q.has_biases()) out.b.reserve(q.b.size() * E);
    } else {
      if (std::vector<int64_t>(out.w_shape.begin() + 1, out.w_shape.end()) != q.w_shape ||
          std::vector<int64_t>(out.s_shape.begin() + 1, out.s_shape.end()) != q.s_shape)
        throw err(p + ": shape differs from expert 0's");
      if (q.has_biases() != out.has_biases())
        throw err(mlp + ".experts.*." + proj + ": biases present for some experts only");
    }
    out.w.insert(out.w.end(), q.w.begin(), q.w.end());
    out.s.insert(out.s.end(), q.s.begin(), q.s.end());
    out.b.insert(out.b.end(), q.b.begin(), q.b.end());
  }
  return out;
}

void Checkpoint::check_q(int i, const char* name, const HostQ& q, std::vector<int64_t> lead, int64_t n,
                         int64_t k) const {
  const int per_word = 32 / config_.quant_bits;
  std::vector<int64_t> ws = lead, ss = lead;
  ws.insert(ws.end(), {n, k / per_word});
  ss.insert(ss.end(), {n, k / config_.quant_group_size});
  if (q.w_shape != ws)
    throw err("layer " + std::to_string(i) + " " + name + ".weight: shape " + shape_str(q.w_shape) +
              ", config gives " + shape_str(ws));
  if (q.s_shape != ss)
    throw err("layer " + std::to_string(i) + " " + name + ".scales: shape " + shape_str(q.s_shape) +
              ", config gives " + shape_str(ss));
}

HostLayer Checkpoint::moe_layer(int i) const {
  const ModelConfig& c = config_;
  const std::string mlp = "layers." + std::to_string(i) + ".mlp";
  if (!has(mlp + ".gate.weight")) throw err("layer " + std::to_string(i) + " has no router (" + mlp + ".gate.weight)");
  if (has(mlp + ".gate.scales")) throw err(mlp + ".gate is quantized: a quantized router is not implemented");
  if (c.quant_bits != 4)
    throw err("quantization bits = " + std::to_string(c.quant_bits) + ": only 4-bit affine weights are implemented");
  const int64_t E = c.experts(), H = c.hidden_size, I = c.moe_intermediate_size, Is = c.shared_inter();
  HostLayer L;
  const TensorView& r = get(mlp + ".gate.weight", "BF16");
  if (r.shape != std::vector<int64_t>{E, H})
    throw err("layer " + std::to_string(i) + " router: shape " + shape_str(r.shape) + ", config gives " +
              shape_str({E, H}));
  L.router_w = copy_out<uint16_t>(r);
  L.gate = stacked(mlp, "gate_proj");
  L.up = stacked(mlp, "up_proj");
  L.down = stacked(mlp, "down_proj");
  check_q(i, "gate", L.gate, {E}, I, H);
  check_q(i, "up", L.up, {E}, I, H);
  check_q(i, "down", L.down, {E}, H, I);
  if (has(mlp + ".shared_expert.gate_proj.weight")) {
    L.has_shared = true;
    L.shared_gate = qmatrix(mlp + ".shared_expert.gate_proj");
    L.shared_up = qmatrix(mlp + ".shared_expert.up_proj");
    L.shared_down = qmatrix(mlp + ".shared_expert.down_proj");
    if (has(mlp + ".shared_expert_gate.scales"))
      throw err(mlp + ".shared_expert_gate is quantized: not implemented");
    const TensorView& g = get(mlp + ".shared_expert_gate.weight", "BF16");
    if (g.numel() != H) throw err("layer " + std::to_string(i) + " shared_expert_gate: " + shape_str(g.shape));
    L.shared_expert_gate_w = copy_out<uint16_t>(g);
    check_q(i, "shared_gate", L.shared_gate, {}, Is, H);
    check_q(i, "shared_up", L.shared_up, {}, Is, H);
    check_q(i, "shared_down", L.shared_down, {}, H, Is);
  } else if (Is) {
    throw err("layer " + std::to_string(i) + ": config has a shared expert (" + std::to_string(Is) +
              ") but the checkpoint has none");
  }
  return L;
}

HostLayer Checkpoint::sigmoid_moe_layer(int i) const {
  const ModelConfig& c = config_;
  const std::string mx = "layers." + std::to_string(i) + ".mixer";
  if (!has(mx + ".gate.weight")) throw err("layer " + std::to_string(i) + " has no router (" + mx + ".gate.weight)");
  if (has(mx + ".gate.scales")) throw err(mx + ".gate is quantized: a quantized router is not implemented");
  if (c.quant_bits != 4)
    throw err("quantization bits = " + std::to_string(c.quant_bits) + ": only 4-bit affine weights are implemented");
  const int64_t E = c.experts(), H = c.hidden_size, I = c.moe_intermediate_size, Is = c.shared_inter();
  HostLayer L;
  L.sigmoid = true;
  const TensorView& r = get(mx + ".gate.weight", "BF16");
  if (r.shape != std::vector<int64_t>{E, H})
    throw err("layer " + std::to_string(i) + " router_w: shape " + shape_str(r.shape) + ", config gives " +
              shape_str({E, H}));
  L.router_w = copy_out<uint16_t>(r);
  if (has(mx + ".gate.e_score_correction_bias")) {
    const TensorView& b = get(mx + ".gate.e_score_correction_bias");
    if (b.numel() != E || b.shape.size() != 1)
      throw err("layer " + std::to_string(i) + " correction bias: shape " + shape_str(b.shape) + ", config gives (" +
                std::to_string(E) + ",)");
    if (b.dtype == "F32") {
      L.correction_bias = copy_out<float>(b);
    } else if (b.dtype == "BF16") {
      const std::vector<uint16_t> v = copy_out<uint16_t>(b);
      L.correction_bias.resize(v.size());
      for (size_t j = 0; j < v.size(); ++j) {
        const uint32_t u = static_cast<uint32_t>(v[j]) << 16;
        std::memcpy(&L.correction_bias[j], &u, 4);
      }
    } else {
      throw err(mx + ".gate.e_score_correction_bias: " + b.dtype + ", expected F32 or BF16");
    }
  }
  L.up = qmatrix(mx + ".switch_mlp.fc1");
  L.down = qmatrix(mx + ".switch_mlp.fc2");
  check_q(i, "fc1", L.up, {E}, I, H);
  check_q(i, "fc2", L.down, {E}, H, I);
  if (has(mx + ".shared_experts.up_proj.weight")) {
    L.has_shared = true;
    L.shared_up = qmatrix(mx + ".shared_experts.up_proj");
    L.shared_down = qmatrix(mx + ".shared_experts.down_proj");
    check_q(i, "shared_up", L.shared_up, {}, Is, H);
    check_q(i, "shared_down", L.shared_down, {}, H, Is);
  } else if (Is) {
    throw err("layer " + std::to_string(i) + ": config has a shared expert (" + std::to_string(Is) +
              ") but the checkpoint has none");
  }
  return L;
}

}  // namespace flashmoe
