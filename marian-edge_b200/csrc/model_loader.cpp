// model_loader.cpp -- Marian binary v1 reader and Q8 schema check (host C++).
#include "model_loader.h"

#include <algorithm>
#include <cmath>
#include <cstring>
#include <set>

#include "marian_cuda.h"

namespace mc {

namespace {

constexpr uint64_t kTypeInt8 = 0x0101;
constexpr uint64_t kTypeFloat32 = 0x0404;
constexpr uint64_t kTypeIntgemm8 = 0x4101;
constexpr size_t kMaxFileBytes = 128u * 1024 * 1024;
constexpr uint64_t kMaxTensors = 4096;
constexpr uint64_t kMaxNameBytes = 16 * 1024;
constexpr uint64_t kMaxRank = 8;
constexpr size_t kAlign = 256;

struct Reader {
  const uint8_t* p;
  size_t len, pos = 0;
  bool take(size_t n, const uint8_t** out) {
    if (n > len - pos) return false;
    *out = p + pos;
    pos += n;
    return true;
  }
  bool u64(uint64_t* v) {
    const uint8_t* b;
    if (!take(8, &b)) return false;
    std::memcpy(v, b, 8);
    return true;
  }
  bool i32(int32_t* v) {
    const uint8_t* b;
    if (!take(4, &b)) return false;
    std::memcpy(v, b, 4);
    return true;
  }
};

struct Header {
  uint64_t name_len, type, rank, data_len;
};

}  // namespace

std::string parse_marian_v1(const uint8_t* data, size_t len, HostModel* out) {
  if (len > kMaxFileBytes) return "model exceeds the maximum file size";
  Reader r{data, len};
  uint64_t version = 0, count = 0;
  if (!r.u64(&version) || !r.u64(&count)) return "truncated header";
  if (version != 1) return "unsupported version " + std::to_string(version) + "; expected 1";
  if (count == 0 || count > kMaxTensors) return "tensor count outside 1..=4096";
  std::vector<Header> hs(count);
  for (uint64_t i = 0; i < count; ++i) {
    Header& h = hs[i];
    if (!r.u64(&h.name_len) || !r.u64(&h.type) || !r.u64(&h.rank) || !r.u64(&h.data_len))
      return "truncated tensor header";
    if (h.type != kTypeInt8 && h.type != kTypeFloat32 && h.type != kTypeIntgemm8)
      return "unsupported tensor type";
    if (h.name_len < 2 || h.name_len > kMaxNameBytes) return "tensor name length out of range";
    if (h.rank == 0 || h.rank > kMaxRank) return "tensor rank out of range";
    if (h.data_len == 0 || h.data_len > kMaxFileBytes) return "invalid tensor data length";
  }
  std::vector<std::string> names(count);
  std::set<std::string> seen;
  for (uint64_t i = 0; i < count; ++i) {
    const uint8_t* b;
    if (!r.take(hs[i].name_len, &b)) return "truncated tensor name";
    if (b[hs[i].name_len - 1] != 0 || std::memchr(b, 0, hs[i].name_len - 1) != nullptr)
      return "tensor name is not one NUL-terminated string";
    names[i].assign(reinterpret_cast<const char*>(b), hs[i].name_len - 1);
    if (!seen.insert(names[i]).second) return "duplicate tensor name " + names[i];
  }
  std::vector<std::vector<int64_t>> shapes(count);
  for (uint64_t i = 0; i < count; ++i) {
    for (uint64_t k = 0; k < hs[i].rank; ++k) {
      int32_t d;
      if (!r.i32(&d)) return "truncated shape";
      if (d <= 0) return "tensor " + names[i] + " has a non-positive shape dimension";
      shapes[i].push_back(d);
    }
  }
  uint64_t pad = 0;
  const uint8_t* padding;
  if (!r.u64(&pad) || !r.take(pad, &padding)) return "truncated header padding";
  for (uint64_t i = 0; i < pad; ++i)
    if (padding[i]) return "header alignment padding contains non-zero bytes";
  if (r.pos % kAlign) return "tensor data is not 256-byte aligned";
  for (uint64_t i = 0; i < count; ++i) {
    HostTensor t;
    t.name = names[i];
    t.shape = shapes[i];
    const int64_t n = t.elements();
    if (n <= 0 || n > (int64_t)kMaxFileBytes) return t.name + ": element count overflows";
    size_t logical = 0;
    if (hs[i].type == kTypeInt8) {
      t.type = TensorType::Int8;
      logical = (size_t)n;
    } else if (hs[i].type == kTypeFloat32) {
      t.type = TensorType::Float32;
      logical = (size_t)n * 4;
    } else {
      t.type = TensorType::Intgemm8;
      logical = (size_t)n + 4;
    }
    const size_t expected =
        t.type == TensorType::Int8 ? logical : (logical + kAlign - 1) / kAlign * kAlign;
    if (hs[i].data_len != expected) return t.name + ": record length mismatch";
    const uint8_t* b;
    if (!r.take(hs[i].data_len, &b)) return t.name + ": truncated payload";
    for (size_t k = logical; k < hs[i].data_len; ++k)
      if (b[k]) return t.name + ": record padding contains non-zero bytes";
    if (t.type == TensorType::Float32) {
      t.f32.resize(n);
      std::memcpy(t.f32.data(), b, (size_t)n * 4);
      for (float v : t.f32)
        if (!std::isfinite(v)) return t.name + ": float32 payload is not finite";
    } else {
      t.i8.resize(n);
      std::memcpy(t.i8.data(), b, (size_t)n);
      if (t.type == TensorType::Intgemm8) {
        for (int8_t v : t.i8)
          if (v == -128) return t.name + ": symmetric intgemm8 payload contains -128";
        std::memcpy(&t.quant_mult, b + n, 4);
        if (!std::isfinite(t.quant_mult) || t.quant_mult <= 0.0f)
          return t.name + ": intgemm8 quantization multiplier must be finite and positive";
      }
    }
    out->order.push_back(t.name);
    out->tensors.emplace(t.name, std::move(t));
  }
  if (r.pos != len) return std::to_string(len - r.pos) + " trailing bytes remain after the final tensor";
  return "";
}

std::string activation_scale(const HostModel& m, const std::string& weight, float* alpha) {
  auto it = m.tensors.find(weight + "_QuantMultA");
  if (it == m.tensors.end()) return "missing tensor " + weight + "_QuantMultA";
  const HostTensor& t = it->second;
  if (t.elements() != 1) return t.name + ": activation scale must be scalar";
  float s = 0.0f;
  if (t.type == TensorType::Float32) s = t.f32[0];
  else if (t.type == TensorType::Intgemm8) s = (float)t.i8[0] / t.quant_mult;
  else return t.name + ": activation scale must be float32 or intgemm8";
  if (!std::isfinite(s) || s <= 0.0f) return t.name + ": activation scale must be finite and positive";
  *alpha = s;
  return "";
}

namespace {

constexpr char kAlphaSuffix[] = "_QuantMultA";
constexpr char kRowSuffix[] = "_QuantMultRows";

bool ends_with(const std::string& s, const char* suffix) {
  const size_t n = std::strlen(suffix);
  return s.size() >= n && s.compare(s.size() - n, n, suffix) == 0;
}

}  // namespace

std::string validate_q8(const HostModel& m, Q8Inventory* inv) {
  *inv = Q8Inventory();
  for (const std::string& name : m.order) {
    const HostTensor& t = m.tensors.at(name);
    if (ends_with(name, kAlphaSuffix)) {
      const std::string weight = name.substr(0, name.size() - std::strlen(kAlphaSuffix));
      float a;
      std::string err = activation_scale(m, weight, &a);
      if (!err.empty()) return err;
      auto w = m.tensors.find(weight);
      if (w == m.tensors.end()) return "missing tensor " + weight;
      if (w->second.type != TensorType::Intgemm8)
        return name + ": activation scale refers to non-Q8 tensor " + weight;
      ++inv->activation_scales;
      continue;
    }
    if (ends_with(name, kRowSuffix)) {
      const std::string weight = name.substr(0, name.size() - std::strlen(kRowSuffix));
      auto w = m.tensors.find(weight);
      if (w == m.tensors.end()) return "missing tensor " + weight;
      if (w->second.type != TensorType::Intgemm8 || ends_with(weight, "_Wemb") || w->second.shape.size() != 2)
        return name + ": row multipliers refer to a tensor that is not a dense Q8 weight";
      const int64_t out = w->second.shape[1];
      const bool shape_ok = (t.shape.size() == 2 && t.shape[0] == 1 && t.shape[1] == out) ||
                            (t.shape.size() == 1 && t.shape[0] == out);
      if (t.type != TensorType::Float32 || !shape_ok)
        return name + ": row multipliers must be float32 [1, " + std::to_string(out) + "]";
      for (float v : t.f32)
        if (!std::isfinite(v) || v <= 0.0f) return name + ": row multipliers must be finite and positive";
      ++inv->row_scaled;
      continue;
    }
    if (t.type != TensorType::Intgemm8) continue;
    if (t.shape.size() != 2) return name + ": Q8 weight must have rank 2";
    if (ends_with(name, "_Wemb")) {
      ++inv->embeddings;
    } else {
      float a;
      std::string err = activation_scale(m, name, &a);
      if (!err.empty()) return err;
      ++inv->dense_linears;
    }
  }
  if (inv->dense_linears + inv->embeddings == 0) return "model contains no intgemm8 weight tensors";
  return "";
}

std::vector<float> weight_row_mults(const HostModel& m, const std::string& weight) {
  auto it = m.tensors.find(weight + kRowSuffix);
  if (it == m.tensors.end()) return {};
  return it->second.f32;
}

namespace {

std::string expect_shape(const HostModel& m, const std::string& name, std::vector<int64_t> shape,
                         TensorType type) {
  auto it = m.tensors.find(name);
  if (it == m.tensors.end()) return "missing tensor " + name;
  const HostTensor& t = it->second;
  if (t.type != type) return name + ": unexpected tensor type";
  bool ok = t.shape == shape;
  // f32 vectors may be stored as [n] or [1, n] (legacy_q8.rs:677-693)
  if (!ok && shape.size() == 2 && shape[0] == 1 && t.shape.size() == 1 && t.shape[0] == shape[1]) ok = true;
  if (!ok) return name + ": unexpected shape";
  return "";
}

void add_dense(std::set<std::string>* names, const std::string& n) {
  names->insert(n);
  names->insert(n + "_QuantMultA");
}

}  // namespace

std::string validate_schema(HostModel* m) {
  auto& T = m->tensors;
  auto emb = T.find("encoder_Wemb");
  if (emb == T.end()) return "missing tensor encoder_Wemb";
  if (emb->second.shape.size() != 2) return "encoder_Wemb must be rank 2";
  m->vocab_src = (int)emb->second.shape[0];
  m->dim = (int)emb->second.shape[1];
  auto demb = T.find("decoder_Wemb");
  if (demb == T.end() || demb->second.shape.size() != 2) return "missing tensor decoder_Wemb";
  m->vocab_tgt = (int)demb->second.shape[0];
  auto w1 = T.find("encoder_l1_ffn_W1");
  if (w1 == T.end() || w1->second.shape.size() != 2) return "missing tensor encoder_l1_ffn_W1";
  m->ffn = (int)w1->second.shape[1];
  m->enc_layers = 0;
  while (T.count("encoder_l" + std::to_string(m->enc_layers + 1) + "_self_Wq")) ++m->enc_layers;
  int ssru = 0, self = 0;
  while (T.count("decoder_l" + std::to_string(ssru + 1) + "_rnn_W")) ++ssru;
  while (T.count("decoder_l" + std::to_string(self + 1) + "_self_Wq")) ++self;
  if ((ssru > 0) == (self > 0)) return "decoder must be all SSRU or all self-attention layers";
  m->decoder_kind = self > 0 ? 1 : 0;
  m->dec_layers = self > 0 ? self : ssru;
  if (m->enc_layers < 1 || m->dec_layers < 1 || m->enc_layers > 16 || m->dec_layers > 4)
    return "unsupported layer counts";
  // heads from the embedded model.yml
  m->heads = 8;
  auto yml = T.find("special:model.yml");
  if (yml == T.end() || yml->second.type != TensorType::Int8)
    return "special:model.yml must be a raw int8 byte tensor";
  {
    std::string text(reinterpret_cast<const char*>(yml->second.i8.data()), yml->second.i8.size());
    auto p = text.find("transformer-heads:");
    if (p != std::string::npos) m->heads = std::atoi(text.c_str() + p + 18);
  }
  const int d = m->dim, f = m->ffn;
  // the kernels take d a multiple of 128 up to 1024, head dims 32/48/64 and
  // heads in groups of 4 (the shipped graph: d 384, 8 heads of 48)
  if (m->heads <= 0 || d % m->heads != 0 || d % 128 != 0 || f % 16 != 0 || d > 1024 ||
      (d / m->heads != 32 && d / m->heads != 48 && d / m->heads != 64) || m->heads > 16 ||
      m->heads % 4 != 0)
    return "unsupported dimensions";
  if (m->vocab_src <= 2 || m->vocab_tgt <= 2)
    return "unsupported vocabulary size";
  std::set<std::string> expected = {"encoder_Wemb", "decoder_Wemb", "decoder_Wemb_QuantMultA",
                                    "decoder_ff_logit_out_b", "special:model.yml"};
  std::string e;
  const auto I8 = TensorType::Intgemm8, F32 = TensorType::Float32;
  auto dense = [&](const std::string& n, int in, int out, const char* bias) -> std::string {
    add_dense(&expected, n);
    std::string err = expect_shape(*m, n, {in, out}, I8);
    if (err.empty() && T.count(n + kRowSuffix)) {  // optional per-row multipliers
      expected.insert(n + kRowSuffix);
      err = expect_shape(*m, n + kRowSuffix, {1, out}, F32);
    }
    if (err.empty() && bias) {
      expected.insert(bias);
      err = expect_shape(*m, bias, {1, out}, F32);
    }
    float a;
    if (err.empty()) err = activation_scale(*m, n, &a);
    return err;
  };
  auto ln = [&](const std::string& p) -> std::string {
    expected.insert(p + "_scale");
    expected.insert(p + "_bias");
    std::string err = expect_shape(*m, p + "_scale", {1, d}, F32);
    if (err.empty()) err = expect_shape(*m, p + "_bias", {1, d}, F32);
    return err;
  };
  auto attention = [&](const std::string& p) -> std::string {
    for (const char* w : {"q", "k", "v", "o"}) {
      std::string err = dense(p + "_W" + w, d, d, (p + "_b" + w).c_str());
      if (!err.empty()) return err;
    }
    return ln(p + "_Wo_ln");
  };
  auto ffn = [&](const std::string& p) -> std::string {
    std::string err = dense(p + "_W1", d, f, (p + "_b1").c_str());
    if (err.empty()) err = dense(p + "_W2", f, d, (p + "_b2").c_str());
    if (err.empty()) err = ln(p + "_ffn_ln");
    return err;
  };
  if (!(e = expect_shape(*m, "encoder_Wemb", {m->vocab_src, d}, I8)).empty()) return e;
  if (!(e = expect_shape(*m, "decoder_Wemb", {m->vocab_tgt, d}, I8)).empty()) return e;
  if (!(e = expect_shape(*m, "decoder_ff_logit_out_b", {1, m->vocab_tgt}, F32)).empty()) return e;
  float a;
  if (!(e = activation_scale(*m, "decoder_Wemb", &a)).empty()) return e;
  for (int l = 1; l <= m->enc_layers; ++l) {
    const std::string p = "encoder_l" + std::to_string(l);
    if (!(e = attention(p + "_self")).empty()) return e;
    if (!(e = ffn(p + "_ffn")).empty()) return e;
  }
  for (int l = 1; l <= m->dec_layers; ++l) {
    const std::string p = "decoder_l" + std::to_string(l);
    if (m->decoder_kind == 0) {
      if (!(e = dense(p + "_rnn_W", d, d, nullptr)).empty()) return e;
      if (!(e = dense(p + "_rnn_Wf", d, d, (p + "_rnn_bf").c_str())).empty()) return e;
      if (!(e = ln(p + "_rnn_ffn_ln")).empty()) return e;
    } else {
      if (!(e = attention(p + "_self")).empty()) return e;
    }
    if (!(e = attention(p + "_context")).empty()) return e;
    if (!(e = ffn(p + "_ffn")).empty()) return e;
  }
  for (const auto& kv : T)
    if (!expected.count(kv.first)) return "unexpected tensor " + kv.first;
  if (expected.size() != T.size()) return "tensor schema mismatch";
  Q8Inventory inv;
  return validate_q8(*m, &inv);
}

}  // namespace mc

// Host-only inspection of a model file: MarianBinaryModel::parse and
// validate_q8 (legacy_q8.rs:179-422, 497-542), then the engine's schema
// check.  No device is touched.
extern "C" mc_status mc_inspect_marian_bin(const uint8_t* bytes, size_t len, mc_model_report* report,
                                           char* message, size_t message_capacity) {
  auto say = [&](const std::string& text) {
    if (message && message_capacity) {
      const size_t n = std::min(message_capacity - 1, text.size());
      std::memcpy(message, text.data(), n);
      message[n] = 0;
    }
  };
  say("");
  if (!bytes || !report) return MC_INVALID_INPUT;
  *report = mc_model_report();
  mc::HostModel m;
  std::string err = mc::parse_marian_v1(bytes, len, &m);
  mc::Q8Inventory inv;
  if (err.empty()) err = mc::validate_q8(m, &inv);
  if (!err.empty()) {
    say(err);
    return MC_MODEL;
  }
  report->tensors = m.order.size();
  report->dense_linears = inv.dense_linears;
  report->embeddings = inv.embeddings;
  report->activation_scales = inv.activation_scales;
  report->row_scaled_linears = inv.row_scaled;
  float alpha = 0.0f;
  if (m.tensors.count("decoder_Wemb_QuantMultA") && mc::activation_scale(m, "decoder_Wemb", &alpha).empty())
    report->decoder_output_alpha = alpha;
  const std::string schema = mc::validate_schema(&m);
  if (schema.empty()) {
    report->engine_graph = 1;
    report->decoder_kind = m.decoder_kind;
    report->dim = m.dim;
    report->heads = m.heads;
    report->encoder_layers = m.enc_layers;
    report->decoder_layers = m.dec_layers;
  } else {
    say(schema);  // a valid Q8 file the engine cannot run: why
  }
  return MC_OK;
}
