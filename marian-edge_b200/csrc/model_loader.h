// model_loader.h -- strict reader of Marian binary format v1 and the Q8
// tensor schema the engine consumes.
//
// Parsing rules restate crates/marian-cpu/src/legacy_q8.rs:179-422 (header,
// names, shapes, 256-byte data alignment, zero padding, per-type record
// lengths, intgemm8 trailing quant_mult, rejection of -128) and
// legacy_q8.rs:549-552/646-674 (activation alphas, including the
// accidentally quantized decoder_Wemb_QuantMultA normalised as q/quant_mult).
#pragma once

#include <cstdint>
#include <map>
#include <string>
#include <vector>

namespace mc {

enum class TensorType { Int8, Float32, Intgemm8 };

struct HostTensor {
  std::string name;
  TensorType type;
  std::vector<int64_t> shape;
  std::vector<int8_t> i8;     // Int8 / Intgemm8 values
  std::vector<float> f32;     // Float32 values
  float quant_mult = 1.0f;    // Intgemm8
  int64_t elements() const {
    int64_t n = 1;
    for (auto d : shape) n *= d;
    return n;
  }
};

struct HostModel {
  std::map<std::string, HostTensor> tensors;
  std::vector<std::string> order;
  int dim = 0, heads = 0, ffn = 0, enc_layers = 0, dec_layers = 0, vocab_src = 0, vocab_tgt = 0;
  int decoder_kind = 0;  // 0 SSRU, 1 self-attention
};

// Returns an empty string on success, else the reason.
std::string parse_marian_v1(const uint8_t* data, size_t len, HostModel* out);

// Resolves the static activation alpha of a Q8 weight (<name>_QuantMultA).
std::string activation_scale(const HostModel& m, const std::string& weight, float* alpha);

// Q8 inventory of a parsed file (MarianBinaryModel::validate_q8,
// legacy_q8.rs:497-542): every *_QuantMultA is a valid scalar scale of an
// intgemm8 weight, every intgemm8 tensor is rank 2, every dense one (not
// *_Wemb) has its activation scale, and at least one intgemm8 tensor
// exists.  Also checks the per-row extension: <weight>_QuantMultRows must
// be a finite, positive float32 [1, out] (or [out]) vector of an intgemm8
// dense weight whose header shape is [in, out].
struct Q8Inventory {
  uint64_t dense_linears = 0, embeddings = 0, activation_scales = 0, row_scaled = 0;
};
std::string validate_q8(const HostModel& m, Q8Inventory* inv);

// Per-output-row weight multipliers of a dense Q8 weight (the extension
// above), or an empty vector when the weight has one multiplier per tensor.
std::vector<float> weight_row_mults(const HostModel& m, const std::string& weight);

// Infers the graph (dims, layer counts, decoder kind, heads from
// special:model.yml "transformer-heads") and checks that the tensor set is
// exactly the schema of that graph (q8_engine.rs:1007-1101) with the expected
// shapes.
std::string validate_schema(HostModel* m);

}  // namespace mc
