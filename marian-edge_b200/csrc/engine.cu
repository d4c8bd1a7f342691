// engine.cu -- the marian_cuda engine: model upload, packed varlen encoder,
// paged cross/self caches, and a continuous-batching greedy decoder.
//
// Control flow restated from Q8CpuEngine::translate_token_ids
// (crates/marian-cpu/src/q8_engine.rs:353-466) with three B200 changes:
//   * sources are packed without padding (cu_seqlens) instead of [B, Lmax];
//   * cross keys/values and (for the self-attention decoder) self
//     keys/values live in pools of fixed-size pages addressed through
//     per-slot page tables;
//   * decode rows are the active slots only: finished rows retire at once and
//     queued requests are admitted into free slots between steps
//     (the reference keeps computing finished rows, q8_engine.rs:438-441).
#include <cmath>
#include <cstdio>
#include <cstring>
#include <deque>
#include <string>
#include <unordered_map>
#include <vector>

#include "common.cuh"
#include "kernels.cuh"
#include "marian_cuda.h"
#include "model_loader.h"
#include "q8_gemm.cuh"

namespace {

using namespace mc;

constexpr int kBNs[3] = {64, 128, 256};

int bn_index(int bn) { return bn == 64 ? 0 : (bn == 128 ? 1 : 2); }

struct DevLinear {
  int8_t* w = nullptr;
  float* col_scale = nullptr;  // [out] = 1 / (alpha * weight_mult)
  float* bias = nullptr;       // [out] or null
  int in = 0, out = 0;
  float alpha = 1.0f;          // this linear's own activation alpha
  float scale = 1.0f;          // 1 / (alpha * weight quant_mult)
  CUtensorMap tmap_b[3];       // W tensor maps for BN = 64, 128, 256
};

struct DevAttention {
  DevLinear wq, wk, wv, wo;
  float *ln_g = nullptr, *ln_b = nullptr;
};
struct DevFfn {
  DevLinear w1, w2;
  float *ln_g = nullptr, *ln_b = nullptr;
};
struct DevSsru {
  DevLinear w, wf;
  float *ln_g = nullptr, *ln_b = nullptr;
};

// An activation buffer that feeds GEMMs: int8 [rows, cols] with its A map.
struct QBuf {
  int8_t* p = nullptr;
  int rows = 0, cols = 0;
  CUtensorMap tmap;
};

struct Request {
  uint64_t id;
  std::vector<int32_t> tokens;
  uint32_t max_out, force;
  std::vector<int32_t> output;
  int slot = -1;
  std::vector<int32_t> cross_pages, self_pages;
};

struct Finished {
  uint64_t id;
  std::vector<int32_t> tokens;
};

}  // namespace

struct mc_engine {
  mc_config cfg{};
  std::string error;
  bool ready = true;
  bool loaded = false;
  cudaStream_t stream = nullptr;
  uint32_t* d_status = nullptr;
  HostModel host;  // dims; tensor payloads are released after upload
  int d = 0, heads = 0, ffn = 0, enc_layers = 0, dec_layers = 0, kind = 0, vsrc = 0, vtgt = 0;
  float emb_scale = 1.0f;
  uint64_t weight_bytes = 0;

  // device weights
  std::vector<void*> allocations;
  int8_t* enc_emb = nullptr;
  float enc_emb_mult = 1.0f;
  int8_t* dec_emb = nullptr;
  float dec_emb_mult = 1.0f;
  DevLinear vocab;  // tied output projection over decoder_Wemb
  uint32_t* cand_bits = nullptr;
  float* positions = nullptr;
  std::vector<DevAttention> enc_attn, dec_self, dec_ctx;
  std::vector<DevFfn> enc_ffn, dec_ffn;
  std::vector<DevSsru> dec_ssru;

  // encoder buffers (capacity tmax packed tokens)
  int tmax = 0;
  float *enc_x = nullptr, *enc_x1 = nullptr, *enc_qkv = nullptr, *enc_proj = nullptr;
  QBuf enc_q[kMaxQuantOut];
  QBuf enc_o, enc_h;
  int32_t *enc_tokens = nullptr, *enc_pos = nullptr, *enc_cu = nullptr, *enc_cross_rows = nullptr;
  int32_t* enc_seq_ids = nullptr;  // admitted sequences grouped by length bucket
  struct Bucket {
    int offset, count, max_len;
  };
  std::vector<Bucket> buckets;

  // decoder buffers (capacity rmax rows = slots)
  int rmax = 0;
  float *dec_a = nullptr, *dec_b = nullptr, *dec_qkv = nullptr, *dec_proj = nullptr;
  QBuf dec_q[kMaxQuantOut];
  QBuf dec_o, dec_h;
  int32_t *row_slot = nullptr, *self_row_map = nullptr, *step_tokens = nullptr;
  int32_t *order_self = nullptr, *order_cross = nullptr;  // rows, longest keys first
  uint8_t *eos_mask = nullptr, *done = nullptr;
  unsigned long long* best = nullptr;

  // slots and caches
  int32_t *slot_prev = nullptr, *slot_step = nullptr, *slot_limit = nullptr, *slot_force = nullptr,
          *slot_src = nullptr;
  float* ssru_state = nullptr;
  int pages_per_slot = 0, page_tokens = 16;
  int cross_pool_pages = 0, self_pool_pages = 0;
  int32_t *cross_pages_d = nullptr, *self_pages_d = nullptr;
  std::vector<int32_t> cross_pages_h, self_pages_h;
  std::vector<float*> cross_k, cross_v, self_k, self_v;
  std::vector<int32_t> free_cross, free_self, free_slots;
  bool pages_dirty = true;

  // pinned staging
  int32_t* h_i32 = nullptr;  // staging for uploads
  size_t h_i32_cap = 0;
  int32_t* h_step_tokens = nullptr;
  uint8_t* h_done = nullptr;
  uint32_t* h_status = nullptr;

  // scheduler
  std::deque<Request*> queue;
  std::vector<Request*> slot_req;    // [rmax]
  std::vector<int32_t> active;       // slots in row order
  std::vector<Finished> finished;
  uint64_t steps = 0, launches = 0;
  float* last_state = nullptr;  // final decoder state buffer of the last step

  // admission staging on the device
  int32_t *adm_slots = nullptr, *adm_limits = nullptr, *adm_force = nullptr, *adm_src = nullptr;

  // optional per-kernel-class timing (mc_profile): CUDA event pairs on the
  // engine stream around each launch, harvested after each synchronization
  struct ProfRec {
    int kind;
    double flops, bytes;
    cudaEvent_t a, b;
  };
  bool profiling = false;
  std::vector<ProfRec> prof_pending;
  std::vector<cudaEvent_t> event_pool;
  double prof_ms[MC_KERNEL_KINDS] = {}, prof_flops[MC_KERNEL_KINDS] = {}, prof_bytes[MC_KERNEL_KINDS] = {};
  uint64_t prof_n[MC_KERNEL_KINDS] = {};

  ~mc_engine();
};

namespace {

#define CK(call)                                                                  \
  do {                                                                            \
    cudaError_t e_ = (call);                                                      \
    if (e_ != cudaSuccess) return fail_cuda(e, #call, e_);                        \
  } while (0)

mc_status fail(mc_engine* e, mc_status st, const std::string& msg) {
  e->error = msg;
  return st;
}

mc_status fail_cuda(mc_engine* e, const char* what, cudaError_t err) {
  e->error = std::string(what) + ": " + cudaGetErrorString(err);
  e->ready = false;
  return MC_CUDA;
}

int prof_begin(mc_engine* e, int kind, double flops, double bytes) {
  if (!e->profiling) return -1;
  auto ev = [&]() {
    cudaEvent_t x;
    if (!e->event_pool.empty()) {
      x = e->event_pool.back();
      e->event_pool.pop_back();
    } else {
      cudaEventCreate(&x);
    }
    return x;
  };
  mc_engine::ProfRec r{kind, flops, bytes, ev(), ev()};
  cudaEventRecord(r.a, e->stream);
  e->prof_pending.push_back(r);
  return (int)e->prof_pending.size() - 1;
}

void prof_end(mc_engine* e, int idx) {
  if (idx >= 0) cudaEventRecord(e->prof_pending[idx].b, e->stream);
}

// Call after the engine stream is synchronized.
void prof_harvest(mc_engine* e) {
  for (auto& r : e->prof_pending) {
    float ms = 0.0f;
    if (cudaEventElapsedTime(&ms, r.a, r.b) == cudaSuccess) {
      e->prof_ms[r.kind] += ms;
      e->prof_flops[r.kind] += r.flops;
      e->prof_bytes[r.kind] += r.bytes;
      e->prof_n[r.kind] += 1;
    }
    e->event_pool.push_back(r.a);
    e->event_pool.push_back(r.b);
  }
  e->prof_pending.clear();
}

#define PROFILED(kind, flops, bytes, stmt)                     \
  do {                                                         \
    const int pi_ = prof_begin(e, (kind), (flops), (bytes));   \
    stmt;                                                      \
    prof_end(e, pi_);                                          \
  } while (0)

template <class T>
cudaError_t dalloc(mc_engine* e, T** p, size_t count) {
  void* q = nullptr;
  cudaError_t r = cudaMalloc(&q, count * sizeof(T) + 256);
  if (r == cudaSuccess) {
    cudaMemsetAsync(q, 0, count * sizeof(T) + 256, e->stream);
    e->allocations.push_back(q);
    *p = static_cast<T*>(q);
  }
  return r;
}

// Host-to-device copy on the engine stream (ordered after dalloc's memset),
// synchronous because the source is usually a temporary.
cudaError_t h2d(mc_engine* e, void* dst, const void* src, size_t bytes) {
  cudaError_t r = cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, e->stream);
  if (r == cudaSuccess) r = cudaStreamSynchronize(e->stream);
  return r;
}

// marian-model/src/position.rs:5-21, computed on the host with the C
// library's expf/sinf/cosf/logf (the functions Rust's f32 methods call).
std::vector<float> sinusoidal_positions(int dim) {
  std::vector<float> v((size_t)kMaxPosition * dim);
  const int half = dim / 2;
  const float ln1e4 = logf(10000.0f);
  for (int p = 0; p < kMaxPosition; ++p)
    for (int i = 0; i < half; ++i) {
      volatile float num = -(float)i * ln1e4;
      const float frequency = expf(num / (float)(half - 1));
      volatile float arg = (float)p * frequency;
      v[(size_t)p * dim + i] = sinf(arg);
      v[(size_t)p * dim + half + i] = cosf(arg);
    }
  return v;
}

mc_status upload_linear(mc_engine* e, const std::string& wname, const char* bname, DevLinear* L) {
  const HostTensor& w = e->host.tensors.at(wname);
  L->in = (int)w.shape[0];
  L->out = (int)w.shape[1];
  std::string err = activation_scale(e->host, wname, &L->alpha);
  if (!err.empty()) return fail(e, MC_MODEL, err);
  CK(dalloc(e, &L->w, w.i8.size()));
  CK(cudaMemcpyAsync(L->w, w.i8.data(), w.i8.size(), cudaMemcpyHostToDevice, e->stream));
  const float inv = 1.0f / (L->alpha * w.quant_mult);  // q8_gemm.rs:438
  L->scale = inv;
  std::vector<float> cs(L->out, inv);
  CK(dalloc(e, &L->col_scale, cs.size()));
  CK(cudaMemcpyAsync(L->col_scale, cs.data(), cs.size() * 4, cudaMemcpyHostToDevice, e->stream));
  if (bname) {
    const HostTensor& b = e->host.tensors.at(bname);
    CK(dalloc(e, &L->bias, b.f32.size()));
    CK(cudaMemcpyAsync(L->bias, b.f32.data(), b.f32.size() * 4, cudaMemcpyHostToDevice, e->stream));
  }
  CK(cudaStreamSynchronize(e->stream));  // host vectors above are temporaries
  e->weight_bytes += w.i8.size() + (size_t)L->out * 4 * (bname ? 2 : 1);
  for (int i = 0; i < 3; ++i)
    if (!encode_tmap_i8(&L->tmap_b[i], L->w, L->out, L->in, kBNs[i]))
      return fail(e, MC_MODEL, wname + ": tensor map rejected");
  return MC_OK;
}

mc_status upload_f32(mc_engine* e, const std::string& name, float** out) {
  const HostTensor& t = e->host.tensors.at(name);
  CK(dalloc(e, out, t.f32.size()));
  CK(h2d(e, *out, t.f32.data(), t.f32.size() * 4));
  e->weight_bytes += t.f32.size() * 4;
  return MC_OK;
}

mc_status upload_attention(mc_engine* e, const std::string& p, DevAttention* a) {
  mc_status st;
  if ((st = upload_linear(e, p + "_Wq", (p + "_bq").c_str(), &a->wq))) return st;
  if ((st = upload_linear(e, p + "_Wk", (p + "_bk").c_str(), &a->wk))) return st;
  if ((st = upload_linear(e, p + "_Wv", (p + "_bv").c_str(), &a->wv))) return st;
  if ((st = upload_linear(e, p + "_Wo", (p + "_bo").c_str(), &a->wo))) return st;
  if ((st = upload_f32(e, p + "_Wo_ln_scale", &a->ln_g))) return st;
  return upload_f32(e, p + "_Wo_ln_bias", &a->ln_b);
}

mc_status upload_ffn(mc_engine* e, const std::string& p, DevFfn* f) {
  mc_status st;
  if ((st = upload_linear(e, p + "_W1", (p + "_b1").c_str(), &f->w1))) return st;
  if ((st = upload_linear(e, p + "_W2", (p + "_b2").c_str(), &f->w2))) return st;
  if ((st = upload_f32(e, p + "_ffn_ln_scale", &f->ln_g))) return st;
  return upload_f32(e, p + "_ffn_ln_bias", &f->ln_b);
}

mc_status make_qbuf(mc_engine* e, QBuf* q, int rows, int cols) {
  CK(dalloc(e, &q->p, (size_t)rows * cols));
  q->rows = rows;
  q->cols = cols;
  if (!encode_tmap_i8(&q->tmap, q->p, rows, cols, 128)) return fail(e, MC_MODEL, "activation tensor map rejected");
  return MC_OK;
}

// ---- GEMM launch helpers ---------------------------------------------------
struct GroupSpec {
  const QBuf* a;
  const DevLinear* w;
  int mode;
  void* out;
  int ldo, col_off;
  const int32_t* row_map;
  bool relu;
  float alpha;  // next linear's alpha (kEpiQ8)
};

mc_status gemm(mc_engine* e, int kind, int m, const GroupSpec* specs, int n_groups,
               unsigned long long* argmax = nullptr, const uint8_t* eos = nullptr) {
  if (m <= 0) return MC_OK;
  GemmParams p;
  std::memset(&p, 0, sizeof(p));
  int max_n = 0;
  for (int i = 0; i < n_groups; ++i) max_n = std::max(max_n, specs[i].w->out);
  const int bn = pick_bn(m, max_n);
  for (int i = 0; i < n_groups; ++i) {
    const GroupSpec& s = specs[i];
    GemmGroup& g = p.g[i];
    g.tmap_a = s.a->tmap;
    g.tmap_b = s.w->tmap_b[bn_index(bn)];
    g.col_scale = nullptr;  // per-tensor weight scale (q8_gemm.rs:438)
    g.uniform_scale = s.w->scale;
    g.bias = s.w->bias;
    g.out = s.out;
    g.row_map = s.row_map;
    g.n = s.w->out;
    g.ldo = s.ldo;
    g.col_off = s.col_off;
    g.alpha = s.alpha;
    g.mode = s.mode;
    g.relu = s.relu;
    g.argmax = argmax;
    g.cand_bits = e->cand_bits;
    g.eos_mask = eos;
  }
  p.m = m;
  p.k = specs[0].w->in;
  p.num_groups = n_groups;
  p.max_n = max_n;
  p.status = e->d_status;
  double flops = 0, bytes = 0;
  for (int i = 0; i < n_groups; ++i) {
    const double n = specs[i].w->out, k = specs[i].w->in;
    flops += 2.0 * m * n * k;
    const double out_bytes = specs[i].mode == kEpiArgmax ? 8.0 * m
                             : specs[i].mode == kEpiQ8   ? 1.0 * m * n
                                                         : 4.0 * m * n;
    bytes += (double)m * k + n * k + 4.0 * n * (specs[i].w->bias ? 2 : 1) + out_bytes;
  }
  PROFILED(kind, flops, bytes, CK(launch_q8_gemm(p, bn, e->stream)));
  ++e->launches;
  return MC_OK;
}

QuantOut quant_out(const QBuf* bufs, std::initializer_list<float> alphas) {
  QuantOut q;
  std::memset(&q, 0, sizeof(q));
  q.base = bufs[0].p;
  q.stride = bufs[1].p - bufs[0].p;
  q.count = 0;
  for (float a : alphas) q.alpha[q.count++] = a;
  return q;
}

QuantOut quant_out_vec(const QBuf* bufs, const std::vector<float>& alphas) {
  QuantOut q;
  std::memset(&q, 0, sizeof(q));
  q.base = bufs[0].p;
  q.stride = bufs[1].p - bufs[0].p;
  q.count = (int)alphas.size();
  for (size_t i = 0; i < alphas.size(); ++i) q.alpha[i] = alphas[i];
  return q;
}

// Alphas of the linears that read the encoder layer input / decoder layer input.
std::vector<float> enc_input_alphas(mc_engine* e, int layer) {
  if (layer < e->enc_layers) {
    const DevAttention& a = e->enc_attn[layer];
    return {a.wq.alpha, a.wk.alpha, a.wv.alpha};
  }
  std::vector<float> v;  // after the last layer: cross K/V of every decoder layer
  for (int l = 0; l < e->dec_layers; ++l) {
    v.push_back(e->dec_ctx[l].wk.alpha);
    v.push_back(e->dec_ctx[l].wv.alpha);
  }
  return v;
}

std::vector<float> dec_input_alphas(mc_engine* e, int layer) {
  if (layer >= e->dec_layers) return {e->vocab.alpha};
  if (e->kind == 0) return {e->dec_ssru[layer].w.alpha, e->dec_ssru[layer].wf.alpha};
  const DevAttention& a = e->dec_self[layer];
  return {a.wq.alpha, a.wk.alpha, a.wv.alpha};
}

// ---- encoder pass over packed admitted sources ------------------------------
mc_status run_encoder(mc_engine* e, int T, int batch, int max_len, double sum_len_sq) {
  const int d = e->d;
  const double rows_d = (double)T * d;
  PROFILED(MC_K_EMBED, 0.0, rows_d * (1 + 4 + 4 + 3),
           launch_embed_encoder(e->enc_tokens, e->enc_pos, T, e->enc_emb, e->enc_emb_mult,
                                e->emb_scale, e->positions, d, e->enc_x,
                                quant_out_vec(e->enc_q, enc_input_alphas(e, 0)), e->d_status,
                                e->stream));
  ++e->launches;
  mc_status st;
  for (int l = 0; l < e->enc_layers; ++l) {
    const DevAttention& a = e->enc_attn[l];
    const DevFfn& f = e->enc_ffn[l];
    GroupSpec qkv[3] = {
        {&e->enc_q[0], &a.wq, kEpiF32, e->enc_qkv, 3 * d, 0, nullptr, false, 0.f},
        {&e->enc_q[1], &a.wk, kEpiF32, e->enc_qkv, 3 * d, d, nullptr, false, 0.f},
        {&e->enc_q[2], &a.wv, kEpiF32, e->enc_qkv, 3 * d, 2 * d, nullptr, false, 0.f}};
    if ((st = gemm(e, MC_K_GEMM_QKV, T, qkv, 3))) return st;
    PROFILED(MC_K_ATTN_ENC, 4.0 * sum_len_sq * d, rows_d * (12 + 1), {
      for (const auto& bk : e->buckets)
        CK(launch_attn_encoder(e->enc_qkv, e->enc_cu, e->enc_seq_ids + bk.offset, bk.count,
                               bk.max_len, d, e->heads, e->enc_o.p, a.wo.alpha, e->d_status,
                               e->stream));
    });
    ++e->launches;
    GroupSpec wo = {&e->enc_o, &a.wo, kEpiF32, e->enc_proj, d, 0, nullptr, false, 0.f};
    if ((st = gemm(e, MC_K_GEMM_OUT, T, &wo, 1))) return st;
    PROFILED(MC_K_LAYERNORM, 0.0, rows_d * 13,
             launch_residual_ln(e->enc_proj, d, e->enc_x, d, a.ln_g, a.ln_b, T, d, e->enc_x1,
                                quant_out(e->enc_q, {f.w1.alpha}), e->d_status, e->stream));
    GroupSpec w1 = {&e->enc_q[0], &f.w1, kEpiQ8, e->enc_h.p, e->ffn, 0, nullptr, true, f.w2.alpha};
    if ((st = gemm(e, MC_K_GEMM_FFN1, T, &w1, 1))) return st;
    GroupSpec w2 = {&e->enc_h, &f.w2, kEpiF32, e->enc_proj, d, 0, nullptr, false, 0.f};
    if ((st = gemm(e, MC_K_GEMM_FFN2, T, &w2, 1))) return st;
    PROFILED(MC_K_LAYERNORM, 0.0, rows_d * (12 + enc_input_alphas(e, l + 1).size()),
             launch_residual_ln(e->enc_proj, d, e->enc_x1, d, f.ln_g, f.ln_b, T, d, e->enc_x,
                                quant_out_vec(e->enc_q, enc_input_alphas(e, l + 1)), e->d_status,
                                e->stream));
    e->launches += 2;
  }
  // cross keys/values of every decoder layer into the paged pools
  // (q8_engine.rs:560-567)
  std::vector<GroupSpec> cross;
  for (int l = 0; l < e->dec_layers; ++l) {
    cross.push_back({&e->enc_q[2 * l], &e->dec_ctx[l].wk, kEpiF32, e->cross_k[l], d, 0,
                     e->enc_cross_rows, false, 0.f});
    cross.push_back({&e->enc_q[2 * l + 1], &e->dec_ctx[l].wv, kEpiF32, e->cross_v[l], d, 0,
                     e->enc_cross_rows, false, 0.f});
  }
  for (size_t i = 0; i < cross.size(); i += kMaxGemmGroups)
    if ((st = gemm(e, MC_K_GEMM_CROSSKV, T, cross.data() + i, (int)std::min<size_t>(kMaxGemmGroups, cross.size() - i))))
      return st;
  return MC_OK;
}

// ---- one decode step over the active rows --------------------------------------
mc_status run_decode_step(mc_engine* e, int R) {
  const int d = e->d;
  float* x = e->dec_a;   // layer input
  float* y = e->dec_b;   // next
  // key counts for the attention roofline: self = step + 1, cross = source
  double self_keys = 0, cross_keys = 0;
  for (int s : e->active) {
    const Request* q = e->slot_req[s];
    if (!q) continue;
    self_keys += (double)q->output.size() + 1;
    cross_keys += (double)q->tokens.size();
  }
  const double rows_d = (double)R * d;
  PROFILED(MC_K_EMBED, 0.0, rows_d * (1 + 4 + 4 + 3),
           launch_embed_decoder(R, e->row_slot, e->slot_prev, e->slot_step, e->slot_force,
                                e->dec_emb, e->dec_emb_mult, e->emb_scale, e->positions, d, x,
                                quant_out_vec(e->dec_q, dec_input_alphas(e, 0)), e->eos_mask,
                                e->kind == 1 ? e->self_pages_d : nullptr, e->pages_per_slot,
                                e->page_tokens, e->self_row_map, e->d_status, e->stream));
  ++e->launches;
  mc_status st;
  for (int l = 0; l < e->dec_layers; ++l) {
    const DevAttention& c = e->dec_ctx[l];
    const DevFfn& f = e->dec_ffn[l];
    if (e->kind == 1) {
      const DevAttention& a = e->dec_self[l];
      GroupSpec qkv[3] = {
          {&e->dec_q[0], &a.wq, kEpiF32, e->dec_qkv, d, 0, nullptr, false, 0.f},
          {&e->dec_q[1], &a.wk, kEpiF32, e->self_k[l], d, 0, e->self_row_map, false, 0.f},
          {&e->dec_q[2], &a.wv, kEpiF32, e->self_v[l], d, 0, e->self_row_map, false, 0.f}};
      if ((st = gemm(e, MC_K_GEMM_QKV, R, qkv, 3))) return st;
      PROFILED(MC_K_ATTN_SELF, 4.0 * self_keys * d, 8.0 * self_keys * d + rows_d * 5,
               CK(launch_attn_decode(e->dec_qkv, d, R, e->row_slot, e->order_self, e->slot_step, 1,
                                     e->self_pages_d, e->pages_per_slot, e->page_tokens,
                                     e->self_k[l], e->self_v[l], d, e->heads, e->dec_o.p,
                                     a.wo.alpha, e->d_status, e->stream)));
      GroupSpec wo = {&e->dec_o, &a.wo, kEpiF32, e->dec_proj, d, 0, nullptr, false, 0.f};
      if ((st = gemm(e, MC_K_GEMM_OUT, R, &wo, 1))) return st;
      PROFILED(MC_K_LAYERNORM, 0.0, rows_d * 13,
               launch_residual_ln(e->dec_proj, d, x, d, a.ln_g, a.ln_b, R, d, y,
                                  quant_out(e->dec_q, {c.wq.alpha}), e->d_status, e->stream));
      e->launches += 2;
    } else {
      const DevSsru& s = e->dec_ssru[l];
      GroupSpec wf[2] = {
          {&e->dec_q[0], &s.w, kEpiF32, e->dec_qkv, 2 * d, 0, nullptr, false, 0.f},
          {&e->dec_q[1], &s.wf, kEpiF32, e->dec_qkv, 2 * d, d, nullptr, false, 0.f}};
      if ((st = gemm(e, MC_K_GEMM_QKV, R, wf, 2))) return st;
      PROFILED(MC_K_SSRU, 0.0, rows_d * 25,
               launch_ssru(e->dec_qkv, 2 * d, d, e->ssru_state + (size_t)l * e->rmax * d,
                           e->row_slot, x, s.ln_g, s.ln_b, R, d, y,
                           quant_out(e->dec_q, {c.wq.alpha}), e->d_status, e->stream));
      ++e->launches;
    }
    std::swap(x, y);
    GroupSpec wq = {&e->dec_q[0], &c.wq, kEpiF32, e->dec_qkv, d, 0, nullptr, false, 0.f};
    if ((st = gemm(e, MC_K_GEMM_QKV, R, &wq, 1))) return st;
    PROFILED(MC_K_ATTN_CROSS, 4.0 * cross_keys * d, 8.0 * cross_keys * d + rows_d * 5,
             CK(launch_attn_decode(e->dec_qkv, d, R, e->row_slot, e->order_cross, e->slot_src, 0,
                                   e->cross_pages_d, e->pages_per_slot, e->page_tokens,
                                   e->cross_k[l], e->cross_v[l], d, e->heads, e->dec_o.p,
                                   c.wo.alpha, e->d_status, e->stream)));
    GroupSpec wo = {&e->dec_o, &c.wo, kEpiF32, e->dec_proj, d, 0, nullptr, false, 0.f};
    if ((st = gemm(e, MC_K_GEMM_OUT, R, &wo, 1))) return st;
    PROFILED(MC_K_LAYERNORM, 0.0, rows_d * 13,
             launch_residual_ln(e->dec_proj, d, x, d, c.ln_g, c.ln_b, R, d, y,
                                quant_out(e->dec_q, {f.w1.alpha}), e->d_status, e->stream));
    std::swap(x, y);
    GroupSpec w1 = {&e->dec_q[0], &f.w1, kEpiQ8, e->dec_h.p, e->ffn, 0, nullptr, true, f.w2.alpha};
    if ((st = gemm(e, MC_K_GEMM_FFN1, R, &w1, 1))) return st;
    GroupSpec w2 = {&e->dec_h, &f.w2, kEpiF32, e->dec_proj, d, 0, nullptr, false, 0.f};
    if ((st = gemm(e, MC_K_GEMM_FFN2, R, &w2, 1))) return st;
    PROFILED(MC_K_LAYERNORM, 0.0, rows_d * (12 + dec_input_alphas(e, l + 1).size()),
             launch_residual_ln(e->dec_proj, d, x, d, f.ln_g, f.ln_b, R, d, y,
                                quant_out_vec(e->dec_q, dec_input_alphas(e, l + 1)), e->d_status,
                                e->stream));
    std::swap(x, y);
    e->launches += 3;
  }
  // tied vocabulary projection + masked argmax (q8_engine.rs:749-790)
  GroupSpec voc = {&e->dec_q[0], &e->vocab, kEpiArgmax, nullptr, 0, 0, nullptr, false, 0.f};
  if ((st = gemm(e, MC_K_GEMM_VOCAB, R, &voc, 1, e->best, e->eos_mask))) return st;
  PROFILED(MC_K_FINALIZE, 0.0, (double)R * 29,
           launch_finalize(R, e->row_slot, e->best, e->slot_prev, e->slot_step, e->slot_limit,
                           e->step_tokens, e->done, e->d_status, e->stream));
  ++e->launches;
  e->last_state = x;
  return MC_OK;
}

}  // namespace

// ============================================================================
// engine lifecycle, scheduling and the C ABI
// ============================================================================

mc_engine::~mc_engine() {
  if (stream) cudaStreamSynchronize(stream);
  for (auto& r : prof_pending) {
    cudaEventDestroy(r.a);
    cudaEventDestroy(r.b);
  }
  for (cudaEvent_t ev : event_pool) cudaEventDestroy(ev);
  for (void* p : allocations) cudaFree(p);
  if (d_status) cudaFree(d_status);
  if (h_i32) cudaFreeHost(h_i32);
  if (h_step_tokens) cudaFreeHost(h_step_tokens);
  if (h_done) cudaFreeHost(h_done);
  if (h_status) cudaFreeHost(h_status);
  if (stream) cudaStreamDestroy(stream);
  for (Request* r : queue) delete r;
  for (Request* r : slot_req) delete r;
}

namespace {

mc_status set_device(mc_engine* e) {
  CK(cudaSetDevice(e->cfg.device));
  return MC_OK;
}

mc_status allocate_buffers(mc_engine* e) {
  const int d = e->d, F = e->ffn;
  const int T = e->tmax, R = e->rmax;
  CK(dalloc(e, &e->enc_x, (size_t)T * d));
  CK(dalloc(e, &e->enc_x1, (size_t)T * d));
  CK(dalloc(e, &e->enc_qkv, (size_t)T * 3 * d));
  CK(dalloc(e, &e->enc_proj, (size_t)T * d));
  // quantized copies: one contiguous block so copy i = base + i * stride
  int8_t* eq = nullptr;
  CK(dalloc(e, &eq, (size_t)kMaxQuantOut * T * d));
  for (int i = 0; i < kMaxQuantOut; ++i) {
    e->enc_q[i].p = eq + (size_t)i * T * d;
    e->enc_q[i].rows = T;
    e->enc_q[i].cols = d;
    if (!encode_tmap_i8(&e->enc_q[i].tmap, e->enc_q[i].p, T, d, 128)) return fail(e, MC_MODEL, "tensor map");
  }
  mc_status st;
  if ((st = make_qbuf(e, &e->enc_o, T, d))) return st;
  if ((st = make_qbuf(e, &e->enc_h, T, F))) return st;
  CK(dalloc(e, &e->enc_tokens, T));
  CK(dalloc(e, &e->enc_pos, T));
  CK(dalloc(e, &e->enc_cu, T + 1));
  CK(dalloc(e, &e->enc_cross_rows, T));
  CK(dalloc(e, &e->enc_seq_ids, R));

  CK(dalloc(e, &e->dec_a, (size_t)R * d));
  CK(dalloc(e, &e->dec_b, (size_t)R * d));
  CK(dalloc(e, &e->dec_qkv, (size_t)R * 3 * d));
  CK(dalloc(e, &e->dec_proj, (size_t)R * d));
  int8_t* dq = nullptr;
  CK(dalloc(e, &dq, (size_t)kMaxQuantOut * R * d));
  for (int i = 0; i < kMaxQuantOut; ++i) {
    e->dec_q[i].p = dq + (size_t)i * R * d;
    e->dec_q[i].rows = R;
    e->dec_q[i].cols = d;
    if (!encode_tmap_i8(&e->dec_q[i].tmap, e->dec_q[i].p, R, d, 128)) return fail(e, MC_MODEL, "tensor map");
  }
  if ((st = make_qbuf(e, &e->dec_o, R, d))) return st;
  if ((st = make_qbuf(e, &e->dec_h, R, F))) return st;
  CK(dalloc(e, &e->row_slot, R));
  CK(dalloc(e, &e->order_self, R));
  CK(dalloc(e, &e->order_cross, R));
  CK(dalloc(e, &e->self_row_map, R));
  CK(dalloc(e, &e->step_tokens, R));
  CK(dalloc(e, &e->eos_mask, R));
  CK(dalloc(e, &e->done, R));
  CK(dalloc(e, &e->best, R));
  CK(dalloc(e, &e->slot_prev, R));
  CK(dalloc(e, &e->slot_step, R));
  CK(dalloc(e, &e->slot_limit, R));
  CK(dalloc(e, &e->slot_force, R));
  CK(dalloc(e, &e->slot_src, R));
  CK(dalloc(e, &e->adm_slots, R));
  CK(dalloc(e, &e->adm_limits, R));
  CK(dalloc(e, &e->adm_force, R));
  CK(dalloc(e, &e->adm_src, R));
  if (e->kind == 0) CK(dalloc(e, &e->ssru_state, (size_t)e->dec_layers * R * d));

  e->page_tokens = (int)e->cfg.page_tokens;
  e->pages_per_slot = (kMaxSeq + e->page_tokens - 1) / e->page_tokens;
  const int pool = e->cfg.kv_pages ? (int)e->cfg.kv_pages : R * e->pages_per_slot;
  e->cross_pool_pages = pool;
  e->self_pool_pages = e->kind == 1 ? pool : 0;
  const size_t pool_rows = (size_t)pool * e->page_tokens;
  e->cross_k.resize(e->dec_layers);
  e->cross_v.resize(e->dec_layers);
  for (int l = 0; l < e->dec_layers; ++l) {
    CK(dalloc(e, &e->cross_k[l], pool_rows * d));
    CK(dalloc(e, &e->cross_v[l], pool_rows * d));
  }
  if (e->kind == 1) {
    e->self_k.resize(e->dec_layers);
    e->self_v.resize(e->dec_layers);
    for (int l = 0; l < e->dec_layers; ++l) {
      CK(dalloc(e, &e->self_k[l], pool_rows * d));
      CK(dalloc(e, &e->self_v[l], pool_rows * d));
    }
  }
  CK(dalloc(e, &e->cross_pages_d, (size_t)R * e->pages_per_slot));
  CK(dalloc(e, &e->self_pages_d, (size_t)R * e->pages_per_slot));
  e->cross_pages_h.assign((size_t)R * e->pages_per_slot, 0);
  e->self_pages_h.assign((size_t)R * e->pages_per_slot, 0);
  e->free_cross.clear();
  e->free_self.clear();
  for (int p = pool - 1; p >= 0; --p) e->free_cross.push_back(p);
  for (int p = e->self_pool_pages - 1; p >= 0; --p) e->free_self.push_back(p);
  e->free_slots.clear();
  for (int s = R - 1; s >= 0; --s) e->free_slots.push_back(s);
  e->slot_req.assign(R, nullptr);

  e->h_i32_cap = (size_t)4 * T + 6 * R + 16;
  CK(cudaHostAlloc(&e->h_i32, e->h_i32_cap * sizeof(int32_t), cudaHostAllocDefault));
  CK(cudaHostAlloc(&e->h_step_tokens, (size_t)R * sizeof(int32_t), cudaHostAllocDefault));
  CK(cudaHostAlloc(&e->h_done, (size_t)R, cudaHostAllocDefault));
  CK(cudaStreamSynchronize(e->stream));
  return MC_OK;
}

uint32_t request_limit(const mc_engine* e, const Request* r) {
  uint64_t lim = r->max_out;
  if (r->force > 0 && r->force < lim) lim = r->force;
  const uint64_t by_len = (uint64_t)r->tokens.size() * std::max<uint32_t>(1, e->cfg.max_length_factor);
  lim = std::min<uint64_t>(lim, by_len);
  lim = std::min<uint64_t>(lim, kMaxSeq);
  return (uint32_t)lim;
}

void release_slot(mc_engine* e, Request* r) {
  for (int p : r->cross_pages) e->free_cross.push_back(p);
  for (int p : r->self_pages) e->free_self.push_back(p);
  r->cross_pages.clear();
  r->self_pages.clear();
  if (r->slot >= 0) {
    e->slot_req[r->slot] = nullptr;
    e->free_slots.push_back(r->slot);
  }
  r->slot = -1;
}

void finish_request(mc_engine* e, Request* r) {
  release_slot(e, r);
  e->finished.push_back({r->id, std::move(r->output)});
  delete r;
}

// Drops every queued and in-flight request (after a failed step).
void abort_all(mc_engine* e) {
  for (Request* r : e->queue) delete r;
  e->queue.clear();
  for (int s : e->active) {
    Request* r = e->slot_req[s];
    if (r) {
      release_slot(e, r);
      delete r;
    }
  }
  e->active.clear();
}

mc_status check_status(mc_engine* e) {
  const uint32_t bits = *e->h_status;
  if (!bits) return MC_OK;
  *e->h_status = 0;
  CK(cudaMemsetAsync(e->d_status, 0, sizeof(uint32_t), e->stream));
  CK(cudaStreamSynchronize(e->stream));
  abort_all(e);
  if (bits & kStatusWaitTimeout) {
    e->ready = false;
    return fail(e, MC_DEVICE_TIMEOUT, "a device wait timed out");
  }
  if (bits & kStatusBadIndex) {
    e->ready = false;
    return fail(e, MC_INFERENCE, "a device index check failed");
  }
  return fail(e, MC_INFERENCE, "activation contains a non-finite value");
}

// Admits queued requests into free slots and runs one packed encoder pass.
mc_status admit(mc_engine* e, std::vector<Request*>* admitted) {
  int T = 0, max_len = 0;
  const int pt = e->page_tokens;
  // Admission granularity: an encoder pass over a handful of sources costs
  // nearly as much launch latency as one over hundreds, so wait until an
  // eighth of the slots are free -- unless nothing is running or the whole
  // queue fits (which keeps latency low under light load).
  const size_t free_slots = e->free_slots.size();
  if (!e->active.empty() && free_slots < (size_t)std::max(1, e->rmax / 8) &&
      e->queue.size() > free_slots)
    return MC_OK;
  while (!e->queue.empty() && !e->free_slots.empty()) {
    Request* r = e->queue.front();
    const int L = (int)r->tokens.size();
    const uint32_t lim = request_limit(e, r);
    if (lim == 0) {  // nothing to generate
      e->queue.pop_front();
      finish_request(e, r);
      continue;
    }
    if (T + L > e->tmax) break;
    const int need_c = (L + pt - 1) / pt;
    const int need_s = e->kind == 1 ? (int)((lim + pt - 1) / pt) : 0;
    if ((int)e->free_cross.size() < need_c || (int)e->free_self.size() < need_s) break;
    e->queue.pop_front();
    r->slot = e->free_slots.back();
    e->free_slots.pop_back();
    for (int i = 0; i < need_c; ++i) {
      r->cross_pages.push_back(e->free_cross.back());
      e->free_cross.pop_back();
    }
    for (int i = 0; i < need_s; ++i) {
      r->self_pages.push_back(e->free_self.back());
      e->free_self.pop_back();
    }
    int32_t* cp = e->cross_pages_h.data() + (size_t)r->slot * e->pages_per_slot;
    for (int i = 0; i < need_c; ++i) cp[i] = r->cross_pages[i];
    int32_t* sp = e->self_pages_h.data() + (size_t)r->slot * e->pages_per_slot;
    for (int i = 0; i < need_s; ++i) sp[i] = r->self_pages[i];
    e->slot_req[r->slot] = r;
    T += L;
    max_len = std::max(max_len, L);
    admitted->push_back(r);
  }
  const int B = (int)admitted->size();
  if (B == 0) return MC_OK;
  // staging: tokens[T] pos[T] rows[T] cu[B+1] slots[B] limits[B] force[B] src[B]
  int32_t* h = e->h_i32;
  int32_t *tok = h, *pos = h + T, *rows = h + 2 * T, *cu = h + 3 * T, *slots = cu + B + 1,
          *lims = slots + B, *force = lims + B, *src = force + B, *seq_ids = src + B;
  int t = 0;
  double sum_len_sq = 0;
  cu[0] = 0;
  for (int b = 0; b < B; ++b) {
    Request* r = (*admitted)[b];
    const int L = (int)r->tokens.size();
    for (int i = 0; i < L; ++i, ++t) {
      tok[t] = r->tokens[i];
      pos[t] = i;
      rows[t] = r->cross_pages[i / pt] * pt + i % pt;
    }
    cu[b + 1] = t;
    sum_len_sq += (double)L * L;
    slots[b] = r->slot;
    lims[b] = (int32_t)request_limit(e, r);
    force[b] = (int32_t)r->force;
    src[b] = L;
  }
  // length buckets for the encoder attention (shared memory follows length)
  e->buckets.clear();
  {
    const int bounds[4] = {32, 64, 128, kMaxSeq};
    int off = 0, lo = 0;
    for (int hi : bounds) {
      const int start = off;
      for (int b = 0; b < B; ++b)
        if (src[b] > lo && src[b] <= hi) seq_ids[off++] = b;
      if (off > start) e->buckets.push_back({start, off - start, hi});
      lo = hi;
    }
  }
  cudaStream_t s = e->stream;
  CK(cudaMemcpyAsync(e->enc_seq_ids, seq_ids, B * 4, cudaMemcpyHostToDevice, s));
  CK(cudaMemcpyAsync(e->enc_tokens, tok, T * 4, cudaMemcpyHostToDevice, s));
  CK(cudaMemcpyAsync(e->enc_pos, pos, T * 4, cudaMemcpyHostToDevice, s));
  CK(cudaMemcpyAsync(e->enc_cross_rows, rows, T * 4, cudaMemcpyHostToDevice, s));
  CK(cudaMemcpyAsync(e->enc_cu, cu, (B + 1) * 4, cudaMemcpyHostToDevice, s));
  CK(cudaMemcpyAsync(e->adm_slots, slots, B * 4, cudaMemcpyHostToDevice, s));
  CK(cudaMemcpyAsync(e->adm_limits, lims, B * 4, cudaMemcpyHostToDevice, s));
  CK(cudaMemcpyAsync(e->adm_force, force, B * 4, cudaMemcpyHostToDevice, s));
  CK(cudaMemcpyAsync(e->adm_src, src, B * 4, cudaMemcpyHostToDevice, s));
  const size_t pt_bytes = (size_t)e->rmax * e->pages_per_slot * 4;
  CK(cudaMemcpyAsync(e->cross_pages_d, e->cross_pages_h.data(), pt_bytes, cudaMemcpyHostToDevice, s));
  if (e->kind == 1)
    CK(cudaMemcpyAsync(e->self_pages_d, e->self_pages_h.data(), pt_bytes, cudaMemcpyHostToDevice, s));
  mc_status st = run_encoder(e, T, B, max_len, sum_len_sq);
  if (st) return st;
  launch_init_slots(B, e->adm_slots, e->adm_limits, e->adm_force, e->adm_src, e->slot_prev,
                    e->slot_step, e->slot_limit, e->slot_force, e->slot_src, e->ssru_state,
                    e->dec_layers, e->rmax, e->d, s);
  ++e->launches;
  // the page-table copies read pageable host memory: finish before edits
  CK(cudaStreamSynchronize(s));
  prof_harvest(e);
  for (Request* r : *admitted) e->active.push_back(r->slot);
  return MC_OK;
}

// Row orders for the decode attention launches: rows with the most keys
// first (counting sort; self keys = step + 1, cross keys = source length).
void build_row_orders(mc_engine* e, int32_t* order_self, int32_t* order_cross) {
  const int R = (int)e->active.size();
  int count_s[kMaxSeq + 2] = {0}, count_c[kMaxSeq + 2] = {0};
  std::vector<int> ks(R), kc(R);
  for (int r = 0; r < R; ++r) {
    const Request* q = e->slot_req[e->active[r]];
    ks[r] = std::min<int>(kMaxSeq + 1, (int)q->output.size() + 1);
    kc[r] = std::min<int>(kMaxSeq + 1, (int)q->tokens.size());
    ++count_s[kMaxSeq + 1 - ks[r]];
    ++count_c[kMaxSeq + 1 - kc[r]];
  }
  for (int i = 1; i < kMaxSeq + 2; ++i) {
    count_s[i] += count_s[i - 1];
    count_c[i] += count_c[i - 1];
  }
  for (int r = R - 1; r >= 0; --r) {
    order_self[--count_s[kMaxSeq + 1 - ks[r]]] = r;
    order_cross[--count_c[kMaxSeq + 1 - kc[r]]] = r;
  }
}

mc_status decode_once(mc_engine* e) {
  const int R = (int)e->active.size();
  if (R == 0) return MC_OK;
  cudaStream_t s = e->stream;
  std::memcpy(e->h_i32, e->active.data(), R * 4);
  build_row_orders(e, e->h_i32 + R, e->h_i32 + 2 * R);
  CK(cudaMemcpyAsync(e->row_slot, e->h_i32, R * 4, cudaMemcpyHostToDevice, s));
  CK(cudaMemcpyAsync(e->order_self, e->h_i32 + R, R * 4, cudaMemcpyHostToDevice, s));
  CK(cudaMemcpyAsync(e->order_cross, e->h_i32 + 2 * R, R * 4, cudaMemcpyHostToDevice, s));
  mc_status st = run_decode_step(e, R);
  if (st) return st;
  CK(cudaMemcpyAsync(e->h_step_tokens, e->step_tokens, R * 4, cudaMemcpyDeviceToHost, s));
  CK(cudaMemcpyAsync(e->h_done, e->done, R, cudaMemcpyDeviceToHost, s));
  CK(cudaMemcpyAsync(e->h_status, e->d_status, 4, cudaMemcpyDeviceToHost, s));
  CK(cudaStreamSynchronize(s));
  prof_harvest(e);
  ++e->steps;
  if ((st = check_status(e))) return st;
  std::vector<int32_t> keep;
  keep.reserve(R);
  for (int r = 0; r < R; ++r) {
    const int slot = e->active[r];
    Request* q = e->slot_req[slot];
    q->output.push_back(e->h_step_tokens[r]);
    if (e->h_done[r]) finish_request(e, q);
    else keep.push_back(slot);
  }
  e->active.swap(keep);
  return MC_OK;
}

mc_status engine_step(mc_engine* e) {
  if (!e->loaded) return fail(e, MC_MODEL, "no model loaded");
  if (!e->ready) return fail(e, MC_INFERENCE, "engine is not ready after a device failure");
  mc_status st = set_device(e);
  if (st) return st;
  std::vector<Request*> admitted;
  if ((st = admit(e, &admitted))) return st;
  if (!admitted.empty()) {
    CK(cudaMemcpyAsync(e->h_status, e->d_status, 4, cudaMemcpyDeviceToHost, e->stream));
    CK(cudaStreamSynchronize(e->stream));
    if ((st = check_status(e))) return st;
  }
  return decode_once(e);
}

mc_status validate_source(const mc_engine* e, const int32_t* tokens, size_t n, std::string* why) {
  if (n == 0) {
    *why = "each input must contain at least one token";
    return MC_INVALID_INPUT;
  }
  if (n > (size_t)kMaxSeq) {
    *why = "source has " + std::to_string(n) + " tokens; maximum is 256";
    return MC_INVALID_INPUT;
  }
  for (size_t i = 0; i < n; ++i)
    if (tokens[i] < 0 || tokens[i] >= e->vsrc) {
      *why = "source token " + std::to_string(tokens[i]) + " is outside vocabulary " +
             std::to_string(e->vsrc);
      return MC_INVALID_INPUT;
    }
  return MC_OK;
}

}  // namespace

// ---- C ABI ------------------------------------------------------------------------

extern "C" void mc_config_default(mc_config* cfg) {
  if (!cfg) return;
  cfg->device = 0;
  cfg->max_inflight = 1024;
  cfg->max_encode_tokens = 65536;
  cfg->page_tokens = 16;
  cfg->kv_pages = 0;
  cfg->max_length_factor = 3;
}

extern "C" mc_status mc_create(const mc_config* cfg, mc_engine** out) {
  if (!cfg || !out) return MC_INVALID_INPUT;
  *out = nullptr;
  if (cfg->max_inflight == 0 || cfg->max_inflight > 65536 || cfg->max_encode_tokens < 256 ||
      cfg->page_tokens == 0 || cfg->page_tokens > 256 || cfg->max_length_factor < 1 ||
      cfg->max_length_factor > 8)
    return MC_INVALID_INPUT;
  mc_engine* e = new mc_engine();
  e->cfg = *cfg;
  mc_status st = set_device(e);
  if (st == MC_OK) {
    cudaError_t r = cudaStreamCreateWithFlags(&e->stream, cudaStreamNonBlocking);
    if (r == cudaSuccess) r = cudaMalloc(&e->d_status, sizeof(uint32_t));
    if (r == cudaSuccess) r = cudaMemset(e->d_status, 0, sizeof(uint32_t));
    if (r == cudaSuccess) r = cudaHostAlloc(&e->h_status, sizeof(uint32_t), cudaHostAllocDefault);
    if (r != cudaSuccess) st = MC_CUDA;
    else *e->h_status = 0;
  }
  if (st != MC_OK) {
    delete e;
    return st;
  }
  *out = e;
  return MC_OK;
}

extern "C" mc_status mc_load_marian_bin(mc_engine* e, const uint8_t* bytes, size_t len) {
  if (!e || !bytes) return MC_INVALID_INPUT;
  if (e->loaded) return fail(e, MC_MODEL, "a model is already loaded");
  mc_status st = set_device(e);
  if (st) return st;
  HostModel& m = e->host;
  std::string err = parse_marian_v1(bytes, len, &m);
  if (err.empty()) err = validate_schema(&m);
  if (!err.empty()) {
    m = HostModel();
    return fail(e, MC_MODEL, err);
  }
  e->d = m.dim;
  e->heads = m.heads;
  e->ffn = m.ffn;
  e->enc_layers = m.enc_layers;
  e->dec_layers = m.dec_layers;
  e->kind = m.decoder_kind;
  e->vsrc = m.vocab_src;
  e->vtgt = m.vocab_tgt;
  e->emb_scale = sqrtf((float)e->d);  // q8_engine.rs:22 (19.595919 = sqrtf(384))
  e->tmax = (int)e->cfg.max_encode_tokens;
  e->rmax = (int)e->cfg.max_inflight;
  const int d = e->d;
  // embeddings and tied output projection
  {
    const HostTensor& te = m.tensors.at("encoder_Wemb");
    CK(dalloc(e, &e->enc_emb, te.i8.size()));
    CK(h2d(e, e->enc_emb, te.i8.data(), te.i8.size()));
    e->enc_emb_mult = te.quant_mult;
    const HostTensor& td = m.tensors.at("decoder_Wemb");
    CK(dalloc(e, &e->dec_emb, td.i8.size()));
    CK(h2d(e, e->dec_emb, td.i8.data(), td.i8.size()));
    e->dec_emb_mult = td.quant_mult;
    e->weight_bytes += te.i8.size() + td.i8.size();
    DevLinear& v = e->vocab;
    v.w = e->dec_emb;
    v.in = d;
    v.out = e->vtgt;
    if (!(err = activation_scale(m, "decoder_Wemb", &v.alpha)).empty()) return fail(e, MC_MODEL, err);
    v.scale = 1.0f / (v.alpha * e->dec_emb_mult);  // q8_engine.rs:772
    std::vector<float> cs(e->vtgt, v.scale);
    CK(dalloc(e, &v.col_scale, cs.size()));
    CK(h2d(e, v.col_scale, cs.data(), cs.size() * 4));
    if ((st = upload_f32(e, "decoder_ff_logit_out_b", &v.bias))) return st;
    for (int i = 0; i < 3; ++i)
      if (!encode_tmap_i8(&v.tmap_b[i], v.w, v.out, v.in, kBNs[i]))
        return fail(e, MC_MODEL, "vocabulary tensor map rejected");
    // full-vocabulary candidates: every id but 1 and 7..38 (shortlist.rs:150-198)
    std::vector<uint32_t> bits((e->vtgt + 31) / 32, 0xFFFFFFFFu);
    if (e->vtgt % 32) bits.back() = (1u << (e->vtgt % 32)) - 1u;
    auto clear = [&](int id) { bits[id >> 5] &= ~(1u << (id & 31)); };
    if (e->vtgt > 1) clear(1);
    for (int id = 7; id < std::min(e->vtgt, 39); ++id) clear(id);
    CK(dalloc(e, &e->cand_bits, bits.size()));
    CK(h2d(e, e->cand_bits, bits.data(), bits.size() * 4));
  }
  std::vector<float> pos = sinusoidal_positions(d);
  CK(dalloc(e, &e->positions, pos.size()));
  CK(h2d(e, e->positions, pos.data(), pos.size() * 4));
  e->enc_attn.resize(e->enc_layers);
  e->enc_ffn.resize(e->enc_layers);
  for (int l = 0; l < e->enc_layers; ++l) {
    const std::string p = "encoder_l" + std::to_string(l + 1);
    if ((st = upload_attention(e, p + "_self", &e->enc_attn[l]))) return st;
    if ((st = upload_ffn(e, p + "_ffn", &e->enc_ffn[l]))) return st;
  }
  e->dec_ctx.resize(e->dec_layers);
  e->dec_ffn.resize(e->dec_layers);
  if (e->kind == 1) e->dec_self.resize(e->dec_layers);
  else e->dec_ssru.resize(e->dec_layers);
  for (int l = 0; l < e->dec_layers; ++l) {
    const std::string p = "decoder_l" + std::to_string(l + 1);
    if (e->kind == 1) {
      if ((st = upload_attention(e, p + "_self", &e->dec_self[l]))) return st;
    } else {
      DevSsru& s = e->dec_ssru[l];
      if ((st = upload_linear(e, p + "_rnn_W", nullptr, &s.w))) return st;
      if ((st = upload_linear(e, p + "_rnn_Wf", (p + "_rnn_bf").c_str(), &s.wf))) return st;
      if ((st = upload_f32(e, p + "_rnn_ffn_ln_scale", &s.ln_g))) return st;
      if ((st = upload_f32(e, p + "_rnn_ffn_ln_bias", &s.ln_b))) return st;
    }
    if ((st = upload_attention(e, p + "_context", &e->dec_ctx[l]))) return st;
    if ((st = upload_ffn(e, p + "_ffn", &e->dec_ffn[l]))) return st;
  }
  for (auto& kv : m.tensors) {  // payloads now live on the device
    std::vector<int8_t>().swap(kv.second.i8);
    std::vector<float>().swap(kv.second.f32);
  }
  if ((st = allocate_buffers(e))) return st;
  e->loaded = true;
  return MC_OK;
}

extern "C" mc_status mc_model_info_get(const mc_engine* e, mc_model_info* info) {
  if (!e || !info || !e->loaded) return MC_INVALID_INPUT;
  info->dim = e->d;
  info->heads = e->heads;
  info->ffn_dim = e->ffn;
  info->encoder_layers = e->enc_layers;
  info->decoder_layers = e->dec_layers;
  info->decoder_kind = e->kind;
  info->source_vocab = e->vsrc;
  info->target_vocab = e->vtgt;
  info->weight_bytes = e->weight_bytes;
  return MC_OK;
}

extern "C" void mc_destroy(mc_engine* e) {
  if (!e) return;
  cudaSetDevice(e->cfg.device);
  delete e;
}

extern "C" size_t mc_last_error(const mc_engine* e, char* buf, size_t cap) {
  if (!e) return 0;
  if (buf && cap) {
    const size_t n = std::min(cap - 1, e->error.size());
    std::memcpy(buf, e->error.data(), n);
    buf[n] = 0;
  }
  return e->error.size();
}

extern "C" int32_t mc_is_ready(const mc_engine* e) { return e && e->ready ? 1 : 0; }

extern "C" void* mc_stream(const mc_engine* e) { return e ? (void*)e->stream : nullptr; }

extern "C" mc_status mc_submit(mc_engine* e, uint64_t id, const int32_t* tokens, uint32_t n,
                               uint32_t max_out, uint32_t force_len) {
  if (!e) return MC_INVALID_INPUT;
  if (!e->loaded) return fail(e, MC_MODEL, "no model loaded");
  if (!e->ready) return fail(e, MC_INFERENCE, "engine is not ready after a device failure");
  std::string why;
  if (!tokens && n) return fail(e, MC_INVALID_INPUT, "null tokens");
  mc_status st = validate_source(e, tokens, n, &why);
  if (st) return fail(e, st, why);
  Request* r = new Request();
  r->id = id;
  r->tokens.assign(tokens, tokens + n);
  r->max_out = max_out;
  r->force = force_len;
  e->queue.push_back(r);
  return MC_OK;
}

extern "C" mc_status mc_step(mc_engine* e, uint32_t* active_after, uint32_t* queued_after) {
  if (!e) return MC_INVALID_INPUT;
  mc_status st = engine_step(e);
  if (active_after) *active_after = (uint32_t)e->active.size();
  if (queued_after) *queued_after = (uint32_t)e->queue.size();
  return st;
}

extern "C" mc_status mc_poll(mc_engine* e, uint64_t* ids, uint32_t* lengths, uint32_t max_results,
                             int32_t* tokens, size_t token_capacity, uint32_t* n_results) {
  if (!e || !n_results) return MC_INVALID_INPUT;
  uint32_t n = 0;
  size_t used = 0;
  size_t i = 0;
  for (; i < e->finished.size() && n < max_results; ++i) {
    const Finished& f = e->finished[i];
    if (used + f.tokens.size() > token_capacity) break;
    ids[n] = f.id;
    lengths[n] = (uint32_t)f.tokens.size();
    if (!f.tokens.empty()) std::memcpy(tokens + used, f.tokens.data(), f.tokens.size() * 4);
    used += f.tokens.size();
    ++n;
  }
  e->finished.erase(e->finished.begin(), e->finished.begin() + i);
  *n_results = n;
  return MC_OK;
}

namespace {

mc_status validate_batch(mc_engine* e, const int32_t* tokens, size_t n_tokens,
                         const uint32_t* offsets, uint32_t batch) {
  if (!e->loaded) return fail(e, MC_MODEL, "no model loaded");
  if (!e->ready) return fail(e, MC_INFERENCE, "engine is not ready after a device failure");
  if (!offsets || batch == 0 || offsets[0] != 0 || offsets[batch] != n_tokens || (!tokens && n_tokens))
    return fail(e, MC_INVALID_INPUT, "invalid packed batch offsets");
  for (uint32_t b = 0; b < batch; ++b) {
    if (offsets[b + 1] <= offsets[b])
      return fail(e, MC_INVALID_INPUT, "each input must contain at least one token");
    std::string why;
    mc_status st = validate_source(e, tokens + offsets[b], offsets[b + 1] - offsets[b], &why);
    if (st) return fail(e, st, why);
  }
  if (!e->queue.empty() || !e->active.empty())
    return fail(e, MC_INVALID_INPUT, "engine has streaming requests in flight");
  return MC_OK;
}

}  // namespace

extern "C" mc_status mc_translate_token_ids(mc_engine* e, const int32_t* tokens, size_t n_tokens,
                                            const uint32_t* offsets, uint32_t batch,
                                            const uint32_t* max_out, const uint32_t* force_len,
                                            int32_t* out_tokens, size_t out_capacity,
                                            uint32_t* out_offsets) {
  if (!e) return MC_INVALID_INPUT;
  mc_status st = validate_batch(e, tokens, n_tokens, offsets, batch);
  if (st) return st;
  if (!max_out || !out_offsets || (!out_tokens && out_capacity))
    return fail(e, MC_INVALID_INPUT, "null output or limit buffers");
  for (uint32_t b = 0; b < batch; ++b) {
    Request* r = new Request();
    r->id = b;
    r->tokens.assign(tokens + offsets[b], tokens + offsets[b + 1]);
    r->max_out = max_out[b];
    r->force = force_len ? force_len[b] : 0;
    e->queue.push_back(r);
  }
  const uint64_t step_bound = (uint64_t)batch * (kMaxSeq + 2) + 16;
  for (uint64_t i = 0; i < step_bound && (!e->queue.empty() || !e->active.empty()); ++i) {
    if ((st = engine_step(e))) {
      abort_all(e);
      e->finished.clear();
      return st;
    }
  }
  if (!e->queue.empty() || !e->active.empty()) {
    abort_all(e);
    e->finished.clear();
    return fail(e, MC_INFERENCE, "scheduler made no progress");
  }
  std::vector<const std::vector<int32_t>*> by_row(batch, nullptr);
  for (const Finished& f : e->finished)
    if (f.id < batch) by_row[f.id] = &f.tokens;
  size_t used = 0;
  out_offsets[0] = 0;
  for (uint32_t b = 0; b < batch; ++b) {
    const size_t n = by_row[b] ? by_row[b]->size() : 0;
    if (used + n > out_capacity) {
      e->finished.clear();
      return fail(e, MC_INVALID_INPUT, "output capacity is too small");
    }
    if (n) std::memcpy(out_tokens + used, by_row[b]->data(), n * 4);
    used += n;
    out_offsets[b + 1] = (uint32_t)used;
  }
  e->finished.clear();
  return MC_OK;
}

extern "C" mc_status mc_trace_first_step(mc_engine* e, const int32_t* tokens, size_t n_tokens,
                                         const uint32_t* offsets, uint32_t batch,
                                         float* encoder_output, float* cross_key,
                                         float* cross_value, float* decoder_state) {
  if (!e) return MC_INVALID_INPUT;
  mc_status st = validate_batch(e, tokens, n_tokens, offsets, batch);
  if (st) return st;
  if (batch > (uint32_t)e->rmax || n_tokens > (size_t)e->tmax)
    return fail(e, MC_INVALID_INPUT, "trace batch exceeds one encoder pass");
  if ((st = set_device(e))) return st;
  uint32_t lmax = 0;
  for (uint32_t b = 0; b < batch; ++b) lmax = std::max(lmax, offsets[b + 1] - offsets[b]);
  for (uint32_t b = 0; b < batch; ++b) {
    Request* r = new Request();
    r->id = b;
    r->tokens.assign(tokens + offsets[b], tokens + offsets[b + 1]);
    r->max_out = kMaxSeq;
    r->force = 0;
    e->queue.push_back(r);
  }
  std::vector<Request*> admitted;
  if ((st = admit(e, &admitted))) {
    abort_all(e);
    return st;
  }
  if (admitted.size() != batch) {
    abort_all(e);
    return fail(e, MC_INVALID_INPUT, "trace batch does not fit the free slots or pages");
  }
  const int d = e->d;
  const size_t row_bytes = (size_t)d * 4;
  if (encoder_output) {
    for (uint32_t b = 0; b < batch; ++b)
      for (uint32_t i = 0; i < offsets[b + 1] - offsets[b]; ++i)
        CK(cudaMemcpy(encoder_output + ((size_t)b * lmax + i) * d, e->enc_x + (size_t)(offsets[b] + i) * d,
                      row_bytes, cudaMemcpyDeviceToHost));
  }
  for (int l = 0; l < e->dec_layers && (cross_key || cross_value); ++l)
    for (uint32_t b = 0; b < batch; ++b) {
      const Request* r = admitted[b];
      for (uint32_t i = 0; i < offsets[b + 1] - offsets[b]; ++i) {
        const size_t row = (size_t)r->cross_pages[i / e->page_tokens] * e->page_tokens + i % e->page_tokens;
        const size_t dst = (((size_t)l * batch + b) * lmax + i) * d;
        if (cross_key)
          CK(cudaMemcpy(cross_key + dst, e->cross_k[l] + row * d, row_bytes, cudaMemcpyDeviceToHost));
        if (cross_value)
          CK(cudaMemcpy(cross_value + dst, e->cross_v[l] + row * d, row_bytes, cudaMemcpyDeviceToHost));
      }
    }
  const int R = (int)e->active.size();
  std::memcpy(e->h_i32, e->active.data(), R * 4);
  build_row_orders(e, e->h_i32 + R, e->h_i32 + 2 * R);
  CK(cudaMemcpyAsync(e->row_slot, e->h_i32, R * 4, cudaMemcpyHostToDevice, e->stream));
  CK(cudaMemcpyAsync(e->order_self, e->h_i32 + R, R * 4, cudaMemcpyHostToDevice, e->stream));
  CK(cudaMemcpyAsync(e->order_cross, e->h_i32 + 2 * R, R * 4, cudaMemcpyHostToDevice, e->stream));
  if ((st = run_decode_step(e, (int)e->active.size()))) {
    abort_all(e);
    return st;
  }
  CK(cudaMemcpyAsync(e->h_status, e->d_status, 4, cudaMemcpyDeviceToHost, e->stream));
  CK(cudaStreamSynchronize(e->stream));
  prof_harvest(e);
  if ((st = check_status(e))) return st;
  if (decoder_state)
    CK(cudaMemcpy(decoder_state, e->last_state, (size_t)batch * row_bytes, cudaMemcpyDeviceToHost));
  abort_all(e);
  return MC_OK;
}

extern "C" mc_status mc_profile(mc_engine* e, int32_t enable) {
  if (!e) return MC_INVALID_INPUT;
  if (e->stream) cudaStreamSynchronize(e->stream);
  prof_harvest(e);
  e->profiling = enable != 0;
  for (int k = 0; k < MC_KERNEL_KINDS; ++k) {
    e->prof_ms[k] = e->prof_flops[k] = e->prof_bytes[k] = 0.0;
    e->prof_n[k] = 0;
  }
  return MC_OK;
}

extern "C" mc_status mc_profile_read(const mc_engine* e, int32_t kind, uint64_t* launches,
                                     double* ms, double* flops, double* bytes) {
  if (!e || kind < 0 || kind >= MC_KERNEL_KINDS) return MC_INVALID_INPUT;
  if (launches) *launches = e->prof_n[kind];
  if (ms) *ms = e->prof_ms[kind];
  if (flops) *flops = e->prof_flops[kind];
  if (bytes) *bytes = e->prof_bytes[kind];
  return MC_OK;
}

extern "C" uint64_t mc_launch_count(const mc_engine* e) { return e ? e->launches : 0; }
