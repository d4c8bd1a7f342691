// engine.cu -- the marian_cuda engine: model upload, packed varlen encoder,
// paged cross/self caches, and a continuous-batching greedy decoder.
//
// Control flow restated from Q8CpuEngine::translate_token_ids
// (crates/marian-cpu/src/q8_engine.rs:353-466) with four B200 changes:
//   * sources are packed without padding (cu_seqlens) instead of [B, Lmax];
//   * cross keys/values and (for the self-attention decoder) self
//     keys/values live in pools of fixed-size pages addressed through
//     per-slot page tables;
//   * decode rows are the active slots only: finished rows retire at once and
//     queued requests are admitted into free slots between steps
//     (the reference keeps computing finished rows, q8_engine.rs:438-441);
//   * the active rows are split over lanes: each lane has its own CUDA
//     stream, activation buffers and decode step (replayed from a CUDA graph
//     captured once per lane), and the host completes one lane's step and
//     relaunches it while the other lanes' steps run, so the latency-bound
//     kernels of several steps overlap on the GPU.  Weights, slots, page
//     pools and page tables are shared; lanes use disjoint slots and pages.
#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <deque>
#include <string>
#include <unordered_map>
#include <vector>

#include "common.cuh"
#include "kernels.cuh"
#include "linear_ln.cuh"
#include "marian_cuda.h"
#include "model_loader.h"
#include "q8_gemm.cuh"

namespace {

using namespace mc;

constexpr int kBNs[3] = {64, 128, 256};
constexpr int kMaxLanes = 8;

int bn_index(int bn) { return bn == 64 ? 0 : (bn == 128 ? 1 : 2); }

struct DevLinear {
  int8_t* w = nullptr;
  float* col_scale = nullptr;  // [out] = 1 / (alpha * weight_mult)
  float* bias = nullptr;       // [out] or null
  int in = 0, out = 0;
  float alpha = 1.0f;          // this linear's own activation alpha
  float scale = 1.0f;          // 1 / (alpha * weight quant_mult)
  bool per_row = false;        // col_scale holds 1 / (alpha * row multiplier[n])
  CUtensorMap tmap_b[3];       // W tensor maps for BN = 64, 128, 256
  CUtensorMap tmap_ln;         // W tensor map for the fused LayerNorm kernel
  bool has_ln_map = false;     // (box out / linear_ln_cluster(out) rows)
  CUtensorMap tmap_proj;       // W as the fused kernel's second linear
  bool has_proj_map = false;   // (box out / linear_ln_cluster(in) rows)
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

// Per-kernel-class timing (mc_profile): CUDA event pairs on a lane's stream
// around each launch, harvested after the lane's step is complete.
struct ProfRec {
  int kind;
  double flops, bytes;
  cudaEvent_t a, b;
};

// One decode step enqueued on a lane and not yet applied on the host.
struct StepInFlight {
  std::vector<int32_t> joins;  // admitted slots the step's row table appends
  int parity = 0;              // which result buffers (and graph) the step uses
  int rows_bound = 0;          // its rows: exact once the step before it is applied
  cudaEvent_t tl_start = nullptr, tl_end = nullptr;  // mc_timeline
};

// One lane: a stream, the activation buffers of an encoder pass and of a
// decode step, and the rows (slots) whose steps run on it.
//
// The row table a step runs over lives on the device: the step's first
// kernel (launch_step_rows) drops the rows the previous step finished and
// appends the slots admitted since, so a lane keeps up to kStepDepth steps
// enqueued and the host applies a step's tokens while the next one runs.
// The host mirrors the table: `active` is the previous applied step's rows
// minus the ones it finished; an enqueued step's rows are `active` (as it
// will be when the steps before it are applied) followed by its joins.
constexpr int kStepDepth = 2;

struct Lane {
  int id = 0;
  int cap = 0;                       // scheduling limit on active rows
  cudaStream_t stream = nullptr;     // decode steps
  bool own_stream = false;
  cudaStream_t enc_stream = nullptr; // encoder passes of admissions
  cudaEvent_t enc_done = nullptr;    // the last admission's encoder pass is complete
  // encoder attention buckets side by side (see launch_encoder_buckets)
  cudaEvent_t enc_fork = nullptr, enc_join = nullptr;
  bool enc_alone = false;  // the pass being enqueued has no decode step beside it
  cudaStream_t cur = nullptr;        // stream the launch helpers use
  uint32_t* d_status = nullptr;      // error bits of this lane's kernels

  // encoder pass (capacity tmax packed tokens)
  float *enc_x = nullptr, *enc_x1 = nullptr, *enc_qkv = nullptr, *enc_proj = nullptr;
  QBuf enc_q[kMaxQuantOut];
  QBuf enc_o, enc_h;
  // admission block, pinned on the host and mirrored on the device:
  // tokens[T] pos[T] cross_rows[T] cu[B+1] slots[B] limits[B] force[B]
  // src[B] seq_ids[B] page_rows[2][B][pages_per_slot]
  int32_t* adm_h = nullptr;
  int32_t* adm_d = nullptr;
  size_t adm_cap = 0;  // int32 entries
  struct Bucket {
    int offset, count, max_len;
  };
  std::vector<Bucket> buckets;

  // decode step (capacity rmax rows)
  float *dec_a = nullptr, *dec_b = nullptr, *dec_qkv = nullptr, *dec_proj = nullptr;
  QBuf dec_q[kMaxQuantOut];
  QBuf dec_o, dec_h;
  // device row table [4 + 3 * rmax]: row count, 3 unused, then row slots,
  // self-attention row order and cross-attention row order (most keys
  // first), rmax each -- written by each step's launch_step_rows
  int32_t* rows_d = nullptr;
  int32_t* rows_scratch = nullptr;   // [rmax]
  int32_t* join_d = nullptr;         // [1 + rmax]: count, then the appended slots
  int32_t *self_row_map = nullptr, *step_tokens = nullptr;
  uint8_t *eos_mask = nullptr, *done = nullptr;
  unsigned long long* best = nullptr;
  // per parity (two steps in flight): pinned join block and read-backs
  int32_t* join_h[kStepDepth] = {};
  int32_t* h_step_tokens[kStepDepth] = {};
  uint8_t* h_done[kStepDepth] = {};
  uint32_t* h_status[kStepDepth] = {};
  cudaEvent_t step_done[kStepDepth] = {};  // recorded after the step's read-backs

  std::vector<int32_t> active;   // rows surviving the last applied step, in table order
  std::vector<int32_t> ready;    // admitted slots whose encoder pass is done; next step appends them
  std::vector<int32_t> pending;  // admitted slots whose encoder pass is in flight
  std::deque<StepInFlight> inflight;
  int next_parity = 0;
  bool enc_in_flight = false;
  float* last_state = nullptr;  // final decoder state of the last step
  int eager_steps = 0;
  cudaGraphExec_t graph[kStepDepth] = {};  // decode step for up to `cap` rows, per parity
  bool graph_tried[kStepDepth] = {};
  uint64_t graph_kernels = 0;
  std::vector<ProfRec> prof_pending;
  cudaEvent_t tl_prev_end = nullptr;  // mc_timeline: end of the last applied step

  int32_t* row_slot() const { return rows_d + 4; }
};

}  // namespace

struct mc_engine {
  mc_config cfg{};
  std::string error;
  bool ready = true;
  bool loaded = false;
  cudaStream_t stream = nullptr;  // load stream; lane 0 runs on it
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
  DevLinear vocab;  // tied output projection over decoder_Wemb; its bias is
                    // candidate-masked (-inf at excluded ids) and padded
  float* positions = nullptr;
  std::vector<DevAttention> enc_attn, dec_self, dec_ctx;
  std::vector<DevFfn> enc_ffn, dec_ffn;
  std::vector<DevSsru> dec_ssru;

  int tmax = 0;  // packed tokens per encoder pass
  int rmax = 0;  // slots

  // lexical shortlist (mc_load_shortlist): device copy of the offsets and
  // targets, per-slot candidate bitmasks, and per source token whether it
  // maps to EOS (the reference requires EOS among a sentence's candidates)
  bool has_shortlist = false;
  int sl_first_num = 0, sl_words = 0;
  int32_t *sl_offsets = nullptr, *sl_targets = nullptr;
  uint32_t* sl_masks = nullptr;
  std::vector<uint8_t> sl_maps_eos;

  // slots and caches (shared by the lanes)
  int32_t *slot_prev = nullptr, *slot_step = nullptr, *slot_limit = nullptr, *slot_force = nullptr,
          *slot_src = nullptr;
  float* ssru_state = nullptr;
  int pages_per_slot = 0, page_tokens = 16;
  int cross_pool_pages = 0, self_pool_pages = 0;
  int32_t *cross_pages_d = nullptr, *self_pages_d = nullptr;
  std::vector<float*> cross_k, cross_v, self_k, self_v;
  // tensor maps of the pools for the decode attention (encode_tmap_kv)
  std::vector<KvBoxMaps> cross_k_map, cross_v_map, self_k_map, self_v_map;
  std::vector<int32_t> free_cross, free_self, free_slots;

  std::vector<Lane> lanes;
  bool use_graphs = true;
  // decode sub-layers end in one fused linear + residual + LayerNorm launch
  // (linear_ln.cu) when the width allows; MARIAN_CUDA_FUSED_LN=0 selects the
  // separate GEMM and LayerNorm kernels (same results)
  bool fuse_ln = true;

  // scheduler
  std::deque<Request*> queue;
  std::vector<Request*> slot_req;  // [rmax]
  std::vector<Finished> finished;
  uint64_t steps = 0, launches = 0;

  bool profiling = false;
  std::vector<cudaEvent_t> event_pool;
  bool timeline = false;
  uint64_t tl_steps = 0;
  double tl_busy_ms = 0.0, tl_gap_ms = 0.0;
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

// A timing event from the engine's pool.
cudaEvent_t pooled_event(mc_engine* e) {
  cudaEvent_t x = nullptr;
  if (!e->event_pool.empty()) {
    x = e->event_pool.back();
    e->event_pool.pop_back();
  } else {
    cudaEventCreate(&x);
  }
  return x;
}

int prof_begin(mc_engine* e, Lane& L, int kind, double flops, double bytes) {
  if (!e->profiling) return -1;
  ProfRec r{kind, flops, bytes, pooled_event(e), pooled_event(e)};
  cudaEventRecord(r.a, L.cur);
  L.prof_pending.push_back(r);
  return (int)L.prof_pending.size() - 1;
}

void prof_end(Lane& L, int idx) {
  if (idx >= 0) cudaEventRecord(L.prof_pending[idx].b, L.cur);
}

// Call after the lane's stream is synchronized.
void prof_harvest(mc_engine* e, Lane& L) {
  for (auto& r : L.prof_pending) {
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
  L.prof_pending.clear();
}

// Timeline of lane L's decode stream (call once step F is complete): the
// step's duration between the events recorded before and after its work,
// and the stream's idle time since the previous step ended.
void timeline_harvest(mc_engine* e, Lane& L, StepInFlight& F) {
  if (!F.tl_start) return;
  float busy = 0.0f, gap = 0.0f;
  if (cudaEventElapsedTime(&busy, F.tl_start, F.tl_end) == cudaSuccess) {
    e->tl_busy_ms += busy;
    ++e->tl_steps;
  }
  if (L.tl_prev_end && cudaEventElapsedTime(&gap, L.tl_prev_end, F.tl_start) == cudaSuccess)
    e->tl_gap_ms += gap;
  if (L.tl_prev_end) e->event_pool.push_back(L.tl_prev_end);
  e->event_pool.push_back(F.tl_start);
  L.tl_prev_end = F.tl_end;
  F.tl_start = F.tl_end = nullptr;
}

void timeline_drop(mc_engine* e, Lane& L) {
  for (StepInFlight& F : L.inflight)
    for (cudaEvent_t* ev : {&F.tl_start, &F.tl_end})
      if (*ev) {
        e->event_pool.push_back(*ev);
        *ev = nullptr;
      }
  if (L.tl_prev_end) e->event_pool.push_back(L.tl_prev_end);
  L.tl_prev_end = nullptr;
}

#define PROFILED(kind, flops, bytes, stmt)                        \
  do {                                                            \
    const int pi_ = prof_begin(e, L, (kind), (flops), (bytes));   \
    stmt;                                                         \
    prof_end(L, pi_);                                             \
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

// Host-to-device copy on the load stream (ordered after dalloc's memset),
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
  if (!std::isfinite(inv) || inv <= 0.0f)
    return fail(e, MC_MODEL, wname + ": 1 / (activation scale * quantization multiplier) is not finite");
  L->scale = inv;
  std::vector<float> cs(L->out, inv);
  // per-output-row multipliers (the loader's _QuantMultRows extension):
  // column n of the GEMM output dequantizes with 1 / (alpha * mult[n])
  const std::vector<float> rows = weight_row_mults(e->host, wname);
  if (!rows.empty()) {
    if ((int)rows.size() != L->out) return fail(e, MC_MODEL, wname + ": row multiplier count mismatch");
    for (int n = 0; n < L->out; ++n) {
      cs[n] = 1.0f / (L->alpha * rows[n]);
      if (!std::isfinite(cs[n]) || cs[n] <= 0.0f)
        return fail(e, MC_MODEL, wname + ": 1 / (activation scale * row multiplier) is not finite");
    }
    L->per_row = true;
  }
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
  if (const int c = linear_ln_cluster(L->out)) {
    if (!encode_tmap_i8(&L->tmap_ln, L->w, L->out, L->in, L->out / c))
      return fail(e, MC_MODEL, wname + ": tensor map rejected");
    L->has_ln_map = true;
  }
  if (const int c = linear_ln_cluster(L->in)) {
    if (L->out % c == 0 && L->out / c <= 256 && (L->out / c) % 32 == 0) {
      if (!encode_tmap_i8(&L->tmap_proj, L->w, L->out, L->in, L->out / c))
        return fail(e, MC_MODEL, wname + ": tensor map rejected");
      L->has_proj_map = true;
    }
  }
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

// One grouped GEMM launch on the lane's stream.  m is the row capacity the
// grid is sized for; m_dev (nullable) is the device row count the kernel
// reads.  flops/bytes for the profile use m_prof rows.
mc_status gemm(mc_engine* e, Lane& L, int kind, int m, const int32_t* m_dev, double m_prof,
               const GroupSpec* specs, int n_groups, unsigned long long* argmax = nullptr,
               const uint8_t* eos = nullptr) {
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
    // per-tensor weight scale (q8_gemm.rs:438), or the per-row extension's
    g.col_scale = s.w->per_row ? s.w->col_scale : nullptr;
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
    g.eos_mask = eos;
    if (s.mode == kEpiArgmax && e->has_shortlist) {
      g.cand_rows = e->sl_masks;
      g.cand_slot = L.row_slot();
      g.cand_words = e->sl_words;
    }
  }
  p.m = m;
  p.m_dev = m_dev;
  p.k = specs[0].w->in;
  p.num_groups = n_groups;
  p.max_n = max_n;
  p.status = L.d_status;
  double flops = 0, bytes = 0;
  for (int i = 0; i < n_groups; ++i) {
    const double n = specs[i].w->out, k = specs[i].w->in;
    flops += 2.0 * m_prof * n * k;
    const double out_bytes = specs[i].mode == kEpiArgmax ? 8.0 * m_prof
                             : specs[i].mode == kEpiQ8   ? 1.0 * m_prof * n
                                                         : 4.0 * m_prof * n;
    bytes += m_prof * k + n * k + 4.0 * n * (specs[i].w->bias ? 2 : 1) + out_bytes;
  }
  PROFILED(kind, flops, bytes, CK(launch_q8_gemm(p, bn, L.cur)));
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

// Device pointers of one admission block (see Lane::adm_h).
struct AdmLayout {
  int T = 0, B = 0;
  size_t tok = 0, pos = 0, crow = 0, cu = 0, slots = 0, lims = 0, force = 0, src = 0, seq_ids = 0,
         pages = 0, end = 0;
};

AdmLayout adm_layout(int T, int B, int pps) {
  AdmLayout a;
  a.T = T;
  a.B = B;
  a.tok = 0;
  a.pos = a.tok + T;
  a.crow = a.pos + T;
  a.cu = a.crow + T;
  a.slots = a.cu + B + 1;
  a.lims = a.slots + B;
  a.force = a.lims + B;
  a.src = a.force + B;
  a.seq_ids = a.src + B;
  a.pages = a.seq_ids + B;
  a.end = a.pages + (size_t)2 * B * pps;
  return a;
}

// ---- encoder pass over packed admitted sources ------------------------------

// The encoder attention over the pass's length buckets (disjoint sequences,
// so independent): one launch per bucket, shared memory sized to its
// longest sequence.  When no decode step runs beside the pass (and outside
// profiling) the shorter buckets run on the lane's idle decode stream,
// forked from the encoder stream after the QKV projection and joined back
// before the output projection, so the few long sequences' CTAs run beside
// the many short ones instead of after them.  Beside decode steps the
// buckets stay on the encoder stream: more encoder CTAs at once would hold
// SMs that the latency-bound decode chain waits for.
cudaError_t launch_encoder_buckets(mc_engine* e, Lane& L, const int32_t* cu, const int32_t* seq_ids, int d,
                                   float alpha) {
  const int nb = (int)L.buckets.size();
  const bool fork = !e->profiling && L.enc_alone && nb > 1 && L.cur != L.stream;
  cudaError_t err = cudaSuccess;
  if (fork && ((err = cudaEventRecord(L.enc_fork, L.cur)) != cudaSuccess ||
               (err = cudaStreamWaitEvent(L.stream, L.enc_fork, 0)) != cudaSuccess))
    return err;
  for (int i = 0; i < nb; ++i) {
    const Lane::Bucket& bk = L.buckets[i];
    cudaStream_t s = (fork && i < nb - 1) ? L.stream : L.cur;
    err = launch_attn_encoder(L.enc_qkv, cu, seq_ids + bk.offset, bk.count, bk.max_len, d, e->heads, L.enc_o.p,
                              alpha, L.d_status, s);
    if (err != cudaSuccess) return err;
  }
  if (fork && ((err = cudaEventRecord(L.enc_join, L.stream)) != cudaSuccess ||
               (err = cudaStreamWaitEvent(L.cur, L.enc_join, 0)) != cudaSuccess))
    return err;
  return cudaSuccess;
}

mc_status run_encoder(mc_engine* e, Lane& L, const AdmLayout& A, double sum_len_sq) {
  const int d = e->d;
  const int T = A.T;
  const int32_t* adm = L.adm_d;
  const double rows_d = (double)T * d;
  PROFILED(MC_K_EMBED, 0.0, rows_d * (1 + 4 + 4 + 3),
           launch_embed_encoder(adm + A.tok, adm + A.pos, T, e->enc_emb, e->enc_emb_mult,
                                e->emb_scale, e->positions, d, L.enc_x,
                                quant_out_vec(L.enc_q, enc_input_alphas(e, 0)), L.d_status,
                                L.cur));
  ++e->launches;
  mc_status st;
  for (int l = 0; l < e->enc_layers; ++l) {
    const DevAttention& a = e->enc_attn[l];
    const DevFfn& f = e->enc_ffn[l];
    GroupSpec qkv[3] = {
        {&L.enc_q[0], &a.wq, kEpiF32, L.enc_qkv, 3 * d, 0, nullptr, false, 0.f},
        {&L.enc_q[1], &a.wk, kEpiF32, L.enc_qkv, 3 * d, d, nullptr, false, 0.f},
        {&L.enc_q[2], &a.wv, kEpiF32, L.enc_qkv, 3 * d, 2 * d, nullptr, false, 0.f}};
    if ((st = gemm(e, L, MC_K_GEMM_QKV, T, nullptr, T, qkv, 3))) return st;
    PROFILED(MC_K_ATTN_ENC, 4.0 * sum_len_sq * d, rows_d * (12 + 1),
             CK(launch_encoder_buckets(e, L, adm + A.cu, adm + A.seq_ids, d, a.wo.alpha)));
    e->launches += L.buckets.size();
    GroupSpec wo = {&L.enc_o, &a.wo, kEpiF32, L.enc_proj, d, 0, nullptr, false, 0.f};
    if ((st = gemm(e, L, MC_K_GEMM_OUT, T, nullptr, T, &wo, 1))) return st;
    PROFILED(MC_K_LAYERNORM, 0.0, rows_d * 13,
             launch_residual_ln(L.enc_proj, d, L.enc_x, d, a.ln_g, a.ln_b, T, nullptr, d, L.enc_x1,
                                quant_out(L.enc_q, {f.w1.alpha}), L.d_status, L.cur));
    GroupSpec w1 = {&L.enc_q[0], &f.w1, kEpiQ8, L.enc_h.p, e->ffn, 0, nullptr, true, f.w2.alpha};
    if ((st = gemm(e, L, MC_K_GEMM_FFN1, T, nullptr, T, &w1, 1))) return st;
    GroupSpec w2 = {&L.enc_h, &f.w2, kEpiF32, L.enc_proj, d, 0, nullptr, false, 0.f};
    if ((st = gemm(e, L, MC_K_GEMM_FFN2, T, nullptr, T, &w2, 1))) return st;
    PROFILED(MC_K_LAYERNORM, 0.0, rows_d * (12 + enc_input_alphas(e, l + 1).size()),
             launch_residual_ln(L.enc_proj, d, L.enc_x1, d, f.ln_g, f.ln_b, T, nullptr, d, L.enc_x,
                                quant_out_vec(L.enc_q, enc_input_alphas(e, l + 1)), L.d_status,
                                L.cur));
    e->launches += 2;
  }
  // cross keys/values of every decoder layer into the paged pools
  // (q8_engine.rs:560-567)
  std::vector<GroupSpec> cross;
  for (int l = 0; l < e->dec_layers; ++l) {
    cross.push_back({&L.enc_q[2 * l], &e->dec_ctx[l].wk, kEpiF32, e->cross_k[l], d, 0,
                     adm + A.crow, false, 0.f});
    cross.push_back({&L.enc_q[2 * l + 1], &e->dec_ctx[l].wv, kEpiF32, e->cross_v[l], d, 0,
                     adm + A.crow, false, 0.f});
  }
  for (size_t i = 0; i < cross.size(); i += kMaxGemmGroups)
    if ((st = gemm(e, L, MC_K_GEMM_CROSSKV, T, nullptr, T, cross.data() + i,
                   (int)std::min<size_t>(kMaxGemmGroups, cross.size() - i))))
      return st;
  return MC_OK;
}

// A decode linear whose output feeds residual + LayerNorm: one fused launch
// (linear_ln.cu) when the model width allows, else the GEMM into dec_proj
// and the LayerNorm kernel.  Both give the same bits.
// proj_kind(e, w): how the fused launch can also compute linear w of its
// normalized rows: 1 for a d x d linear (the cross-attention query), 2 for
// the FFN's first linear (4d x d, ReLU, int8 output; d = 128, 256, 512),
// 0 when it cannot.
int proj_kind(const mc_engine* e, const DevLinear& w) {
  if (!e->fuse_ln || !w.has_proj_map || w.in != e->d) return 0;
  if (w.out == e->d) return 1;
  if (w.out == 4 * e->d && (e->d == 128 || e->d == 256 || e->d == 512)) return 2;
  return 0;
}

mc_status linear_ln(mc_engine* e, Lane& L, int gemm_kind, const QBuf* a, const DevLinear& w,
                    const float* residual, const float* gamma, const float* beta, int cap,
                    const int32_t* m_dev, double m_prof, float* out, const QuantOut& q,
                    const DevLinear* proj = nullptr, void* proj_out = nullptr, float proj_alpha = 0.f) {
  const int d = e->d;
  const double rows_d = m_prof * d;
  if (e->fuse_ln && w.has_ln_map && w.out == d) {
    LinearLnParams p;
    std::memset(&p, 0, sizeof(p));
    p.tmap_a = a->tmap;
    p.tmap_b = w.tmap_ln;
    p.col_scale = w.per_row ? w.col_scale : nullptr;
    p.uniform_scale = w.scale;
    p.bias = w.bias;
    p.residual = residual;
    p.ldr = d;
    p.gamma = gamma;
    p.beta = beta;
    p.out = out;
    p.q = q;
    p.cap = cap;
    p.m_dev = m_dev;
    p.k = w.in;
    p.status = L.d_status;
    double flops = 2.0 * rows_d * w.in;
    double bytes = m_prof * w.in + (double)d * w.in + 16.0 * d + rows_d * (8 + q.count);
    if (proj) {  // a second linear of the normalized rows, same launch
      p.proj = proj_kind(e, *proj);
      if (!p.proj) return fail(e, MC_CUDA, "fused second linear requested for an unsupported shape");
      p.tmap_b2 = proj->tmap_proj;
      p.col_scale2 = proj->per_row ? proj->col_scale : nullptr;
      p.uniform_scale2 = proj->scale;
      p.bias2 = proj->bias;
      p.ldo2 = proj->out;
      p.alpha2 = proj->alpha;
      if (p.proj == 1)
        p.out2 = static_cast<float*>(proj_out);
      else
        p.out2q = static_cast<int8_t*>(proj_out);
      p.alpha3 = proj_alpha;
      flops += 2.0 * m_prof * proj->out * d;
      bytes += (double)proj->out * d + 8.0 * proj->out + m_prof * proj->out * (p.proj == 1 ? 4 : 1);
    }
    PROFILED(MC_K_GEMM_LN, flops, bytes, CK(launch_q8_linear_ln(p, d, L.cur)));
    ++e->launches;
    return MC_OK;
  }
  if (proj) return fail(e, MC_CUDA, "fused projection requested without the fused kernel");
  GroupSpec spec = {a, &w, kEpiF32, L.dec_proj, d, 0, nullptr, false, 0.f};
  mc_status st = gemm(e, L, gemm_kind, cap, m_dev, m_prof, &spec, 1);
  if (st) return st;
  PROFILED(MC_K_LAYERNORM, 0.0, rows_d * (12 + q.count),
           launch_residual_ln(L.dec_proj, d, residual, d, gamma, beta, cap, m_dev, d, out, q, L.d_status,
                              L.cur));
  ++e->launches;
  return MC_OK;
}

// ---- one decode step over a lane's active rows -------------------------------
// Grids cover `cap` rows; the kernels read the step's row count from the
// lane's rows block (rows_d[0]), so the same launches serve any row count up
// to cap and can be replayed from a CUDA graph.
// `rows` (the step's slots, known exactly when profiling) only feeds the
// profile's algorithmic byte and flop counts.
mc_status run_decode_step(mc_engine* e, Lane& L, int cap, const std::vector<int32_t>& rows) {
  const int d = e->d;
  float* x = L.dec_a;   // layer input
  float* y = L.dec_b;   // next
  const int32_t* nrows = L.rows_d;
  const int32_t* row_slot = L.row_slot();
  const int32_t* order_self = row_slot + e->rmax;
  const int32_t* order_cross = order_self + e->rmax;
  // key counts for the attention roofline: self = step + 1, cross = source
  double self_keys = 0, cross_keys = 0;
  if (e->profiling) {
    for (int s : rows) {
      const Request* q = e->slot_req[s];
      if (!q) continue;
      self_keys += (double)q->output.size() + 1;
      cross_keys += (double)q->tokens.size();
    }
  }
  const double R = (double)rows.size();
  const double rows_d = R * d;
  PROFILED(MC_K_EMBED, 0.0, rows_d * (1 + 4 + 4 + 3),
           launch_embed_decoder(cap, nrows, row_slot, e->slot_prev, e->slot_step, e->slot_force,
                                e->dec_emb, e->dec_emb_mult, e->emb_scale, e->positions, d, x,
                                quant_out_vec(L.dec_q, dec_input_alphas(e, 0)), L.eos_mask,
                                e->kind == 1 ? e->self_pages_d : nullptr, e->pages_per_slot,
                                e->page_tokens, L.self_row_map, L.d_status, L.cur));
  ++e->launches;
  mc_status st;
  for (int l = 0; l < e->dec_layers; ++l) {
    const DevAttention& c = e->dec_ctx[l];
    const DevFfn& f = e->dec_ffn[l];
    bool q_done = false;  // the cross-attention query came with the first LayerNorm
    if (e->kind == 1) {
      const DevAttention& a = e->dec_self[l];
      GroupSpec qkv[3] = {
          {&L.dec_q[0], &a.wq, kEpiF32, L.dec_qkv, d, 0, nullptr, false, 0.f},
          {&L.dec_q[1], &a.wk, kEpiF32, e->self_k[l], d, 0, L.self_row_map, false, 0.f},
          {&L.dec_q[2], &a.wv, kEpiF32, e->self_v[l], d, 0, L.self_row_map, false, 0.f}};
      if ((st = gemm(e, L, MC_K_GEMM_QKV, cap, nrows, R, qkv, 3))) return st;
      PROFILED(MC_K_ATTN_SELF, 4.0 * self_keys * d, 8.0 * self_keys * d + rows_d * 5,
               CK(launch_attn_decode(L.dec_qkv, d, cap, nrows, row_slot, order_self, e->slot_step, 1,
                                     e->self_pages_d, e->pages_per_slot, e->page_tokens,
                                     &e->self_k_map[l], &e->self_v_map[l], d, e->heads, L.dec_o.p,
                                     a.wo.alpha, L.d_status, L.cur)));
      // the first LayerNorm's rows also feed the cross-attention query:
      // one launch computes both when the fused kernel applies
      if (proj_kind(e, c.wq) == 1 && a.wo.has_ln_map && a.wo.out == d) {
        QuantOut none;
        std::memset(&none, 0, sizeof(none));
        if ((st = linear_ln(e, L, MC_K_GEMM_OUT, &L.dec_o, a.wo, x, a.ln_g, a.ln_b, cap, nrows, R, y, none,
                            &c.wq, L.dec_qkv)))
          return st;
        q_done = true;
      } else if ((st = linear_ln(e, L, MC_K_GEMM_OUT, &L.dec_o, a.wo, x, a.ln_g, a.ln_b, cap, nrows, R, y,
                                 quant_out(L.dec_q, {c.wq.alpha})))) {
        return st;
      }
      ++e->launches;
    } else {
      const DevSsru& s = e->dec_ssru[l];
      GroupSpec wf[2] = {
          {&L.dec_q[0], &s.w, kEpiF32, L.dec_qkv, 2 * d, 0, nullptr, false, 0.f},
          {&L.dec_q[1], &s.wf, kEpiF32, L.dec_qkv, 2 * d, d, nullptr, false, 0.f}};
      if ((st = gemm(e, L, MC_K_GEMM_QKV, cap, nrows, R, wf, 2))) return st;
      PROFILED(MC_K_SSRU, 0.0, rows_d * 25,
               launch_ssru(L.dec_qkv, 2 * d, d, e->ssru_state + (size_t)l * e->rmax * d,
                           row_slot, x, s.ln_g, s.ln_b, cap, nrows, d, y,
                           quant_out(L.dec_q, {c.wq.alpha}), L.d_status, L.cur));
      ++e->launches;
    }
    std::swap(x, y);
    if (!q_done) {
      GroupSpec wq = {&L.dec_q[0], &c.wq, kEpiF32, L.dec_qkv, d, 0, nullptr, false, 0.f};
      if ((st = gemm(e, L, MC_K_GEMM_QKV, cap, nrows, R, &wq, 1))) return st;
    }
    PROFILED(MC_K_ATTN_CROSS, 4.0 * cross_keys * d, 8.0 * cross_keys * d + rows_d * 5,
             CK(launch_attn_decode(L.dec_qkv, d, cap, nrows, row_slot, order_cross, e->slot_src, 0,
                                   e->cross_pages_d, e->pages_per_slot, e->page_tokens,
                                   &e->cross_k_map[l], &e->cross_v_map[l], d, e->heads, L.dec_o.p,
                                   c.wo.alpha, L.d_status, L.cur)));
    // the second LayerNorm's rows also feed the FFN's first linear: one
    // launch computes both when the fused kernel applies
    const bool ffn_fused = proj_kind(e, f.w1) == 2 && c.wo.has_ln_map && c.wo.out == d;
    if (ffn_fused) {
      QuantOut none;
      std::memset(&none, 0, sizeof(none));
      if ((st = linear_ln(e, L, MC_K_GEMM_OUT, &L.dec_o, c.wo, x, c.ln_g, c.ln_b, cap, nrows, R, y, none,
                          &f.w1, L.dec_h.p, f.w2.alpha)))
        return st;
    } else if ((st = linear_ln(e, L, MC_K_GEMM_OUT, &L.dec_o, c.wo, x, c.ln_g, c.ln_b, cap, nrows, R, y,
                               quant_out(L.dec_q, {f.w1.alpha})))) {
      return st;
    }
    std::swap(x, y);
    if (!ffn_fused) {
      GroupSpec w1 = {&L.dec_q[0], &f.w1, kEpiQ8, L.dec_h.p, e->ffn, 0, nullptr, true, f.w2.alpha};
      if ((st = gemm(e, L, MC_K_GEMM_FFN1, cap, nrows, R, &w1, 1))) return st;
    }
    if ((st = linear_ln(e, L, MC_K_GEMM_FFN2, &L.dec_h, f.w2, x, f.ln_g, f.ln_b, cap, nrows, R, y,
                        quant_out_vec(L.dec_q, dec_input_alphas(e, l + 1)))))
      return st;
    std::swap(x, y);
    ++e->launches;
  }
  // tied vocabulary projection + masked argmax (q8_engine.rs:749-790)
  GroupSpec voc = {&L.dec_q[0], &e->vocab, kEpiArgmax, nullptr, 0, 0, nullptr, false, 0.f};
  if ((st = gemm(e, L, MC_K_GEMM_VOCAB, cap, nrows, R, &voc, 1, L.best, L.eos_mask))) return st;
  PROFILED(MC_K_FINALIZE, 0.0, R * 29,
           launch_finalize(cap, nrows, row_slot, L.best, e->slot_prev, e->slot_step, e->slot_limit,
                           L.step_tokens, L.done, L.d_status, L.cur));
  ++e->launches;
  L.last_state = x;
  return MC_OK;
}

}  // namespace

// ============================================================================
// engine lifecycle, scheduling and the C ABI
// ============================================================================

mc_engine::~mc_engine() {
  for (Lane& L : lanes) {
    if (L.stream) cudaStreamSynchronize(L.stream);
    if (L.enc_stream) cudaStreamSynchronize(L.enc_stream);
  }
  if (stream) cudaStreamSynchronize(stream);
  for (Lane& L : lanes) {
    for (auto& r : L.prof_pending) {
      cudaEventDestroy(r.a);
      cudaEventDestroy(r.b);
    }
    for (StepInFlight& F : L.inflight)
      for (cudaEvent_t ev : {F.tl_start, F.tl_end})
        if (ev) cudaEventDestroy(ev);
    if (L.tl_prev_end) cudaEventDestroy(L.tl_prev_end);
    for (int i = 0; i < kStepDepth; ++i) {
      if (L.graph[i]) cudaGraphExecDestroy(L.graph[i]);
      if (L.h_status[i]) cudaFreeHost(L.h_status[i]);
      if (L.join_h[i]) cudaFreeHost(L.join_h[i]);
      if (L.h_step_tokens[i]) cudaFreeHost(L.h_step_tokens[i]);
      if (L.h_done[i]) cudaFreeHost(L.h_done[i]);
      if (L.step_done[i]) cudaEventDestroy(L.step_done[i]);
    }
    if (L.adm_h) cudaFreeHost(L.adm_h);
    if (L.own_stream && L.stream) cudaStreamDestroy(L.stream);
    if (L.enc_stream) cudaStreamDestroy(L.enc_stream);
    if (L.enc_done) cudaEventDestroy(L.enc_done);
    if (L.enc_fork) cudaEventDestroy(L.enc_fork);
    if (L.enc_join) cudaEventDestroy(L.enc_join);
  }
  for (cudaEvent_t ev : event_pool) cudaEventDestroy(ev);
  for (void* p : allocations) cudaFree(p);
  if (stream) cudaStreamDestroy(stream);
  for (Request* r : queue) delete r;
  for (Request* r : slot_req) delete r;
}

namespace {

mc_status set_device(mc_engine* e) {
  CK(cudaSetDevice(e->cfg.device));
  return MC_OK;
}

mc_status allocate_lane(mc_engine* e, Lane& L) {
  const int d = e->d, F = e->ffn;
  const int T = e->tmax, R = e->rmax;
  CK(dalloc(e, &L.d_status, 1));
  CK(dalloc(e, &L.enc_x, (size_t)T * d));
  CK(dalloc(e, &L.enc_x1, (size_t)T * d));
  CK(dalloc(e, &L.enc_qkv, (size_t)T * 3 * d));
  CK(dalloc(e, &L.enc_proj, (size_t)T * d));
  // quantized copies: one contiguous block so copy i = base + i * stride
  int8_t* eq = nullptr;
  CK(dalloc(e, &eq, (size_t)kMaxQuantOut * T * d));
  for (int i = 0; i < kMaxQuantOut; ++i) {
    L.enc_q[i].p = eq + (size_t)i * T * d;
    L.enc_q[i].rows = T;
    L.enc_q[i].cols = d;
    if (!encode_tmap_i8(&L.enc_q[i].tmap, L.enc_q[i].p, T, d, 128)) return fail(e, MC_MODEL, "tensor map");
  }
  mc_status st;
  if ((st = make_qbuf(e, &L.enc_o, T, d))) return st;
  if ((st = make_qbuf(e, &L.enc_h, T, F))) return st;
  L.adm_cap = adm_layout(T, R, e->pages_per_slot).end + 16;
  CK(dalloc(e, &L.adm_d, L.adm_cap));
  CK(cudaHostAlloc(&L.adm_h, L.adm_cap * sizeof(int32_t), cudaHostAllocDefault));

  CK(dalloc(e, &L.dec_a, (size_t)R * d));
  CK(dalloc(e, &L.dec_b, (size_t)R * d));
  CK(dalloc(e, &L.dec_qkv, (size_t)R * 3 * d));
  CK(dalloc(e, &L.dec_proj, (size_t)R * d));
  int8_t* dq = nullptr;
  CK(dalloc(e, &dq, (size_t)kMaxQuantOut * R * d));
  for (int i = 0; i < kMaxQuantOut; ++i) {
    L.dec_q[i].p = dq + (size_t)i * R * d;
    L.dec_q[i].rows = R;
    L.dec_q[i].cols = d;
    if (!encode_tmap_i8(&L.dec_q[i].tmap, L.dec_q[i].p, R, d, 128)) return fail(e, MC_MODEL, "tensor map");
  }
  if ((st = make_qbuf(e, &L.dec_o, R, d))) return st;
  if ((st = make_qbuf(e, &L.dec_h, R, F))) return st;
  CK(dalloc(e, &L.rows_d, (size_t)4 + 3 * R));  // zeroed: an empty table
  CK(dalloc(e, &L.rows_scratch, R));
  CK(dalloc(e, &L.join_d, (size_t)1 + R));
  CK(dalloc(e, &L.self_row_map, R));
  CK(dalloc(e, &L.step_tokens, R));
  CK(dalloc(e, &L.eos_mask, R));
  CK(dalloc(e, &L.done, R));
  CK(dalloc(e, &L.best, R));
  for (int i = 0; i < kStepDepth; ++i) {
    CK(cudaHostAlloc(&L.join_h[i], ((size_t)1 + R) * sizeof(int32_t), cudaHostAllocDefault));
    std::memset(L.join_h[i], 0, ((size_t)1 + R) * sizeof(int32_t));
    CK(cudaHostAlloc(&L.h_step_tokens[i], (size_t)R * sizeof(int32_t), cudaHostAllocDefault));
    CK(cudaHostAlloc(&L.h_done[i], (size_t)R, cudaHostAllocDefault));
    CK(cudaHostAlloc(&L.h_status[i], sizeof(uint32_t), cudaHostAllocDefault));
    *L.h_status[i] = 0;
    CK(cudaEventCreateWithFlags(&L.step_done[i], cudaEventDisableTiming));
  }
  return MC_OK;
}

mc_status allocate_buffers(mc_engine* e) {
  const int d = e->d;
  const int R = e->rmax;
  CK(dalloc(e, &e->slot_prev, R));
  CK(dalloc(e, &e->slot_step, R));
  CK(dalloc(e, &e->slot_limit, R));
  CK(dalloc(e, &e->slot_force, R));
  CK(dalloc(e, &e->slot_src, R));
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
  const int group_cols = 4 * (d / e->heads);
  auto kv_maps = [&](const std::vector<float*>& pools, std::vector<KvBoxMaps>* maps) {
    maps->resize(pools.size());
    for (size_t l = 0; l < pools.size(); ++l)
      for (int i = 0; i < 4; ++i)
        if (!encode_tmap_kv(&(*maps)[l].box[i], pools[l], pool_rows, d, e->page_tokens, group_cols, 8 >> i))
          return false;
    return true;
  };
  if (!kv_maps(e->cross_k, &e->cross_k_map) || !kv_maps(e->cross_v, &e->cross_v_map) ||
      !kv_maps(e->self_k, &e->self_k_map) || !kv_maps(e->self_v, &e->self_v_map))
    return fail(e, MC_MODEL, "KV-cache tensor map rejected");
  CK(dalloc(e, &e->cross_pages_d, (size_t)R * e->pages_per_slot));
  CK(dalloc(e, &e->self_pages_d, (size_t)R * e->pages_per_slot));
  e->free_cross.clear();
  e->free_self.clear();
  for (int p = pool - 1; p >= 0; --p) e->free_cross.push_back(p);
  for (int p = e->self_pool_pages - 1; p >= 0; --p) e->free_self.push_back(p);
  e->free_slots.clear();
  for (int s = R - 1; s >= 0; --s) e->free_slots.push_back(s);
  e->slot_req.assign(R, nullptr);

  const int n_lanes = std::max(1, std::min<int>(e->cfg.lanes ? (int)e->cfg.lanes : 1, std::min(kMaxLanes, R)));
  e->lanes.resize(n_lanes);
  int prio_low = 0, prio_high = 0;
  CK(cudaDeviceGetStreamPriorityRange(&prio_low, &prio_high));
  for (int i = 0; i < n_lanes; ++i) {
    Lane& L = e->lanes[i];
    L.id = i;
    L.cap = (R + n_lanes - 1) / n_lanes;
    if (i == 0) {
      L.stream = e->stream;
    } else {
      CK(cudaStreamCreateWithPriority(&L.stream, cudaStreamNonBlocking, prio_high));
      L.own_stream = true;
    }
    CK(cudaStreamCreateWithPriority(&L.enc_stream, cudaStreamNonBlocking, prio_low));
    CK(cudaEventCreateWithFlags(&L.enc_done, cudaEventDisableTiming));
    CK(cudaEventCreateWithFlags(&L.enc_fork, cudaEventDisableTiming));
    CK(cudaEventCreateWithFlags(&L.enc_join, cudaEventDisableTiming));
    L.cur = L.stream;
    mc_status st = allocate_lane(e, L);
    if (st) return st;
  }
  CK(prepare_q8_gemm());
  CK(prepare_q8_linear_ln());
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

// Drops every queued and in-flight request (after a failed step).  Waits for
// every lane's work first: their kernels may still read the slots and pages
// released here.  The lanes' device row tables are emptied.
void abort_all(mc_engine* e) {
  for (Lane& L : e->lanes) {
    cudaStreamSynchronize(L.stream);
    cudaStreamSynchronize(L.enc_stream);
    L.enc_in_flight = false;
    L.cur = L.stream;
    for (auto& r : L.prof_pending) {
      e->event_pool.push_back(r.a);
      e->event_pool.push_back(r.b);
    }
    L.prof_pending.clear();
    timeline_drop(e, L);
    if (L.rows_d) {
      cudaMemsetAsync(L.rows_d, 0, sizeof(int32_t), L.stream);
      cudaStreamSynchronize(L.stream);
    }
  }
  for (Request* r : e->queue) delete r;
  e->queue.clear();
  auto drop = [e](std::vector<int32_t>& list) {
    for (int s : list) {
      Request* r = e->slot_req[s];
      if (r) {
        release_slot(e, r);
        delete r;
      }
    }
    list.clear();
  };
  for (Lane& L : e->lanes) {
    drop(L.active);
    drop(L.ready);
    drop(L.pending);
    for (StepInFlight& F : L.inflight) drop(F.joins);
    L.inflight.clear();
  }
}

// The status bits one completed step read back (its own kernels' and,
// since the word is only cleared here, any earlier ones').
mc_status check_status(mc_engine* e, Lane& L, int parity) {
  const uint32_t bits = *L.h_status[parity];
  if (!bits) return MC_OK;
  for (int i = 0; i < kStepDepth; ++i) *L.h_status[i] = 0;
  CK(cudaMemsetAsync(L.d_status, 0, sizeof(uint32_t), L.stream));
  CK(cudaStreamSynchronize(L.stream));
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

// Rows of lane L occupying slots: applied, joined or waiting to join, in
// enqueued steps, or waiting for their encoder pass.
size_t lane_rows(const Lane& L) {
  size_t n = L.active.size() + L.ready.size() + L.pending.size();
  for (const StepInFlight& F : L.inflight) n += F.joins.size();
  return n;
}

// Admits queued requests into free slots of lane L and enqueues one packed
// encoder pass for them on the lane's encoder stream, which runs alongside
// the lane's decode steps; the admitted slots wait in L.pending until the
// pass completes (join_pending).  Asynchronous: the staging block is pinned
// and the lane's previous pass has completed.  `cap` overrides the lane's
// row limit (per-layer capture).  With profiling on, the pass runs on the
// decode stream so kernel times are not shared.
mc_status admit(mc_engine* e, Lane& L, int cap) {
  if (L.enc_in_flight) return MC_OK;
  int T = 0;
  const int pt = e->page_tokens;
  const int pps = e->pages_per_slot;
  const int used = (int)lane_rows(L);
  const size_t room = cap > used ? (size_t)(cap - used) : 0;
  const size_t avail = std::min(room, e->free_slots.size());
  // Admission granularity: an encoder pass over a handful of sources costs
  // nearly as much launch latency as one over hundreds, so wait until an
  // eighth of the lane is free -- unless the lane is idle or the whole
  // queue fits (which keeps latency low under light load).
  if (avail == 0 || e->queue.empty()) return MC_OK;
  const bool decoding = !L.active.empty() || !L.ready.empty() || !L.inflight.empty();
  if (decoding && avail < (size_t)std::max(1, cap / 8) && e->queue.size() > avail) return MC_OK;
  std::vector<Request*> admitted;
  while (!e->queue.empty() && admitted.size() < avail) {
    Request* r = e->queue.front();
    const int len = (int)r->tokens.size();
    const uint32_t lim = request_limit(e, r);
    if (lim == 0) {  // nothing to generate
      e->queue.pop_front();
      finish_request(e, r);
      continue;
    }
    if (T + len > e->tmax) break;
    const int need_c = (len + pt - 1) / pt;
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
    e->slot_req[r->slot] = r;
    T += len;
    admitted.push_back(r);
  }
  const int B = (int)admitted.size();
  if (B == 0) return MC_OK;
  const AdmLayout A = adm_layout(T, B, pps);
  int32_t* h = L.adm_h;
  int32_t *tok = h + A.tok, *pos = h + A.pos, *crow = h + A.crow, *cu = h + A.cu,
          *slots = h + A.slots, *lims = h + A.lims, *force = h + A.force, *src = h + A.src,
          *seq_ids = h + A.seq_ids, *pages = h + A.pages;
  int t = 0;
  double sum_len_sq = 0;
  cu[0] = 0;
  for (int b = 0; b < B; ++b) {
    Request* r = admitted[b];
    const int len = (int)r->tokens.size();
    for (int i = 0; i < len; ++i, ++t) {
      tok[t] = r->tokens[i];
      pos[t] = i;
      crow[t] = r->cross_pages[i / pt] * pt + i % pt;
    }
    cu[b + 1] = t;
    sum_len_sq += (double)len * len;
    slots[b] = r->slot;
    lims[b] = (int32_t)request_limit(e, r);
    force[b] = (int32_t)r->force;
    src[b] = len;
    int32_t* cp = pages + (size_t)b * pps;
    int32_t* sp = pages + ((size_t)B + b) * pps;
    for (int i = 0; i < pps; ++i) {
      cp[i] = i < (int)r->cross_pages.size() ? r->cross_pages[i] : 0;
      sp[i] = i < (int)r->self_pages.size() ? r->self_pages[i] : 0;
    }
  }
  // length buckets for the encoder attention (shared memory follows length)
  L.buckets.clear();
  {
    const int bounds[4] = {32, 64, 128, kMaxSeq};
    int off = 0, lo = 0;
    for (int hi : bounds) {
      const int start = off;
      for (int b = 0; b < B; ++b)
        if (src[b] > lo && src[b] <= hi) seq_ids[off++] = b;
      if (off > start) L.buckets.push_back({start, off - start, hi});
      lo = hi;
    }
  }
  cudaStream_t s = e->profiling ? L.stream : L.enc_stream;
  for (Request* r : admitted) L.pending.push_back(r->slot);
  L.enc_in_flight = true;
  L.cur = s;
  CK(cudaMemcpyAsync(L.adm_d, L.adm_h, A.end * sizeof(int32_t), cudaMemcpyHostToDevice, s));
  L.enc_alone = true;
  for (const Lane& X : e->lanes)
    if (!X.active.empty() || !X.inflight.empty()) L.enc_alone = false;
  mc_status st = run_encoder(e, L, A, sum_len_sq);
  L.cur = L.stream;
  if (st) return st;
  const int32_t* ad = L.adm_d;
  launch_init_slots(B, ad + A.slots, ad + A.lims, ad + A.force, ad + A.src, e->slot_prev,
                    e->slot_step, e->slot_limit, e->slot_force, e->slot_src, e->ssru_state,
                    e->dec_layers, e->rmax, e->d, ad + A.pages, e->cross_pages_d,
                    e->kind == 1 ? e->self_pages_d : nullptr, pps, s);
  ++e->launches;
  if (e->has_shortlist) {
    launch_shortlist_masks(B, ad + A.slots, ad + A.tok, ad + A.cu, e->sl_offsets, e->sl_targets,
                           e->sl_first_num, e->vtgt, e->sl_masks, s);
    ++e->launches;
  }
  CK(cudaEventRecord(L.enc_done, s));
  return MC_OK;
}

// Moves the slots of lane L's completed admission to its ready list (the
// next step's row table appends them) and orders the lane's decode stream
// after the encoder pass.  With wait = false an encoder pass still running
// is left pending.
mc_status join_pending(mc_engine* e, Lane& L, bool wait) {
  if (!L.enc_in_flight) return MC_OK;
  if (wait) {
    CK(cudaEventSynchronize(L.enc_done));
  } else {
    const cudaError_t q = cudaEventQuery(L.enc_done);
    if (q == cudaErrorNotReady) return MC_OK;
    CK(q);
  }
  CK(cudaStreamWaitEvent(L.stream, L.enc_done, 0));
  L.ready.insert(L.ready.end(), L.pending.begin(), L.pending.end());
  L.pending.clear();
  L.enc_in_flight = false;
  return MC_OK;
}

// The device work of one decode step of lane L, grids sized for `cap` rows:
// the join block upload, the row table (launch_step_rows), the step's
// kernels, and the read-back of `cap` tokens, finished flags and the status
// word into the parity's pinned buffers.
mc_status enqueue_step(mc_engine* e, Lane& L, int cap, int parity, const std::vector<int32_t>& rows) {
  cudaStream_t s = L.stream;
  CK(cudaMemcpyAsync(L.join_d, L.join_h[parity], ((size_t)1 + cap) * sizeof(int32_t),
                     cudaMemcpyHostToDevice, s));
  launch_step_rows(L.rows_d, e->rmax, L.done, L.join_d, e->slot_step, e->slot_src, L.rows_scratch,
                   L.d_status, s);
  ++e->launches;
  mc_status st = run_decode_step(e, L, cap, rows);
  if (st) return st;
  CK(cudaMemcpyAsync(L.h_step_tokens[parity], L.step_tokens, (size_t)cap * 4, cudaMemcpyDeviceToHost, s));
  CK(cudaMemcpyAsync(L.h_done[parity], L.done, (size_t)cap, cudaMemcpyDeviceToHost, s));
  CK(cudaMemcpyAsync(L.h_status[parity], L.d_status, 4, cudaMemcpyDeviceToHost, s));
  return MC_OK;
}

// Captures lane L's decode step for L.cap rows as a CUDA graph (one per
// parity: they differ in the pinned buffers).  A failed capture is not an
// error: the lane keeps launching eagerly.
void capture_step(mc_engine* e, Lane& L, int parity) {
  L.graph_tried[parity] = true;
  const std::string saved_error = e->error;
  const bool saved_ready = e->ready;
  const uint64_t launches0 = e->launches;
  cudaGraph_t g = nullptr;
  bool ok = cudaStreamBeginCapture(L.stream, cudaStreamCaptureModeThreadLocal) == cudaSuccess;
  if (ok) {
    const mc_status st = enqueue_step(e, L, L.cap, parity, {});
    ok = cudaStreamEndCapture(L.stream, &g) == cudaSuccess && st == MC_OK && g != nullptr;
  }
  if (ok) ok = cudaGraphInstantiate(&L.graph[parity], g, 0) == cudaSuccess;
  if (g) cudaGraphDestroy(g);
  if (!ok) {
    if (L.graph[parity]) cudaGraphExecDestroy(L.graph[parity]);
    L.graph[parity] = nullptr;
    cudaGetLastError();
    e->error = saved_error;
    e->ready = saved_ready;
  }
  L.graph_kernels = e->launches - launches0;
  e->launches = launches0;
}

// Rows the next step of lane L can have at most: those of its newest
// enqueued step (some may finish in it), or the applied survivors, plus the
// slots ready to join.
size_t next_step_bound(const Lane& L) {
  const size_t base = L.inflight.empty() ? L.active.size() : (size_t)L.inflight.back().rows_bound;
  return base + L.ready.size();
}

// Enqueues one decode step of lane L (asynchronous): its row table appends
// the ready slots.  Grids cover the lane's capacity when the step replays
// the parity's graph, else the step's row bound.
mc_status launch_decode(mc_engine* e, Lane& L, bool allow_graph) {
  const size_t bound = next_step_bound(L);
  if (bound == 0) return MC_OK;
  StepInFlight F;
  F.parity = L.next_parity;
  F.rows_bound = (int)bound;
  F.joins.swap(L.ready);
  int32_t* jb = L.join_h[F.parity];
  jb[0] = (int32_t)F.joins.size();
  if (!F.joins.empty()) std::memcpy(jb + 1, F.joins.data(), F.joins.size() * 4);
  const bool graph_ok = allow_graph && e->use_graphs && !e->profiling && (int)bound <= L.cap &&
                        L.eager_steps > 0;
  if (graph_ok && !L.graph_tried[F.parity]) capture_step(e, L, F.parity);
  if (e->timeline) {
    F.tl_start = pooled_event(e);
    F.tl_end = pooled_event(e);
    CK(cudaEventRecord(F.tl_start, L.stream));
  }
  if (graph_ok && L.graph[F.parity]) {
    CK(cudaGraphLaunch(L.graph[F.parity], L.stream));
    e->launches += L.graph_kernels;
  } else {
    std::vector<int32_t> rows;
    if (e->profiling && L.inflight.empty()) {  // exact rows for the profile's counts
      rows = L.active;
      rows.insert(rows.end(), F.joins.begin(), F.joins.end());
    }
    mc_status st = enqueue_step(e, L, (int)bound, F.parity, rows);
    if (st) return st;
    ++L.eager_steps;
  }
  if (e->timeline) CK(cudaEventRecord(F.tl_end, L.stream));
  CK(cudaEventRecord(L.step_done[F.parity], L.stream));
  L.next_parity = (F.parity + 1) % kStepDepth;
  L.inflight.push_back(std::move(F));
  return MC_OK;
}

// Waits for lane L's oldest enqueued step and applies its tokens: its rows
// are the applied survivors followed by its joins (the order its row table
// has on the device); each appends its token, and finished rows retire and
// release their slot and pages.
mc_status apply_step(mc_engine* e, Lane& L) {
  if (L.inflight.empty()) return MC_OK;
  StepInFlight& F = L.inflight.front();
  CK(cudaEventSynchronize(L.step_done[F.parity]));
  prof_harvest(e, L);
  timeline_harvest(e, L, F);
  ++e->steps;
  mc_status st = check_status(e, L, F.parity);
  if (st) return st;
  const int32_t* tok = L.h_step_tokens[F.parity];
  const uint8_t* fin = L.h_done[F.parity];
  std::vector<int32_t> keep;
  keep.reserve(L.active.size() + F.joins.size());
  int r = 0;
  for (const std::vector<int32_t>* part : {&L.active, &F.joins})
    for (int slot : *part) {
      Request* q = e->slot_req[slot];
      q->output.push_back(tok[r]);
      if (fin[r]) finish_request(e, q);
      else keep.push_back(slot);
      ++r;
    }
  L.active.swap(keep);
  L.inflight.pop_front();
  if (!L.inflight.empty())  // the next step's rows are now known exactly
    L.inflight.front().rows_bound = (int)(L.active.size() + L.inflight.front().joins.size());
  return MC_OK;
}

// Rows admitted to any lane: decoding, or waiting for their encoder pass.
size_t total_active(const mc_engine* e) {
  size_t n = 0;
  for (const Lane& L : e->lanes) n += lane_rows(L);
  return n;
}

// One scheduler step.  Each lane in turn: applies its oldest step once
// kStepDepth are enqueued (so the next step, already on the GPU, runs while
// the host applies tokens and retires rows), joins a completed admission,
// enqueues its next step, then admits queued requests (that host work and
// the encoder pass overlap the decode steps).  An idle lane admits first and
// waits for the encoder pass.  With profiling on, each step is applied as
// soon as it is enqueued, so the per-kernel times are not shared with
// another step or lane.
mc_status engine_step(mc_engine* e) {
  if (!e->loaded) return fail(e, MC_MODEL, "no model loaded");
  if (!e->ready) return fail(e, MC_INFERENCE, "engine is not ready after a device failure");
  mc_status st = set_device(e);
  if (st) return st;
  const size_t depth = e->profiling ? 1 : kStepDepth;
  for (Lane& L : e->lanes) {
    while (L.inflight.size() >= depth)
      if ((st = apply_step(e, L))) return st;
    if ((st = join_pending(e, L, false))) {
      abort_all(e);
      return st;
    }
    bool admitted = false;
    if (next_step_bound(L) == 0 && L.inflight.empty()) {
      // idle lane: admit, wait for the encoder pass, then decode its rows
      st = admit(e, L, L.cap);
      if (!st) st = join_pending(e, L, true);
      admitted = true;
    }
    if (!st) {
      if (next_step_bound(L) > 0) st = launch_decode(e, L, true);
      else st = apply_step(e, L);  // nothing to enqueue behind the last step
    }
    if (!st && !admitted) st = admit(e, L, L.cap);
    if (st) {
      abort_all(e);
      return st;
    }
    while (e->profiling && !L.inflight.empty())
      if ((st = apply_step(e, L))) return st;
  }
  return MC_OK;
}

// Applies every lane's enqueued steps (used before returning results that
// must be whole).
mc_status drain_lanes(mc_engine* e) {
  mc_status st;
  for (Lane& L : e->lanes)
    while (!L.inflight.empty())
      if ((st = apply_step(e, L))) return st;
  return MC_OK;
}

mc_status validate_source(const mc_engine* e, const int32_t* tokens, size_t n, std::string* why);

// shortlist.rs:193-196: a sentence whose candidates lack EOS is an error.
mc_status validate_shortlist(const mc_engine* e, const int32_t* tokens, size_t n, std::string* why) {
  if (!e->has_shortlist || e->sl_first_num > 0) return MC_OK;
  for (size_t i = 0; i < n; ++i)
    if (e->sl_maps_eos[tokens[i]]) return MC_OK;
  *why = "lexical shortlist does not contain EOS token 0";
  return MC_INFERENCE;
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
  return validate_shortlist(e, tokens, n, why);
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
  cfg->lanes = 1;
}

extern "C" mc_status mc_create(const mc_config* cfg, mc_engine** out) {
  if (!cfg || !out) return MC_INVALID_INPUT;
  *out = nullptr;
  if (cfg->max_inflight == 0 || cfg->max_inflight > 65536 || cfg->max_encode_tokens < 256 ||
      (cfg->page_tokens != 8 && cfg->page_tokens != 16 && cfg->page_tokens != 32) ||
      cfg->max_length_factor < 1 ||
      cfg->max_length_factor > 8 || cfg->lanes > (uint32_t)kMaxLanes)
    return MC_INVALID_INPUT;
  mc_engine* e = new mc_engine();
  if (const char* v = std::getenv("MARIAN_CUDA_FUSED_LN")) e->fuse_ln = std::strcmp(v, "0") != 0;
  e->cfg = *cfg;
  mc_status st = set_device(e);
  if (st == MC_OK) {
    int lowest = 0, highest = 0;
    cudaError_t r = cudaDeviceGetStreamPriorityRange(&lowest, &highest);
    // decode steps are the latency chain: their streams get the highest
    // priority, encoder passes fill in at the lowest
    if (r == cudaSuccess) r = cudaStreamCreateWithPriority(&e->stream, cudaStreamNonBlocking, highest);
    if (r != cudaSuccess) st = MC_CUDA;
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
    if (!std::isfinite(v.scale) || v.scale <= 0.0f)
      return fail(e, MC_MODEL, "decoder_Wemb: 1 / (activation scale * quantization multiplier) is not finite");
    std::vector<float> cs(e->vtgt, v.scale);
    CK(dalloc(e, &v.col_scale, cs.size()));
    CK(h2d(e, v.col_scale, cs.data(), cs.size() * 4));
    for (int i = 0; i < 3; ++i)
      if (!encode_tmap_i8(&v.tmap_b[i], v.w, v.out, v.in, kBNs[i]))
        return fail(e, MC_MODEL, "vocabulary tensor map rejected");
    // full-vocabulary candidates: every id but 1 and 7..38 (shortlist.rs:150-198),
    // folded into the bias: a non-candidate logit is -inf and never wins the
    // strict '>' argmax; the bias is padded with -inf to whole 32-id chunks
    const HostTensor& tb = m.tensors.at("decoder_ff_logit_out_b");
    if ((int)tb.f32.size() != e->vtgt) return fail(e, MC_MODEL, "decoder_ff_logit_out_b has the wrong size");
    std::vector<float> masked((size_t)(e->vtgt + 255) / 256 * 256, -INFINITY);
    for (int id = 0; id < e->vtgt; ++id) masked[id] = tb.f32[id];
    if (e->vtgt > 1) masked[1] = -INFINITY;
    for (int id = 7; id < std::min(e->vtgt, 39); ++id) masked[id] = -INFINITY;
    CK(dalloc(e, &v.bias, masked.size()));
    CK(h2d(e, v.bias, masked.data(), masked.size() * 4));
    e->weight_bytes += (size_t)e->vtgt * 4;
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
  if (active_after) *active_after = (uint32_t)total_active(e);
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
  if (!e->queue.empty() || total_active(e) != 0)
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
  std::vector<Request*> reqs(batch);
  for (uint32_t b = 0; b < batch; ++b) {
    Request* r = new Request();
    r->id = b;
    r->tokens.assign(tokens + offsets[b], tokens + offsets[b + 1]);
    r->max_out = max_out[b];
    r->force = force_len ? force_len[b] : 0;
    reqs[b] = r;
  }
  // Longest first: the rows of a batch are independent (results come back
  // by request id), so admitting those with the most decode steps first
  // keeps the slots full to the end instead of leaving a tail of steps with
  // few active rows; equal step bounds keep the submission order.
  std::stable_sort(reqs.begin(), reqs.end(), [e](const Request* a, const Request* b) {
    return request_limit(e, a) > request_limit(e, b);
  });
  for (Request* r : reqs) e->queue.push_back(r);
  const uint64_t step_bound = (uint64_t)batch * (kMaxSeq + 2) + 16;
  for (uint64_t i = 0; i < step_bound && (!e->queue.empty() || total_active(e) != 0); ++i) {
    if ((st = engine_step(e))) {
      abort_all(e);
      e->finished.clear();
      return st;
    }
  }
  if ((st = drain_lanes(e))) {
    abort_all(e);
    e->finished.clear();
    return st;
  }
  if (!e->queue.empty() || total_active(e) != 0) {
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

// Encoder pass only (Q8CpuEngine::encode and the cross-cache fill,
// q8_engine.rs:511-574): the batch is admitted as one packed encoder pass
// on lane 0's stream, its cross keys/values are written into cache pages,
// and every slot is released again without a decode step.
extern "C" mc_status mc_encode_token_ids(mc_engine* e, const int32_t* tokens, size_t n_tokens,
                                         const uint32_t* offsets, uint32_t batch,
                                         float* encoder_output) {
  if (!e) return MC_INVALID_INPUT;
  mc_status st = validate_batch(e, tokens, n_tokens, offsets, batch);
  if (st) return st;
  if (batch > (uint32_t)e->rmax || n_tokens > (size_t)e->tmax)
    return fail(e, MC_INVALID_INPUT, "batch exceeds one encoder pass (max_inflight, max_encode_tokens)");
  if ((st = set_device(e))) return st;
  Lane& L = e->lanes[0];
  for (uint32_t b = 0; b < batch; ++b) {
    Request* r = new Request();
    r->id = b;
    r->tokens.assign(tokens + offsets[b], tokens + offsets[b + 1]);
    r->max_out = kMaxSeq;
    r->force = 0;
    e->queue.push_back(r);
  }
  if ((st = admit(e, L, e->rmax)) || (st = join_pending(e, L, true))) {
    abort_all(e);
    return st;
  }
  if (L.ready.size() != batch) {
    abort_all(e);
    return fail(e, MC_INVALID_INPUT, "batch does not fit the free slots or pages");
  }
  CK(cudaStreamSynchronize(L.stream));
  prof_harvest(e, L);
  if (encoder_output)
    CK(cudaMemcpy(encoder_output, L.enc_x, n_tokens * (size_t)e->d * 4, cudaMemcpyDeviceToHost));
  abort_all(e);
  return MC_OK;
}

// Arrival-schedule replay on the calling thread: request b (the packed
// batch's row b) is submitted once arrival_s[b] seconds have passed since
// the call began (arrival_s ascending), mc_step runs while anything is
// queued or decoding, and latency_s[b] receives the time from its arrival to
// the step that returned its last token.  The tokens themselves are
// dropped.  This is the scheduler worker loop's shape
// (marian-core/src/scheduler.rs:494-659) with the host clock as the
// arrival process.
extern "C" mc_status mc_replay(mc_engine* e, const int32_t* tokens, size_t n_tokens,
                               const uint32_t* offsets, uint32_t batch, const uint32_t* max_out,
                               const uint32_t* force_len, const double* arrival_s, double* latency_s) {
  if (!e) return MC_INVALID_INPUT;
  mc_status st = validate_batch(e, tokens, n_tokens, offsets, batch);
  if (st) return st;
  if (!max_out || !arrival_s || !latency_s) return fail(e, MC_INVALID_INPUT, "null replay buffers");
  for (uint32_t b = 1; b < batch; ++b)
    if (!(arrival_s[b] >= arrival_s[b - 1])) return fail(e, MC_INVALID_INPUT, "arrivals are not ascending");
  using clock = std::chrono::steady_clock;
  const auto t0 = clock::now();
  auto now = [&]() { return std::chrono::duration<double>(clock::now() - t0).count(); };
  e->finished.clear();
  uint32_t next = 0, done = 0;
  while (done < batch) {
    double t = now();
    for (; next < batch && arrival_s[next] <= t; ++next) {
      Request* r = new Request();
      r->id = next;
      r->tokens.assign(tokens + offsets[next], tokens + offsets[next + 1]);
      r->max_out = max_out[next];
      r->force = force_len ? force_len[next] : 0;
      e->queue.push_back(r);
    }
    if (e->queue.empty() && total_active(e) == 0) {
      if (next >= batch) break;
      while (now() < arrival_s[next]) {
      }  // idle until the next arrival
      continue;
    }
    if ((st = engine_step(e))) {
      abort_all(e);
      e->finished.clear();
      return st;
    }
    t = now();
    for (const Finished& f : e->finished) {
      if (f.id < batch) latency_s[f.id] = t - arrival_s[f.id];
      ++done;
    }
    e->finished.clear();
  }
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
  Lane& L = e->lanes[0];
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
  if ((st = admit(e, L, e->rmax)) || (st = join_pending(e, L, true))) {
    abort_all(e);
    return st;
  }
  if (L.ready.size() != batch) {
    abort_all(e);
    return fail(e, MC_INVALID_INPUT, "trace batch does not fit the free slots or pages");
  }
  CK(cudaStreamSynchronize(L.stream));
  const int d = e->d;
  const size_t row_bytes = (size_t)d * 4;
  if (encoder_output) {
    for (uint32_t b = 0; b < batch; ++b)
      for (uint32_t i = 0; i < offsets[b + 1] - offsets[b]; ++i)
        CK(cudaMemcpy(encoder_output + ((size_t)b * lmax + i) * d, L.enc_x + (size_t)(offsets[b] + i) * d,
                      row_bytes, cudaMemcpyDeviceToHost));
  }
  for (int l = 0; l < e->dec_layers && (cross_key || cross_value); ++l)
    for (uint32_t b = 0; b < batch; ++b) {
      const Request* r = e->slot_req[L.ready[b]];
      for (uint32_t i = 0; i < offsets[b + 1] - offsets[b]; ++i) {
        const size_t row = (size_t)r->cross_pages[i / e->page_tokens] * e->page_tokens + i % e->page_tokens;
        const size_t dst = (((size_t)l * batch + b) * lmax + i) * d;
        if (cross_key)
          CK(cudaMemcpy(cross_key + dst, e->cross_k[l] + row * d, row_bytes, cudaMemcpyDeviceToHost));
        if (cross_value)
          CK(cudaMemcpy(cross_value + dst, e->cross_v[l] + row * d, row_bytes, cudaMemcpyDeviceToHost));
      }
    }
  if ((st = launch_decode(e, L, false))) {
    abort_all(e);
    return st;
  }
  CK(cudaStreamSynchronize(L.stream));
  prof_harvest(e, L);
  if ((st = check_status(e, L, L.inflight.front().parity))) return st;
  if (decoder_state)
    CK(cudaMemcpy(decoder_state, L.last_state, (size_t)batch * row_bytes, cudaMemcpyDeviceToHost));
  abort_all(e);
  return MC_OK;
}

namespace {

uint64_t read_le64(const uint8_t* p) {
  uint64_t v = 0;
  for (int i = 7; i >= 0; --i) v = (v << 8) | p[i];
  return v;
}

uint32_t read_le32(const uint8_t* p) {
  return (uint32_t)p[0] | ((uint32_t)p[1] << 8) | ((uint32_t)p[2] << 16) | ((uint32_t)p[3] << 24);
}

// LexicalShortlist::from_bytes (marian-model/src/shortlist.rs:59-148).
std::string parse_shortlist(const uint8_t* b, size_t len, uint64_t source_vocab, uint64_t target_vocab,
                            uint64_t* first_num, std::vector<uint64_t>* offsets,
                            std::vector<uint32_t>* targets) {
  constexpr uint64_t kMagic = 17373278592220534773ull;     // shortlist.rs:3
  constexpr uint64_t kMaxTargets = 4000000;                // shortlist.rs:4
  const uint64_t maximum = 48 + (source_vocab + 1) * 8 + kMaxTargets * 4;
  if (len > maximum)
    return "lexical shortlist has " + std::to_string(len) + " bytes; maximum is " + std::to_string(maximum);
  if (len < 48) return "truncated lexical shortlist header";
  const uint64_t magic = read_le64(b), fn = read_le64(b + 16), n_off = read_le64(b + 32),
                 n_tgt = read_le64(b + 40);
  if (magic != kMagic || n_off != source_vocab + 1 || fn > target_vocab || n_tgt > kMaxTargets)
    return "unsupported lexical shortlist format";
  const uint64_t expected = 48 + n_off * 8 + n_tgt * 4;
  if (len != expected)
    return "lexical shortlist has " + std::to_string(len) + " bytes, expected " + std::to_string(expected);
  offsets->resize(n_off);
  for (uint64_t i = 0; i < n_off; ++i) (*offsets)[i] = read_le64(b + 48 + 8 * i);
  bool bad = offsets->front() != 0 || offsets->back() != n_tgt;
  for (uint64_t i = 1; i < n_off && !bad; ++i)
    bad = (*offsets)[i - 1] > (*offsets)[i] || (*offsets)[i] > n_tgt;
  if (bad) return "lexical shortlist offsets are invalid";
  targets->resize(n_tgt);
  const uint8_t* tp = b + 48 + n_off * 8;
  for (uint64_t i = 0; i < n_tgt; ++i) {
    const uint32_t t = read_le32(tp + 4 * i);
    if (t >= target_vocab)
      return "lexical shortlist target " + std::to_string(t) + " exceeds vocabulary " +
             std::to_string(target_vocab);
    (*targets)[i] = t;
  }
  *first_num = fn;
  return "";
}

}  // namespace

extern "C" mc_status mc_load_shortlist(mc_engine* e, const uint8_t* bytes, size_t len) {
  if (!e) return MC_INVALID_INPUT;
  if (!e->loaded) return fail(e, MC_MODEL, "no model loaded");
  if (!e->queue.empty() || total_active(e) != 0)
    return fail(e, MC_INVALID_INPUT, "engine has requests in flight");
  mc_status st = set_device(e);
  if (st) return st;
  if ((st = drain_lanes(e))) return st;  // no step may run with the graphs replaced below
  if (!bytes) {  // back to the full vocabulary
    e->has_shortlist = false;
  } else {
    uint64_t first_num = 0;
    std::vector<uint64_t> offsets;
    std::vector<uint32_t> targets;
    const std::string err = parse_shortlist(bytes, len, (uint64_t)e->vsrc, (uint64_t)e->vtgt, &first_num,
                                            &offsets, &targets);
    if (!err.empty()) return fail(e, MC_MODEL, err);
    if (e->vtgt > 393216) return fail(e, MC_MODEL, "target vocabulary too large for a shortlist");
    std::vector<int32_t> off32(offsets.begin(), offsets.end()), tg32(targets.begin(), targets.end());
    if (tg32.empty()) tg32.push_back(0);
    e->sl_maps_eos.assign(e->vsrc, 0);
    for (int t = 0; t < e->vsrc; ++t)
      for (uint64_t j = offsets[t]; j < offsets[t + 1]; ++j)
        if (targets[j] == 0) e->sl_maps_eos[t] = 1;
    // allocations grow only; they are released with the engine
    CK(dalloc(e, &e->sl_offsets, off32.size()));
    CK(h2d(e, e->sl_offsets, off32.data(), off32.size() * 4));
    CK(dalloc(e, &e->sl_targets, tg32.size()));
    CK(h2d(e, e->sl_targets, tg32.data(), tg32.size() * 4));
    e->sl_words = (e->vtgt + 31) / 32;
    if (!e->sl_masks) CK(dalloc(e, &e->sl_masks, (size_t)e->rmax * e->sl_words));
    e->sl_first_num = (int)first_num;
    e->has_shortlist = true;
  }
  // the decode graphs captured so far bake the vocabulary launch's arguments
  for (Lane& L : e->lanes) {
    for (int i = 0; i < kStepDepth; ++i) {
      if (L.graph[i]) cudaGraphExecDestroy(L.graph[i]);
      L.graph[i] = nullptr;
      L.graph_tried[i] = false;
    }
    L.eager_steps = 0;
  }
  return MC_OK;
}

extern "C" mc_status mc_profile(mc_engine* e, int32_t enable) {
  if (!e) return MC_INVALID_INPUT;
  for (Lane& L : e->lanes) {
    cudaStreamSynchronize(L.stream);
    prof_harvest(e, L);
  }
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

extern "C" mc_status mc_timeline(mc_engine* e, int32_t enable) {
  if (!e) return MC_INVALID_INPUT;
  for (Lane& L : e->lanes) {
    cudaStreamSynchronize(L.stream);
    timeline_drop(e, L);
  }
  e->timeline = enable != 0;
  e->tl_steps = 0;
  e->tl_busy_ms = e->tl_gap_ms = 0.0;
  return MC_OK;
}

extern "C" mc_status mc_timeline_read(const mc_engine* e, uint64_t* steps, double* busy_ms,
                                      double* idle_ms) {
  if (!e) return MC_INVALID_INPUT;
  if (steps) *steps = e->tl_steps;
  if (busy_ms) *busy_ms = e->tl_busy_ms;
  if (idle_ms) *idle_ms = e->tl_gap_ms;
  return MC_OK;
}
