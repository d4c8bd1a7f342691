// kernels.cu -- embedding, residual LayerNorm, SSRU, attention and token
// selection kernels of the Q8 greedy path (sm_100a).
//
// Built with --fmad=false: every expression below rounds after each
// multiply and each add, matching the reference's Rust f32 arithmetic
// (crates/marian-cpu/src/tensor.rs).  exp() is evaluated in double precision
// and rounded once to f32, i.e. the correctly rounded expf in all but
// double-rounding corner cases; the reference's libm expf is correctly
// rounded to within a few thousandths of an ulp, so the two agree except on
// rare inputs.
#include <algorithm>

#include "common.cuh"
#include "kernels.cuh"

namespace mc {

namespace {

constexpr float kLnEps = 1.0e-6f;  // tensor.rs:3

// Rows of a launch: the device count when given (launches replayed from a
// CUDA graph, whose grids cover `cap` rows), else cap.
__device__ __forceinline__ int launch_rows(const int32_t* rows_dev, int cap) {
  return rows_dev ? max(0, min(*rows_dev, cap)) : cap;
}

__device__ __forceinline__ float exp_f32(float x) {
  return static_cast<float>(exp(static_cast<double>(x)));
}

__device__ __forceinline__ void store_quant4(const QuantOut& q, long long elem, float a, float b,
                                             float c, float d, uint32_t* status) {
  for (int i = 0; i < q.count; ++i) {
    const float al = q.alpha[i];
    const uint32_t w = (uint32_t)(uint8_t)quantize_one(a, al, status) |
                       ((uint32_t)(uint8_t)quantize_one(b, al, status) << 8) |
                       ((uint32_t)(uint8_t)quantize_one(c, al, status) << 16) |
                       ((uint32_t)(uint8_t)quantize_one(d, al, status) << 24);
    *reinterpret_cast<uint32_t*>(q.base + i * q.stride + elem) = w;
  }
}

// ---- embeddings ----------------------------------------------------------------
__global__ void embed_encoder_kernel(const int32_t* __restrict__ tokens,
                                     const int32_t* __restrict__ pos_idx, int n_tokens,
                                     const int8_t* __restrict__ emb, float emb_mult,
                                     float emb_scale, const float* __restrict__ positions, int d,
                                     float* __restrict__ x, const __grid_constant__ QuantOut q, uint32_t* status) {
  pdl_enter();
  const int vec_per_row = d >> 2;
  const long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= (long long)n_tokens * vec_per_row) return;
  const int t = static_cast<int>(idx / vec_per_row);
  const int c = static_cast<int>(idx % vec_per_row) * 4;
  const int tok = tokens[t];
  const int p = pos_idx[t];
  const char4 e = *reinterpret_cast<const char4*>(emb + (size_t)tok * d + c);
  const float4 pe = *reinterpret_cast<const float4*>(positions + (size_t)p * d + c);
  float4 v;
  v.x = (float)e.x / emb_mult * emb_scale + pe.x;
  v.y = (float)e.y / emb_mult * emb_scale + pe.y;
  v.z = (float)e.z / emb_mult * emb_scale + pe.z;
  v.w = (float)e.w / emb_mult * emb_scale + pe.w;
  const long long elem = (long long)t * d + c;
  *reinterpret_cast<float4*>(x + elem) = v;
  store_quant4(q, elem, v.x, v.y, v.z, v.w, status);
}

__global__ void embed_decoder_kernel(int cap, const int32_t* __restrict__ rows_dev,
                                     const int32_t* __restrict__ row_slot,
                                     const int32_t* __restrict__ slot_prev,
                                     const int32_t* __restrict__ slot_step,
                                     const int32_t* __restrict__ slot_force,
                                     const int8_t* __restrict__ emb, float emb_mult,
                                     float emb_scale, const float* __restrict__ positions, int d,
                                     float* __restrict__ x, const __grid_constant__ QuantOut q, uint8_t* eos_mask,
                                     const int32_t* __restrict__ self_pages, int pages_per_slot,
                                     int page_tokens, int32_t* self_row_map, uint32_t* status) {
  pdl_enter();
  const int rows = launch_rows(rows_dev, cap);
  const int vec_per_row = d >> 2;
  const long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= (long long)rows * vec_per_row) return;
  const int r = static_cast<int>(idx / vec_per_row);
  const int c = static_cast<int>(idx % vec_per_row) * 4;
  const int slot = row_slot[r];
  const int prev = slot_prev[slot];
  const int t = slot_step[slot];
  if (t < 0 || t >= kMaxPosition) {
    flag_status(status, kStatusBadIndex);
    return;
  }
  const float4 pe = *reinterpret_cast<const float4*>(positions + (size_t)t * d + c);
  float4 v = pe;
  if (prev >= 0) {
    const char4 e = *reinterpret_cast<const char4*>(emb + (size_t)prev * d + c);
    v.x = (float)e.x / emb_mult * emb_scale + pe.x;
    v.y = (float)e.y / emb_mult * emb_scale + pe.y;
    v.z = (float)e.z / emb_mult * emb_scale + pe.z;
    v.w = (float)e.w / emb_mult * emb_scale + pe.w;
  }
  const long long elem = (long long)r * d + c;
  *reinterpret_cast<float4*>(x + elem) = v;
  store_quant4(q, elem, v.x, v.y, v.z, v.w, status);
  if (c == 0) {
    const int force = slot_force[slot];
    eos_mask[r] = (force > 0 && t + 1 < force) ? 1 : 0;
    if (self_pages) {
      const int page = self_pages[(size_t)slot * pages_per_slot + t / page_tokens];
      self_row_map[r] = page * page_tokens + t % page_tokens;
    }
  }
}

// ---- LayerNorm (normalize_row, tensor.rs:372-385) ------------------------------
// A CTA of 4 warps normalizes RPC = 8 rows.  The warps load the rows
// with coalesced 128-bit accesses, form the pre-norm values and stage them in
// shared memory (row stride d + 4 floats, so lanes reading different rows
// at the same column hit distinct banks).  Then lane i of warp 0 owns row i:
// it sums the row left to right, exactly as the reference's
// Iterator::sum, and sums the centred squares (x - mean) * (x - mean) left
// to right (the reference's `var += c * c`, two roundings) -- one warp
// instruction advances RPC rows' ordered sums at once.  All warps then
// normalize and write the rows and their quantized copies coalesced.  The
// staging and normalizing loops have compile-time trip counts, so each
// thread's loads are all in flight at once.
constexpr int kLnThreads = 128;

template <int VPL, int RPC>
__device__ __forceinline__ void ln_rows(float* tile, int row0, int nrows,
                                        const float* __restrict__ gamma,
                                        const float* __restrict__ beta, float* __restrict__ out,
                                        const QuantOut& q, uint32_t* status) {
  constexpr int d = VPL * 128;
  constexpr int ld = d + 4;
  __shared__ float s_mean[RPC], s_inv[RPC];
  __syncthreads();
  if (threadIdx.x < RPC) {
    const int i = threadIdx.x;
    const float* row = tile + i * ld;
    const float fd = (float)d;
    float sum = 0.0f;
#pragma unroll 8
    for (int j = 0; j < d; j += 4) {
      const float4 v = *reinterpret_cast<const float4*>(row + j);
      sum = sum + v.x;
      sum = sum + v.y;
      sum = sum + v.z;
      sum = sum + v.w;
    }
    const float mean = sum / fd;
    float var = 0.0f;
#pragma unroll 8
    for (int j = 0; j < d; j += 4) {
      const float4 v = *reinterpret_cast<const float4*>(row + j);
      const float c0 = v.x - mean, c1 = v.y - mean, c2 = v.z - mean, c3 = v.w - mean;
      var = var + c0 * c0;
      var = var + c1 * c1;
      var = var + c2 * c2;
      var = var + c3 * c3;
    }
    var = var / fd;
    s_mean[i] = mean;
    s_inv[i] = 1.0f / sqrtf(var + kLnEps);
  }
  __syncthreads();
  constexpr int kVec = d / 4;
#pragma unroll
  for (int it = 0; it < RPC * kVec / kLnThreads; ++it) {
    const int idx = threadIdx.x + it * kLnThreads;
    const int rr = idx / kVec, c = (idx - rr * kVec) * 4;
    if (rr >= nrows) break;
    const float4 t = *reinterpret_cast<const float4*>(tile + rr * ld + c);
    const float mean = s_mean[rr], inv = s_inv[rr];
    const float4 g = *reinterpret_cast<const float4*>(gamma + c);
    const float4 b = *reinterpret_cast<const float4*>(beta + c);
    float4 v;
    v.x = (t.x - mean) * inv * g.x + b.x;
    v.y = (t.y - mean) * inv * g.y + b.y;
    v.z = (t.z - mean) * inv * g.z + b.z;
    v.w = (t.w - mean) * inv * g.w + b.w;
    const long long elem = (long long)(row0 + rr) * d + c;
    *reinterpret_cast<float4*>(out + elem) = v;
    store_quant4(q, elem, v.x, v.y, v.z, v.w, status);
  }
}

template <int VPL, int RPC>
__global__ void __launch_bounds__(kLnThreads) residual_ln_kernel(
    const float* __restrict__ a, int lda, const float* __restrict__ r, int ldr,
    const float* __restrict__ gamma, const float* __restrict__ beta, int cap,
    const int32_t* __restrict__ rows_dev, float* __restrict__ out, const __grid_constant__ QuantOut q,
    uint32_t* status) {
  constexpr int d = VPL * 128;
  constexpr int ld = d + 4, kVec = d / 4;
  extern __shared__ __align__(16) float tile[];  // [RPC][d + 4]
  pdl_enter();
  const int rows = launch_rows(rows_dev, cap);
  const int row0 = blockIdx.x * RPC;
  const int nrows = min(RPC, rows - row0);
  if (nrows <= 0) return;
#pragma unroll
  for (int it = 0; it < RPC * kVec / kLnThreads; ++it) {
    const int idx = threadIdx.x + it * kLnThreads;
    const int rr = idx / kVec, c = (idx - rr * kVec) * 4;
    if (rr >= nrows) break;
    const float4 x = *reinterpret_cast<const float4*>(a + (size_t)(row0 + rr) * lda + c);
    const float4 y = *reinterpret_cast<const float4*>(r + (size_t)(row0 + rr) * ldr + c);
    *reinterpret_cast<float4*>(tile + rr * ld + c) = make_float4(x.x + y.x, x.y + y.y, x.z + y.z, x.w + y.w);
  }
  ln_rows<VPL, RPC>(tile, row0, nrows, gamma, beta, out, q, status);
}

// tensor.rs:184-218: gate and state update per element, then the LayerNorm
// of ReLU(state) + residual as above.
template <int VPL, int RPC>
__global__ void __launch_bounds__(kLnThreads) ssru_kernel(
    const float* __restrict__ cf, int ld_cf, int fcol, float* __restrict__ state,
    const int32_t* __restrict__ row_slot, const float* __restrict__ residual,
    const float* __restrict__ gamma, const float* __restrict__ beta, int cap,
    const int32_t* __restrict__ rows_dev, float* __restrict__ out, const __grid_constant__ QuantOut q,
    uint32_t* status) {
  constexpr int d = VPL * 128;
  constexpr int ld = d + 4, kVec = d / 4;
  extern __shared__ __align__(16) float tile[];
  pdl_enter();
  const int rows = launch_rows(rows_dev, cap);
  const int row0 = blockIdx.x * RPC;
  const int nrows = min(RPC, rows - row0);
  if (nrows <= 0) return;
#pragma unroll
  for (int it = 0; it < RPC * kVec / kLnThreads; ++it) {
    const int idx = threadIdx.x + it * kLnThreads;
    const int rr = idx / kVec, c = (idx - rr * kVec) * 4;
    if (rr >= nrows) break;
    const int row = row0 + rr;
    const float4 cv = *reinterpret_cast<const float4*>(cf + (size_t)row * ld_cf + c);
    const float4 fv = *reinterpret_cast<const float4*>(cf + (size_t)row * ld_cf + fcol + c);
    float* st = state + (size_t)row_slot[row] * d + c;
    const float4 sv = *reinterpret_cast<const float4*>(st);
    const float4 rv = *reinterpret_cast<const float4*>(residual + (size_t)row * d + c);
    const float cc[4] = {cv.x, cv.y, cv.z, cv.w}, ff[4] = {fv.x, fv.y, fv.z, fv.w};
    const float ss[4] = {sv.x, sv.y, sv.z, sv.w}, rs[4] = {rv.x, rv.y, rv.z, rv.w};
    float nx[4], o[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const float gate = 1.0f / (1.0f + exp_f32(-ff[u]));
      nx[u] = gate * ss[u] + (1.0f - gate) * cc[u];
      o[u] = fmaxf(nx[u], 0.0f) + rs[u];
    }
    *reinterpret_cast<float4*>(st) = make_float4(nx[0], nx[1], nx[2], nx[3]);
    *reinterpret_cast<float4*>(tile + rr * ld + c) = make_float4(o[0], o[1], o[2], o[3]);
  }
  ln_rows<VPL, RPC>(tile, row0, nrows, gamma, beta, out, q, status);
}

// Warp-per-row variant for small launches (decode steps): each warp owns one
// row end to end, so rows proceed without CTA-wide barriers.  The lanes load
// the row with coalesced 128-bit accesses (lane l holds float4 chunks l,
// l + 32, ...), form the pre-norm values and write them to a per-warp
// shared-memory row; lane 0 sums the row left to right, every lane forms its
// centred squares (x - mean) * (x - mean), and lane 0 sums those left to
// right.
constexpr int kLnWarps = 4;

// VPL = float4 chunks per lane = d / 128.
template <int VPL>
__device__ __forceinline__ float serial_sum(const float* row) {
  constexpr int kVec = VPL * 32;  // float4 per row
  const float4* r4 = reinterpret_cast<const float4*>(row);
  float sum = 0.0f;
#pragma unroll 4
  for (int i = 0; i < kVec; i += 8) {
    float4 v[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) v[u] = r4[i + u];
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      sum = sum + v[u].x;
      sum = sum + v[u].y;
      sum = sum + v[u].z;
      sum = sum + v[u].w;
    }
  }
  return sum;
}

template <int VPL>
__device__ __forceinline__ void load_lane_chunks(const float* __restrict__ v, float4 (&out)[VPL]) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int k = 0; k < VPL; ++k) out[k] = *reinterpret_cast<const float4*>(v + 4 * (lane + 32 * k));
}

// x[k] (this lane's chunks, columns 4 * (lane + 32 k)) hold the pre-norm row;
// row is the warp's shared-memory row buffer.  Writes out and the quantized
// copies of global row `grow` when `store` (warp-uniform) is set.
// gamma / beta: this lane's chunks of the LayerNorm scale and bias, loaded
// by the caller at kernel entry (they are weights: their loads, often from
// DRAM because the KV-cache traffic evicts them, overlap the row's).
template <int VPL>
__device__ __forceinline__ void ln_row(float4 (&x)[VPL], float* row, int grow,
                                       const float4 (&gamma)[VPL], const float4 (&beta)[VPL],
                                       float* __restrict__ out, const QuantOut& q, uint32_t* status,
                                       bool store = true) {
  constexpr int d = VPL * 128;
  const int lane = threadIdx.x & 31;
  float4* r4 = reinterpret_cast<float4*>(row);
#pragma unroll
  for (int k = 0; k < VPL; ++k) r4[lane + 32 * k] = x[k];
  __syncwarp();
  const float fd = (float)d;
  float mean = 0.0f;
  if (lane == 0) mean = serial_sum<VPL>(row) / fd;
  mean = __shfl_sync(0xffffffffu, mean, 0);
  float4 c[VPL];
#pragma unroll
  for (int k = 0; k < VPL; ++k) {
    c[k] = make_float4(x[k].x - mean, x[k].y - mean, x[k].z - mean, x[k].w - mean);
  }
  __syncwarp();  // lane 0 is done reading the row
#pragma unroll
  for (int k = 0; k < VPL; ++k)
    r4[lane + 32 * k] = make_float4(c[k].x * c[k].x, c[k].y * c[k].y, c[k].z * c[k].z, c[k].w * c[k].w);
  __syncwarp();
  float inv = 0.0f;
  if (lane == 0) {
    const float var = serial_sum<VPL>(row) / fd;
    inv = 1.0f / sqrtf(var + kLnEps);
  }
  inv = __shfl_sync(0xffffffffu, inv, 0);
#pragma unroll
  for (int k = 0; k < VPL; ++k) {
    const int col = 4 * (lane + 32 * k);
    const float4 g = gamma[k];
    const float4 b = beta[k];
    float4 v;
    v.x = c[k].x * inv * g.x + b.x;
    v.y = c[k].y * inv * g.y + b.y;
    v.z = c[k].z * inv * g.z + b.z;
    v.w = c[k].w * inv * g.w + b.w;
    if (store) {
      const long long elem = (long long)grow * d + col;
      *reinterpret_cast<float4*>(out + elem) = v;
      store_quant4(q, elem, v.x, v.y, v.z, v.w, status);
    }
  }
}

template <int VPL>
__global__ void __launch_bounds__(kLnWarps * 32) residual_ln_warp_kernel(
    const float* __restrict__ a, int lda, const float* __restrict__ r, int ldr,
    const float* __restrict__ gamma, const float* __restrict__ beta, int cap,
    const int32_t* __restrict__ rows_dev, float* __restrict__ out, const __grid_constant__ QuantOut q,
    uint32_t* status) {
  constexpr int d = VPL * 128;
  __shared__ __align__(16) float rows_s[kLnWarps][d];
  float4 gl[VPL], bl[VPL];
  load_lane_chunks<VPL>(gamma, gl);
  load_lane_chunks<VPL>(beta, bl);
  pdl_enter();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row = blockIdx.x * kLnWarps + warp;
  if (row >= cap) return;
  // The row is loaded together with the device row count, so the two loads'
  // latencies overlap: a row past the count (inside the buffers' cap rows)
  // is normalized like the others and not stored.
  const int rows = launch_rows(rows_dev, cap);
  float4 x[VPL];
#pragma unroll
  for (int k = 0; k < VPL; ++k) {
    const int col = 4 * (lane + 32 * k);
    const float4 u = *reinterpret_cast<const float4*>(a + (size_t)row * lda + col);
    const float4 w = *reinterpret_cast<const float4*>(r + (size_t)row * ldr + col);
    x[k] = make_float4(u.x + w.x, u.y + w.y, u.z + w.z, u.w + w.w);
  }
  ln_row<VPL>(x, rows_s[warp], row, gl, bl, out, q, status, row < rows);
}

// SSRU (tensor.rs:184-218) with the warp-per-row LayerNorm above.
template <int VPL>
__global__ void __launch_bounds__(kLnWarps * 32) ssru_warp_kernel(
    const float* __restrict__ cf, int ld_cf, int fcol, float* __restrict__ state,
    const int32_t* __restrict__ row_slot, const float* __restrict__ residual,
    const float* __restrict__ gamma, const float* __restrict__ beta, int cap,
    const int32_t* __restrict__ rows_dev, float* __restrict__ out, const __grid_constant__ QuantOut q,
    uint32_t* status) {
  constexpr int d = VPL * 128;
  __shared__ __align__(16) float rows_s[kLnWarps][d];
  float4 gl[VPL], bl[VPL];
  load_lane_chunks<VPL>(gamma, gl);
  load_lane_chunks<VPL>(beta, bl);
  pdl_enter();
  const int rows = launch_rows(rows_dev, cap);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row = blockIdx.x * kLnWarps + warp;
  if (row >= rows) return;
  const float* cand = cf + (size_t)row * ld_cf;
  float* st = state + (size_t)row_slot[row] * d;
  float4 x[VPL];
#pragma unroll
  for (int k = 0; k < VPL; ++k) {
    const int col = 4 * (lane + 32 * k);
    const float4 cv = *reinterpret_cast<const float4*>(cand + col);
    const float4 fv = *reinterpret_cast<const float4*>(cand + fcol + col);
    const float4 sv = *reinterpret_cast<const float4*>(st + col);
    const float4 rv = *reinterpret_cast<const float4*>(residual + (size_t)row * d + col);
    const float cc[4] = {cv.x, cv.y, cv.z, cv.w}, ff[4] = {fv.x, fv.y, fv.z, fv.w};
    const float ss[4] = {sv.x, sv.y, sv.z, sv.w}, rr[4] = {rv.x, rv.y, rv.z, rv.w};
    float nx[4], o[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const float gate = 1.0f / (1.0f + exp_f32(-ff[u]));
      nx[u] = gate * ss[u] + (1.0f - gate) * cc[u];
      o[u] = fmaxf(nx[u], 0.0f) + rr[u];
    }
    *reinterpret_cast<float4*>(st + col) = make_float4(nx[0], nx[1], nx[2], nx[3]);
    x[k] = make_float4(o[0], o[1], o[2], o[3]);
  }
  ln_row<VPL>(x, rows_s[warp], row, gl, bl, out, q, status);
}

// ---- attention (attention_into, tensor.rs:251-318) ------------------------------
// Encoder: one CTA of 8 warps per (sequence, head, 32-query chunk); each
// warp owns 4 queries and advances them together, so every dependent chain
// below has 4 (scores) or 8 (outputs) independent neighbours to overlap with.
// K and V of the head are staged in shared memory (K rows padded to HD + 4
// floats: 16-byte aligned with an odd number of 16-byte chunks, so the lanes'
// 128-bit reads of different keys hit distinct banks).  Per query the
// operation order is the reference's: in-order dot products, max, exp, a
// left-to-right sum (lane qq sums query qq), scaling, and a left-to-right
// weighted sum of V per output dimension.  The host launches one grid per
// length bucket so shared memory follows the bucket's longest sequence.
constexpr int kEncWarps = 8;
constexpr int kEncQpw = 4;  // queries per warp, advanced in two pairs

// Asynchronous global -> shared copies (cp.async): 16 bytes (both addresses
// 16-byte aligned) or 4 bytes; cp_async_wait_all waits for this thread's.
__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(smem)), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async4(void* smem, const void* gmem) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_u32(smem)), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

// Packed f32x2 arithmetic (sm_100): each half is one IEEE f32 operation
// rounded to nearest, exactly as the scalar instruction, so pairing two
// independent sums changes no result while halving the issued instructions.
__device__ __forceinline__ unsigned long long f2_pack(float lo, float hi) {
  unsigned long long r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ float2 f2_unpack(unsigned long long v) {
  float lo, hi;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
  return make_float2(lo, hi);
}
// acc + a * b with two roundings per half (the reference's `acc += a * b`;
// never a fused multiply-add).  ptxas contracts mul.rn.f32x2 followed by
// add.rn.f32x2 into one fused f32x2 multiply-add despite the explicit
// rounding modifiers (and --fmad=false), so the sum is issued as
// fma(prod, ones, acc): prod * 1 is exact, leaving the single rounding of
// prod + acc.  `ones` must be a runtime value (a kernel argument) so that
// the multiply by 1 cannot be folded back into an add.
__device__ __forceinline__ unsigned long long f2_mul_add(unsigned long long acc, unsigned long long a,
                                                         unsigned long long b,
                                                         unsigned long long ones) {
  unsigned long long prod, r;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(prod) : "l"(a), "l"(b));
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(prod), "l"(ones), "l"(acc));
  return r;
}

template <int HD>
__global__ void __launch_bounds__(kEncWarps * 32) attn_encoder_kernel(
    const float* __restrict__ qkv, const int32_t* __restrict__ cu,
    const int32_t* __restrict__ seq_ids, int d, int max_len, int8_t* __restrict__ out_q,
    float alpha, float one, uint32_t* status) {
  pdl_enter();
  extern __shared__ __align__(16) float sm[];
  const int b = seq_ids[blockIdx.x];
  const int h = blockIdx.y;
  const int start = cu[b];
  const int len = cu[b + 1] - start;
  if (len <= 0 || len > max_len) {
    if (threadIdx.x == 0 && len > max_len) flag_status(status, kStatusBadIndex);
    return;
  }
  const int q0 = blockIdx.z * 32;
  if (q0 >= len) return;
  const int ld = 3 * d;
  constexpr int KLD = HD + 4;
  float* ks = sm;                                          // [max_len][HD + 4]
  float* vs = ks + (size_t)max_len * KLD;                   // [max_len][HD]
  float* qs = vs + (size_t)max_len * HD;                   // [warps][2 pairs][HD][2]
  float* ps = qs + kEncWarps * kEncQpw * HD;               // [warps][2 pairs][max_len][2]
  // K, V and the queries are staged with asynchronous copies (no register
  // round trip), so every thread has all of its copies in flight at once.
  constexpr int kVec = HD / 4;
  for (int idx = threadIdx.x; idx < len * kVec; idx += blockDim.x) {
    const int j = idx / kVec, i = (idx % kVec) * 4;
    const float* row = qkv + (size_t)(start + j) * ld + h * HD + i;
    cp_async16(ks + j * KLD + i, row + d);
    cp_async16(vs + j * HD + i, row + 2 * d);
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int qb = q0 + warp * kEncQpw;                      // this warp's first query
  const int nq = max(0, min(kEncQpw, len - qb));
  // queries 2p and 2p + 1 interleaved: qw[p][i] = (q_2p[i], q_2p+1[i])
  float* qw = qs + warp * kEncQpw * HD;
  float* pw = ps + warp * kEncQpw * max_len;
  for (int idx = lane; idx < kEncQpw * HD; idx += 32) {
    const int qq = idx / HD, i = idx % HD;
    float* dst = qw + (qq >> 1) * 2 * HD + 2 * i + (qq & 1);
    if (qq < nq)
      cp_async4(dst, qkv + (size_t)(start + qb + qq) * ld + h * HD + i);
    else
      *dst = 0.0f;
  }
  cp_async_wait_all();
  __syncthreads();
  if (nq == 0) return;
  auto pidx = [&](int qq, int j) { return (qq >> 1) * 2 * max_len + 2 * j + (qq & 1); };
  const float scale = 1.0f / sqrtf((float)HD);
  const unsigned long long ones = f2_pack(one, one);
  float mx[kEncQpw];
#pragma unroll
  for (int qq = 0; qq < kEncQpw; ++qq) mx[qq] = -INFINITY;
  for (int j = lane; j < len; j += 32) {
    const float* kr = ks + j * KLD;
    unsigned long long dot[2] = {0ull, 0ull};  // (+0, +0)
#pragma unroll
    for (int i = 0; i < HD; i += 4) {
      const float4 k4 = *reinterpret_cast<const float4*>(kr + i);
      const unsigned long long kx = f2_pack(k4.x, k4.x), ky = f2_pack(k4.y, k4.y),
                               kz = f2_pack(k4.z, k4.z), kw = f2_pack(k4.w, k4.w);
#pragma unroll
      for (int p = 0; p < 2; ++p) {
        const float4 qa = *reinterpret_cast<const float4*>(qw + p * 2 * HD + 2 * i);
        const float4 qc = *reinterpret_cast<const float4*>(qw + p * 2 * HD + 2 * i + 4);
        unsigned long long t = dot[p];
        t = f2_mul_add(t, f2_pack(qa.x, qa.y), kx, ones);
        t = f2_mul_add(t, f2_pack(qa.z, qa.w), ky, ones);
        t = f2_mul_add(t, f2_pack(qc.x, qc.y), kz, ones);
        t = f2_mul_add(t, f2_pack(qc.z, qc.w), kw, ones);
        dot[p] = t;
      }
    }
#pragma unroll
    for (int p = 0; p < 2; ++p) {
      const float2 dd = f2_unpack(dot[p]);
      const float s0 = dd.x * scale, s1 = dd.y * scale;
      *reinterpret_cast<float2*>(pw + pidx(2 * p, j)) = make_float2(s0, s1);
      mx[2 * p] = fmaxf(mx[2 * p], s0);
      mx[2 * p + 1] = fmaxf(mx[2 * p + 1], s1);
    }
  }
#pragma unroll
  for (int qq = 0; qq < kEncQpw; ++qq)
    for (int o = 16; o > 0; o >>= 1) mx[qq] = fmaxf(mx[qq], __shfl_xor_sync(0xffffffffu, mx[qq], o));
  for (int j = lane; j < len; j += 32) {
#pragma unroll
    for (int qq = 0; qq < kEncQpw; ++qq) pw[pidx(qq, j)] = exp_f32(pw[pidx(qq, j)] - mx[qq]);
  }
  __syncwarp();
  float inv_mine = 0.0f;
  if (lane < kEncQpw) {  // lane qq sums query qq's exponentials in key order
    float sum = 0.0f;
#pragma unroll 8
    for (int j = 0; j < len; ++j) sum = sum + pw[pidx(lane, j)];
    inv_mine = 1.0f / sum;
  }
  float inv[kEncQpw];
#pragma unroll
  for (int qq = 0; qq < kEncQpw; ++qq) inv[qq] = __shfl_sync(0xffffffffu, inv_mine, qq);
  for (int j = lane; j < len; j += 32) {
#pragma unroll
    for (int qq = 0; qq < kEncQpw; ++qq) pw[pidx(qq, j)] = pw[pidx(qq, j)] * inv[qq];
  }
  __syncwarp();
  // lane owns output dims 2*lane and 2*lane + 1 of each of the 4 queries;
  // acc[p][c] holds dim c of queries 2p and 2p + 1
  const bool active = 2 * lane < HD;
  unsigned long long acc[2][2] = {{0ull, 0ull}, {0ull, 0ull}};
#pragma unroll 4
  for (int j = 0; j < len; ++j) {
    const float2 v2 = active ? *reinterpret_cast<const float2*>(vs + j * HD + 2 * lane)
                             : make_float2(0.f, 0.f);
    const unsigned long long vx = f2_pack(v2.x, v2.x), vy = f2_pack(v2.y, v2.y);
#pragma unroll
    for (int p = 0; p < 2; ++p) {
      const unsigned long long pp = *reinterpret_cast<const unsigned long long*>(pw + pidx(2 * p, j));
      acc[p][0] = f2_mul_add(acc[p][0], pp, vx, ones);
      acc[p][1] = f2_mul_add(acc[p][1], pp, vy, ones);
    }
  }
  if (active) {
#pragma unroll
    for (int p = 0; p < 2; ++p) {
      const float2 c0 = f2_unpack(acc[p][0]), c1 = f2_unpack(acc[p][1]);
      const float dims[2][2] = {{c0.x, c1.x}, {c0.y, c1.y}};  // [query in pair][dim]
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        const int qq = 2 * p + u;
        if (qq < nq) {
          int8_t* o = out_q + (size_t)(start + qb + qq) * d + h * HD + 2 * lane;
          const uint16_t w2 = (uint16_t)(uint8_t)quantize_one(dims[u][0], alpha, status) |
                              ((uint16_t)(uint8_t)quantize_one(dims[u][1], alpha, status) << 8);
          *reinterpret_cast<uint16_t*>(o) = w2;
        }
      }
    }
  }
}

// Decode: a persistent kernel over work items (active row, group of 4
// heads), taken in row_order (longest rows first) round-robin by the CTAs.
// Warp 4 is the producer: for every item it streams the group's
// slices of the cached keys, then of the values, into a 2-slot shared-memory
// ring, one chunk of 32 keys per slot, with one 3-D TMA copy per 8 cache
// rows (8 rows x 4 * HD floats of one page, through the pool's tensor maps;
// see encode_tmap_kv) completing on the slot's mbarrier; an item's last,
// partial group of keys is copied with a box of 4, 2 or 1 rows, so at most
// 3 rows past its last key are read.  The copies of the next chunks and
// items are in flight while warps 0..3 (one per head of the group) consume
// the current slot.  The 128-byte swizzle of the copies puts the 16-byte
// chunk c of key row r at chunk c ^ (r % 8) of its line, so the lanes'
// reads of different keys in the score loop fall on distinct banks.  Per
// head the operation order is the reference's: lane t scores
// key t with an in-order dot product, max, exp, a left-to-right sum by lane
// 0, scaling, and a left-to-right weighted sum of V per output dim (lane i
// owns dims 2i and 2i + 1).  Every mbarrier wait is bounded; on a timeout
// the kernel records kStatusWaitTimeout and stops, after waiting (bounded)
// for the copies it issued.
constexpr int kDecGroup = 4;    // heads per item
constexpr int kDecChunk = 32;   // keys per ring slot
constexpr int kDecSlots = 2;    // ring depth (three CTAs per SM)
constexpr int kDecThreads = (kDecGroup + 1) * 32;

__device__ __forceinline__ void bulk_copy_g2s(void* smem_dst, const void* gmem_src, uint32_t bytes,
                                              uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(smem_dst)),
      "l"(gmem_src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void mbar_arrive_cta(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// Row of work item `item` (items are (row in row_order, head group)).
__device__ __forceinline__ int item_row(int item, int groups, const int32_t* __restrict__ row_order) {
  const int ro = item / groups;
  return row_order ? row_order[ro] : ro;
}

// Shared-memory float offset of float f (0 <= f < W) of key t of a chunk
// staged as 8-row boxes [W / 32 column blocks][8 rows][32 floats], 128-byte
// swizzled, box_floats apart.
__device__ __forceinline__ int swz(int t, int f, int box_floats) {
  const int r = t & 7, cb = f >> 5, c = (f & 31) >> 2;
  return (t >> 3) * box_floats + cb * 256 + r * 32 + ((c ^ r) << 2) + (f & 3);
}

// A slot's last group of keys may come in a box of R = 4, 2 or 1 rows
// ([column block][R rows][32 floats], line l = block * R + row, chunk c at
// c ^ (l & 7)); keys of earlier groups are in 8-row boxes.  last_box: index
// of the slot's last box; tail_rows: its R.
__device__ __forceinline__ int swz_tail(int t, int f, int box_floats, int last_box, int tail_rows) {
  const int b = t >> 3, r = t & 7, cb = f >> 5, c = (f & 31) >> 2;
  const int rows = b == last_box ? tail_rows : 8;
  const int line = cb * rows + r;
  return b * box_floats + line * 32 + ((c ^ (line & 7)) << 2) + (f & 3);
}

// Rows of the box that holds the last n - 8 * ((n - 1) / 8) keys of a slot.
__device__ __forceinline__ int tail_box_rows(int n) {
  const int nr = n - 8 * ((n - 1) >> 3);
  return nr <= 1 ? 1 : (nr <= 2 ? 2 : (nr <= 4 ? 4 : 8));
}

// Three CTAs share an SM (15 warps: four on some sub-partition, whose 16K
// registers then allow 128 per thread), so twelve consumer warps per SM
// overlap their dependent chains.
template <int HD, int PT>
__global__ void __maxnreg__(128) attn_decode_kernel(
    const float* __restrict__ q, int ldq, const int32_t* __restrict__ rows_dev, int cap,
    const int32_t* __restrict__ row_slot,
    const int32_t* __restrict__ row_order, const int32_t* __restrict__ slot_len, int len_add,
    const int32_t* __restrict__ page_table, int pages_per_slot,
    const __grid_constant__ KvBoxMaps k_maps, const __grid_constant__ KvBoxMaps v_maps, int d,
    int heads, int8_t* __restrict__ out_q, float alpha, uint32_t* status) {
  constexpr int W = kDecGroup * HD;
  constexpr int kBoxFloats = 8 * W;                         // 8 rows (a multiple of 1 KB)
  constexpr int kSlotFloats = (kDecChunk / 8) * kBoxFloats + 256;  // boxes, then q (1 KB)
  extern __shared__ uint8_t dsm_raw[];
  float* dsm = reinterpret_cast<float*>((reinterpret_cast<uintptr_t>(dsm_raw) + 1023) & ~uintptr_t(1023));
  __shared__ __align__(8) uint64_t full_bar[kDecSlots], empty_bar[kDecSlots];
  float* ps = dsm + kDecSlots * kSlotFloats;        // [4][kMaxSeq] scores
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < kDecSlots; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], kDecGroup);
    }
    fence_barrier_init();
    for (int i = 0; i < 4; ++i) {
      tma_prefetch_desc(&k_maps.box[i]);
      tma_prefetch_desc(&v_maps.box[i]);
    }
  }
  __syncthreads();
  pdl_enter();
  const int groups = heads / kDecGroup;
  const int items = launch_rows(rows_dev, cap) * groups;
  const int limit = min(kMaxSeq, pages_per_slot * PT);
  if (warp == kDecGroup) {
    // ---- producer warp ------------------------------------------------------
    // All 32 lanes walk the items: an item's page-table row (at most 32
    // pages: 256 keys of 8-token pages) is fetched by one lane-parallel load,
    // and the next item's row index is loaded one item ahead, so an item
    // costs two dependent global round trips (slot, then its length and
    // pages) instead of one per copied box.  Lane 0 issues the copies.
    int k = 0;
    bool ok = true;
    const uint64_t stream_once = l2_policy_evict_first();  // KV pages: read once per step
    int item = blockIdx.x;
    int r_next = item < items ? item_row(item, groups, row_order) : 0;
    for (; item < items && ok; item += gridDim.x) {
      const int r = r_next;
      const int g = item % groups;
      if (item + (int)gridDim.x < items) r_next = item_row(item + gridDim.x, groups, row_order);
      const int slot = row_slot[r];
      const int len = slot_len[slot] + len_add;
      const int page = lane < pages_per_slot ? page_table[(size_t)slot * pages_per_slot + lane] : 0;
      if (len <= 0 || len > limit) {
        if (lane == 0) flag_status(status, kStatusBadIndex);
        continue;
      }
      for (int pass = 0; pass < 2 && ok; ++pass) {
        const KvBoxMaps* maps = pass == 0 ? &k_maps : &v_maps;
        for (int c0 = 0; c0 < len; c0 += kDecChunk, ++k) {
          const int n = min(kDecChunk, len - c0);
          const int nb = (n + 7) / 8;  // boxes: 8 rows, the last one 8, 4, 2 or 1
          const int tail_rows = tail_box_rows(n);
          const int sl = k % kDecSlots;
          bool free_slot = true;
          if (lane == 0) free_slot = mbar_wait(&empty_bar[sl], ((k / kDecSlots) & 1) ^ 1, status);
          if (!(ok = __shfl_sync(0xffffffffu, free_slot, 0))) break;
          int rows[kDecChunk / 8];  // first cache row of each box (boxes never straddle pages)
#pragma unroll
          for (int b = 0; b < kDecChunk / 8; ++b) {
            const int j = c0 + 8 * b;
            rows[b] = __shfl_sync(0xffffffffu, page, min(j / PT, 31)) * PT + j % PT;
          }
          if (lane == 0) {
            float* dst = dsm + sl * kSlotFloats;
            const uint32_t box_bytes = kBoxFloats * 4, q_bytes = W * 4;
            const uint32_t tail_bytes = (uint32_t)tail_rows * W * 4;
            mbar_arrive_expect_tx(&full_bar[sl], (nb - 1) * box_bytes + tail_bytes + (pass == 0 ? q_bytes : 0));
            if (pass == 0)
              bulk_copy_g2s(dst + (kDecChunk / 8) * kBoxFloats, q + (size_t)r * ldq + g * W, q_bytes,
                            &full_bar[sl]);
            const CUtensorMap* tail_map =
                &maps->box[tail_rows == 8 ? 0 : (tail_rows == 4 ? 1 : (tail_rows == 2 ? 2 : 3))];
            for (int b = 0; b < nb; ++b)
              tma_load_3d_hint(dst + b * kBoxFloats, b == nb - 1 ? tail_map : &maps->box[0], 0, rows[b],
                               g * (W / 32), &full_bar[sl], stream_once);
          }
        }
      }
    }
    // every issued copy lands before the CTA can exit: wait (bounded) for
    // the last fill of each slot
    if (lane == 0)
      for (int kk = max(0, k - kDecSlots); kk < k; ++kk)
        mbar_wait(&full_bar[kk % kDecSlots], (kk / kDecSlots) & 1, status);
    return;
  }
  // ---- consumers: warp h = head h of the item's group -------------------------
  const int h = warp;
  float* ph = ps + h * kMaxSeq;
  const float scale = 1.0f / sqrtf((float)HD);
  const bool active = 2 * lane < HD;
  int k = 0;
  // The next item's row, slot and key count are loaded during this item
  // (one dependent load after each phase), off the critical path.
  int r_next = (int)blockIdx.x < items ? item_row(blockIdx.x, groups, row_order) : 0;
  int len_next = (int)blockIdx.x < items ? slot_len[row_slot[r_next]] + len_add : 0;
  for (int item = blockIdx.x; item < items; item += gridDim.x) {
    const int r = r_next;
    const int len = len_next;
    const int g = item % groups;
    const bool have_next = item + (int)gridDim.x < items;
    if (have_next) r_next = item_row(item + gridDim.x, groups, row_order);
    if (len <= 0 || len > limit) {  // the producer flags it
      if (have_next) len_next = slot_len[row_slot[r_next]] + len_add;
      continue;
    }
    float mx = -INFINITY;
    for (int c0 = 0; c0 < len; c0 += kDecChunk, ++k) {
      const int n = min(kDecChunk, len - c0);
      const int sl = k % kDecSlots;
      if (!__all_sync(0xffffffffu, mbar_wait(&full_bar[sl], (k / kDecSlots) & 1, status))) return;
      const float* base = dsm + sl * kSlotFloats;
      const int last_box = (n - 1) >> 3, tail_rows = tail_box_rows(n);
      if (lane < n) {
        const float* qh = base + (kDecChunk / 8) * kBoxFloats + h * HD;
        float dot = 0.0f;
#pragma unroll
        for (int i = 0; i < HD; i += 4) {
          const float4 k4 = *reinterpret_cast<const float4*>(
              base + swz_tail(lane, h * HD + i, kBoxFloats, last_box, tail_rows));
          const float4 q4 = *reinterpret_cast<const float4*>(qh + i);
          dot = dot + q4.x * k4.x;
          dot = dot + q4.y * k4.y;
          dot = dot + q4.z * k4.z;
          dot = dot + q4.w * k4.w;
        }
        const float sc = dot * scale;
        ph[c0 + lane] = sc;
        mx = fmaxf(mx, sc);
      }
      __syncwarp();
      if (lane == 0) mbar_arrive_cta(&empty_bar[sl]);
    }
    const int slot_next = have_next ? row_slot[r_next] : 0;
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    for (int j = lane; j < len; j += 32) ph[j] = exp_f32(ph[j] - mx);
    __syncwarp();
    float inv = 0.0f;
    if (lane == 0) {
      float sum = 0.0f;
#pragma unroll 8
      for (int j = 0; j < len; ++j) sum = sum + ph[j];
      inv = 1.0f / sum;
    }
    inv = __shfl_sync(0xffffffffu, inv, 0);
    for (int j = lane; j < len; j += 32) ph[j] = ph[j] * inv;
    __syncwarp();
    if (have_next) len_next = slot_len[slot_next] + len_add;
    float acc0 = 0.0f, acc1 = 0.0f;
    for (int c0 = 0; c0 < len; c0 += kDecChunk, ++k) {
      const int n = min(kDecChunk, len - c0);
      const int sl = k % kDecSlots;
      if (!__all_sync(0xffffffffu, mbar_wait(&full_bar[sl], (k / kDecSlots) & 1, status))) return;
      if (active) {
        const float* base = dsm + sl * kSlotFloats;
        const int f = h * HD + 2 * lane;
        const int last_box = (n - 1) >> 3, tail_rows = tail_box_rows(n);
#pragma unroll 4
        for (int t = 0; t < n; ++t) {
          const float2 v2 = *reinterpret_cast<const float2*>(
              base + swz_tail(t, f, kBoxFloats, last_box, tail_rows));
          const float p = ph[c0 + t];
          acc0 = acc0 + v2.x * p;
          acc1 = acc1 + v2.y * p;
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive_cta(&empty_bar[sl]);
    }
    if (active) {
      const uint16_t w2 = (uint16_t)(uint8_t)quantize_one(acc0, alpha, status) |
                          ((uint16_t)(uint8_t)quantize_one(acc1, alpha, status) << 8);
      *reinterpret_cast<uint16_t*>(out_q + (size_t)r * d + g * W + h * HD + 2 * lane) = w2;
    }
  }
}

// ---- activation quantization (q8_gemm.rs:569-590) ------------------------------
__global__ void quantize_kernel(const float* __restrict__ x, long long n4, float alpha,
                                int8_t* __restrict__ out, uint32_t* status) {
  pdl_enter();
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n4) return;
  const float4 v = reinterpret_cast<const float4*>(x)[i];
  const uint32_t w = (uint32_t)(uint8_t)quantize_one(v.x, alpha, status) |
                     ((uint32_t)(uint8_t)quantize_one(v.y, alpha, status) << 8) |
                     ((uint32_t)(uint8_t)quantize_one(v.z, alpha, status) << 16) |
                     ((uint32_t)(uint8_t)quantize_one(v.w, alpha, status) << 24);
  reinterpret_cast<uint32_t*>(out)[i] = w;
}

// ---- token selection ----------------------------------------------------------
__global__ void finalize_kernel(int cap, const int32_t* __restrict__ rows_dev,
                                const int32_t* __restrict__ row_slot,
                                unsigned long long* __restrict__ best, int32_t* slot_prev,
                                int32_t* slot_step, const int32_t* __restrict__ slot_limit,
                                int32_t* step_tokens, uint8_t* done, uint32_t* status) {
  pdl_enter();
  const int r = blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= launch_rows(rows_dev, cap)) return;
  const int slot = row_slot[r];
  const unsigned long long key = best[r];
  best[r] = 0ull;
  int token = 0;
  if (key == 0ull) {
    flag_status(status, kStatusBadIndex);  // no candidate scored
  } else {
    token = static_cast<int>(0xFFFFFFFFu - static_cast<uint32_t>(key & 0xFFFFFFFFull));
  }
  const int t = slot_step[slot];
  slot_step[slot] = t + 1;
  slot_prev[slot] = token;
  step_tokens[r] = token;
  done[r] = (token == 0 || t + 1 >= slot_limit[slot]) ? 1 : 0;
}

// ---- decode-step row table (the batcher's per-step retire and admit) ------------
// One CTA builds the table a decode step runs over, on the device, so the
// host can enqueue the next step before it has read the previous one's
// tokens.  The table (see launch_step_rows) holds the previous step's rows;
// their finished flags are that step's `done`.  The survivors keep their
// order (a stable compaction: block-wide scan over chunks of 1,024 rows,
// staged in `scratch`), the admitted slots listed in the join block are
// appended, and the two attention orders -- most keys first, self keys =
// step + 1, cross keys = source length -- are rebuilt by counting sort.
// The host mirrors the same compaction, so row r of the table is its row r.
constexpr int kRowsThreads = 1024;

__device__ __forceinline__ int block_exclusive_scan(int v, int* warp_sums, int* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) warp_sums[warp] = x;
  __syncthreads();
  if (warp == 0) {
    const int w = warp_sums[lane];
    int s = w;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, s, o);
      if (lane >= o) s += y;
    }
    warp_sums[lane] = s - w;
    if (lane == 31) *total = s;
  }
  __syncthreads();
  return warp_sums[warp] + x - v;
}

__device__ __forceinline__ void row_keys(const int32_t* slot_step, const int32_t* slot_src, int s, int* bs,
                                         int* bc) {
  const int ks = min(kMaxSeq + 1, max(0, slot_step[s] + 1));
  const int kc = min(kMaxSeq + 1, max(0, slot_src[s]));
  *bs = kMaxSeq + 1 - ks;  // bin 0 = most keys
  *bc = kMaxSeq + 1 - kc;
}

__global__ void __launch_bounds__(kRowsThreads) step_rows_kernel(
    int32_t* __restrict__ table, int rmax, const uint8_t* __restrict__ done,
    const int32_t* __restrict__ join, const int32_t* __restrict__ slot_step,
    const int32_t* __restrict__ slot_src, int32_t* __restrict__ scratch, uint32_t* status) {
  constexpr int kBins = kMaxSeq + 2;
  __shared__ int warp_sums[32];
  __shared__ int s_total;
  __shared__ int hist[2][kBins];
  pdl_enter();
  const int tid = threadIdx.x;
  int32_t* row_slot = table + 4;
  int32_t* ord_self = row_slot + rmax;
  int32_t* ord_cross = ord_self + rmax;
  const int r0 = min(max(table[0], 0), rmax);
  for (int i = tid; i < 2 * kBins; i += kRowsThreads) (&hist[0][0])[i] = 0;
  int base = 0;
  for (int c0 = 0; c0 < r0; c0 += kRowsThreads) {
    const int r = c0 + tid;
    const int keep = (r < r0 && done[r] == 0) ? 1 : 0;
    const int slot = keep ? row_slot[r] : 0;
    const int pos = base + block_exclusive_scan(keep, warp_sums, &s_total);
    if (keep) scratch[pos] = slot;
    base += s_total;
    __syncthreads();  // warp_sums and s_total are reused by the next chunk
  }
  int nj = join[0];
  if (nj < 0 || nj > rmax - base) {
    if (tid == 0) flag_status(status, kStatusBadIndex);
    nj = max(0, min(nj, rmax - base));
  }
  for (int i = tid; i < nj; i += kRowsThreads) scratch[base + i] = join[1 + i];
  const int r1 = base + nj;
  __syncthreads();
  for (int r = tid; r < r1; r += kRowsThreads) {
    int s = scratch[r];
    if (s < 0 || s >= rmax) {
      flag_status(status, kStatusBadIndex);
      s = 0;
      scratch[r] = 0;
    }
    int bs, bc;
    row_keys(slot_step, slot_src, s, &bs, &bc);
    atomicAdd(&hist[0][bs], 1);
    atomicAdd(&hist[1][bc], 1);
  }
  __syncthreads();
  if (tid < 64) {  // warp 0 scans the self histogram, warp 1 the cross one
    int* h = hist[tid >> 5];
    const int lane = tid & 31;
    constexpr int kPer = (kBins + 31) / 32;
    int local[kPer];
    int sum = 0;
#pragma unroll
    for (int i = 0; i < kPer; ++i) {
      const int b = lane * kPer + i;
      local[i] = sum;
      sum += b < kBins ? h[b] : 0;
    }
    int x = sum;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, x, o);
      if (lane >= o) x += y;
    }
#pragma unroll
    for (int i = 0; i < kPer; ++i) {
      const int b = lane * kPer + i;
      if (b < kBins) h[b] = x - sum + local[i];
    }
  }
  __syncthreads();
  for (int r = tid; r < r1; r += kRowsThreads) {
    const int s = scratch[r];
    int bs, bc;
    row_keys(slot_step, slot_src, s, &bs, &bc);
    ord_self[atomicAdd(&hist[0][bs], 1)] = r;
    ord_cross[atomicAdd(&hist[1][bc], 1)] = r;
    row_slot[r] = s;
  }
  if (tid == 0) table[0] = r1;
}

__global__ void init_slots_kernel(int n, const int32_t* slots, const int32_t* limits,
                                  const int32_t* force, const int32_t* src_len, int32_t* slot_prev,
                                  int32_t* slot_step, int32_t* slot_limit, int32_t* slot_force,
                                  int32_t* slot_src, float* ssru_state, int layers, int max_slots,
                                  int d, const int32_t* __restrict__ page_rows, int32_t* cross_pages,
                                  int32_t* self_pages, int pages_per_slot) {
  pdl_enter();
  const int i = blockIdx.x;
  if (i >= n) return;
  const int s = slots[i];
  // page-table rows of the admitted slot: [n][pages_per_slot] cross, then
  // [n][pages_per_slot] self
  for (int k = threadIdx.x; k < pages_per_slot; k += blockDim.x) {
    cross_pages[(size_t)s * pages_per_slot + k] = page_rows[(size_t)i * pages_per_slot + k];
    if (self_pages)
      self_pages[(size_t)s * pages_per_slot + k] =
          page_rows[((size_t)n + i) * pages_per_slot + k];
  }
  if (threadIdx.x == 0) {
    slot_prev[s] = -1;
    slot_step[s] = 0;
    slot_limit[s] = limits[i];
    slot_force[s] = force[i];
    slot_src[s] = src_len[i];
  }
  if (ssru_state)
    for (int l = 0; l < layers; ++l)
      for (int k = threadIdx.x; k < d; k += blockDim.x)
        ssru_state[((size_t)l * max_slots + s) * d + k] = 0.0f;
}

// ---- lexical shortlist candidates (shortlist.rs:150-198) ------------------
// One CTA per admitted request builds the slot's candidate bitmask in shared
// memory: ids below first_num, every target of every source token, minus
// UNK (1) and the byte/control fallbacks 7..38, then the first absent ids
// from 50 up until the count is a multiple of 8 -- the reference's set
// (which it then sorts; a bitmask is already in id order).
__global__ void shortlist_mask_kernel(int n, const int32_t* __restrict__ slots,
                                      const int32_t* __restrict__ tokens,
                                      const int32_t* __restrict__ cu,
                                      const int32_t* __restrict__ offsets,
                                      const int32_t* __restrict__ targets, int first_num, int vocab,
                                      int words, uint32_t* __restrict__ masks) {
  extern __shared__ uint32_t cm[];
  __shared__ int s_count;
  pdl_enter();
  const int b = blockIdx.x;
  if (b >= n) return;
  for (int w = threadIdx.x; w < words; w += blockDim.x) {
    const int lo = w * 32;
    cm[w] = first_num >= lo + 32 ? 0xFFFFFFFFu : (first_num > lo ? (1u << (first_num - lo)) - 1u : 0u);
  }
  if (threadIdx.x == 0) s_count = 0;
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nwarps = blockDim.x >> 5;
  for (int i = cu[b] + warp; i < cu[b + 1]; i += nwarps) {
    const int t = tokens[i];
    for (int j = offsets[t] + lane; j < offsets[t + 1]; j += 32) {
      const int id = targets[j];
      atomicOr(&cm[id >> 5], 1u << (id & 31));
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    if (vocab > 1) cm[0] &= ~2u;
    for (int id = 7; id < min(vocab, 39); ++id) cm[id >> 5] &= ~(1u << (id & 31));
  }
  __syncthreads();
  int c = 0;
  for (int w = threadIdx.x; w < words; w += blockDim.x) c += __popc(cm[w]);
  atomicAdd(&s_count, c);
  __syncthreads();
  if (threadIdx.x == 0) {
    int need = (8 - s_count % 8) % 8;
    for (int id = 50; id < vocab && need > 0; ++id) {
      const uint32_t bit = 1u << (id & 31);
      if (!(cm[id >> 5] & bit)) {
        cm[id >> 5] |= bit;
        --need;
      }
    }
  }
  __syncthreads();
  uint32_t* out = masks + (size_t)slots[b] * words;
  for (int w = threadIdx.x; w < words; w += blockDim.x) out[w] = cm[w];
}

__global__ void flag_status_kernel(uint32_t* status) {
  if (threadIdx.x == 0) flag_status(status, kStatusBadIndex);
}

inline void flag_status_host(uint32_t* status, cudaStream_t s) {
  flag_status_kernel<<<1, 32, 0, s>>>(status);
}

inline unsigned blocks_for(long long n, int threads) {
  return static_cast<unsigned>((n + threads - 1) / threads);
}

}  // namespace

void launch_embed_encoder(const int32_t* tokens, const int32_t* pos_idx, int n_tokens,
                          const int8_t* emb, float emb_mult, float emb_scale,
                          const float* positions, int d, float* x, const QuantOut& q,
                          uint32_t* status, cudaStream_t s) {
  if (n_tokens <= 0) return;
  const long long n = (long long)n_tokens * (d / 4);
  launch_pdl(embed_encoder_kernel, blocks_for(n, 256), 256, 0, s, tokens, pos_idx, n_tokens, emb,
             emb_mult, emb_scale, positions, d, x, q, status);
}

void launch_embed_decoder(int rows, const int32_t* rows_dev, const int32_t* row_slot,
                          const int32_t* slot_prev,
                          const int32_t* slot_step, const int32_t* slot_force, const int8_t* emb,
                          float emb_mult, float emb_scale, const float* positions, int d, float* x,
                          const QuantOut& q, uint8_t* eos_mask, const int32_t* self_pages,
                          int pages_per_slot, int page_tokens, int32_t* self_row_map,
                          uint32_t* status, cudaStream_t s) {
  if (rows <= 0) return;
  const long long n = (long long)rows * (d / 4);
  launch_pdl(embed_decoder_kernel, dim3(blocks_for(n, 256)), dim3(256), 0, s,
      rows, rows_dev, row_slot, slot_prev, slot_step, slot_force, emb, emb_mult, emb_scale, positions, d, x,
      q, eos_mask, self_pages, pages_per_slot, page_tokens, self_row_map, status);
}

template <int VPL, int RPC, class Kern, class... Args>
void launch_ln_cfg(Kern kernel, int rows, cudaStream_t s, Args... args) {
  const size_t smem = sizeof(float) * RPC * (VPL * 128 + 4);
  if (smem > 48 * 1024) {
    static unsigned long long configured = 0;
    int dev = 0;
    cudaGetDevice(&dev);
    if (!(configured & (1ull << (dev & 63)))) {
      cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      configured |= 1ull << (dev & 63);
    }
  }
  launch_pdl(kernel, dim3(blocks_for(rows, RPC)), dim3(kLnThreads), smem, s, args...);
}

// Launches of up to kLnWarpRows rows (decode steps) take the warp-per-row
// kernels, whose per-row latency is lower; larger ones (encoder passes) the
// 8-rows-per-CTA kernels, which issue far fewer instructions per row.
constexpr int kLnWarpRows = 2048;

template <int VPL>
void launch_residual_ln_v(const float* a, int lda, const float* r, int ldr, const float* gamma,
                          const float* beta, int rows, const int32_t* rows_dev, float* out,
                          const QuantOut& q, uint32_t* status, cudaStream_t s) {
  if (rows <= kLnWarpRows)
    launch_pdl(residual_ln_warp_kernel<VPL>, dim3(blocks_for(rows, kLnWarps)), dim3(kLnWarps * 32), 0, s,
               a, lda, r, ldr, gamma, beta, rows, rows_dev, out, q, status);
  else
    launch_ln_cfg<VPL, 8>(residual_ln_kernel<VPL, 8>, rows, s, a, lda, r, ldr, gamma, beta, rows, rows_dev, out, q, status);
}

template <int VPL>
void launch_ssru_v(const float* cf, int ld, int fcol, float* state, const int32_t* row_slot,
                   const float* residual, const float* gamma, const float* beta, int rows,
                   const int32_t* rows_dev, float* out, const QuantOut& q, uint32_t* status,
                   cudaStream_t s) {
  if (rows <= kLnWarpRows)
    launch_pdl(ssru_warp_kernel<VPL>, dim3(blocks_for(rows, kLnWarps)), dim3(kLnWarps * 32), 0, s, cf, ld,
               fcol, state, row_slot, residual, gamma, beta, rows, rows_dev, out, q, status);
  else
    launch_ln_cfg<VPL, 8>(ssru_kernel<VPL, 8>, rows, s, cf, ld, fcol, state, row_slot, residual, gamma, beta, rows, rows_dev, out, q, status);
}

void launch_residual_ln(const float* a, int lda, const float* r, int ldr, const float* gamma,
                        const float* beta, int rows, const int32_t* rows_dev, int d, float* out,
                        const QuantOut& q, uint32_t* status, cudaStream_t s) {
  if (rows <= 0) return;
  switch (d) {
    case 128: launch_residual_ln_v<1>(a, lda, r, ldr, gamma, beta, rows, rows_dev, out, q, status, s); break;
    case 256: launch_residual_ln_v<2>(a, lda, r, ldr, gamma, beta, rows, rows_dev, out, q, status, s); break;
    case 384: launch_residual_ln_v<3>(a, lda, r, ldr, gamma, beta, rows, rows_dev, out, q, status, s); break;
    case 512: launch_residual_ln_v<4>(a, lda, r, ldr, gamma, beta, rows, rows_dev, out, q, status, s); break;
    case 640: launch_residual_ln_v<5>(a, lda, r, ldr, gamma, beta, rows, rows_dev, out, q, status, s); break;
    case 768: launch_residual_ln_v<6>(a, lda, r, ldr, gamma, beta, rows, rows_dev, out, q, status, s); break;
    case 896: launch_residual_ln_v<7>(a, lda, r, ldr, gamma, beta, rows, rows_dev, out, q, status, s); break;
    case 1024: launch_residual_ln_v<8>(a, lda, r, ldr, gamma, beta, rows, rows_dev, out, q, status, s); break;
    default: flag_status_host(status, s); break;
  }
}

void launch_ssru(const float* cf, int ld, int fcol, float* state, const int32_t* row_slot,
                 const float* residual, const float* gamma, const float* beta, int rows,
                 const int32_t* rows_dev, int d, float* out, const QuantOut& q, uint32_t* status,
                 cudaStream_t s) {
  if (rows <= 0) return;
  switch (d) {
    case 128: launch_ssru_v<1>(cf, ld, fcol, state, row_slot, residual, gamma, beta, rows, rows_dev, out, q, status, s); break;
    case 256: launch_ssru_v<2>(cf, ld, fcol, state, row_slot, residual, gamma, beta, rows, rows_dev, out, q, status, s); break;
    case 384: launch_ssru_v<3>(cf, ld, fcol, state, row_slot, residual, gamma, beta, rows, rows_dev, out, q, status, s); break;
    case 512: launch_ssru_v<4>(cf, ld, fcol, state, row_slot, residual, gamma, beta, rows, rows_dev, out, q, status, s); break;
    case 640: launch_ssru_v<5>(cf, ld, fcol, state, row_slot, residual, gamma, beta, rows, rows_dev, out, q, status, s); break;
    case 768: launch_ssru_v<6>(cf, ld, fcol, state, row_slot, residual, gamma, beta, rows, rows_dev, out, q, status, s); break;
    case 896: launch_ssru_v<7>(cf, ld, fcol, state, row_slot, residual, gamma, beta, rows, rows_dev, out, q, status, s); break;
    case 1024: launch_ssru_v<8>(cf, ld, fcol, state, row_slot, residual, gamma, beta, rows, rows_dev, out, q, status, s); break;
    default: flag_status_host(status, s); break;
  }
}

template <int HD>
cudaError_t launch_attn_encoder_hd(const float* qkv, const int32_t* cu_seqlens,
                                   const int32_t* seq_ids, int n_seqs, int max_len, int d,
                                   int heads, int8_t* out_q, float alpha, uint32_t* status,
                                   cudaStream_t s) {
  const size_t smem = sizeof(float) * ((size_t)max_len * (2 * HD + 4) +
                                       (size_t)kEncWarps * kEncQpw * HD +
                                       (size_t)kEncWarps * kEncQpw * max_len);
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(attn_encoder_kernel<HD>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem));
    if (e != cudaSuccess) return e;
  }
  const int chunks = (max_len + 31) / 32;
  launch_pdl(attn_encoder_kernel<HD>, dim3(dim3(n_seqs, heads, chunks)), dim3(kEncWarps * 32), smem, s, qkv, cu_seqlens, seq_ids, d,
                                                                        max_len, out_q, alpha, 1.0f, status);
  return cudaGetLastError();
}

cudaError_t launch_attn_encoder(const float* qkv, const int32_t* cu_seqlens,
                                const int32_t* seq_ids, int n_seqs, int max_len, int d, int heads,
                                int8_t* out_q, float alpha, uint32_t* status, cudaStream_t s) {
  if (n_seqs <= 0) return cudaSuccess;
  switch (d / heads) {
    case 32: return launch_attn_encoder_hd<32>(qkv, cu_seqlens, seq_ids, n_seqs, max_len, d, heads, out_q, alpha, status, s);
    case 48: return launch_attn_encoder_hd<48>(qkv, cu_seqlens, seq_ids, n_seqs, max_len, d, heads, out_q, alpha, status, s);
    case 64: return launch_attn_encoder_hd<64>(qkv, cu_seqlens, seq_ids, n_seqs, max_len, d, heads, out_q, alpha, status, s);
    default: return cudaErrorInvalidValue;
  }
}

template <int HD, int PT>
cudaError_t launch_attn_decode_hd(const float* q, int ldq, int rows, const int32_t* rows_dev,
                                  const int32_t* row_slot, const int32_t* row_order,
                                  const int32_t* slot_len, int len_add, const int32_t* page_table,
                                  int pages_per_slot, const KvBoxMaps* k_maps,
                                  const KvBoxMaps* v_maps, int d, int heads, int8_t* out_q,
                                  float alpha, uint32_t* status, cudaStream_t s) {
  constexpr int W = kDecGroup * HD;
  const size_t smem = 1024 + sizeof(float) * ((size_t)kDecSlots * ((kDecChunk / 8) * 8 * W + 256) +
                                              (size_t)kDecGroup * kMaxSeq);
  static unsigned long long configured = 0;  // one bit per device ordinal
  static int sms[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  dev &= 63;
  if (!(configured & (1ull << dev))) {
    cudaError_t e = cudaFuncSetAttribute(attn_decode_kernel<HD, PT>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(attn_decode_kernel<HD, PT>, cudaFuncAttributePreferredSharedMemoryCarveout,
                               (int)cudaSharedmemCarveoutMaxShared);
    if (e != cudaSuccess) return e;
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    sms[dev] = n > 0 ? n : 148;
    configured |= 1ull << dev;
  }
  // three CTAs per SM (the 2-slot ring takes ~70 KB of shared memory per CTA)
  const long long items = (long long)rows * (heads / kDecGroup);
  const int grid = (int)std::min<long long>(items, 3LL * sms[dev]);
  launch_pdl(attn_decode_kernel<HD, PT>, dim3(grid), dim3(kDecThreads), smem, s, q, ldq, rows_dev, rows,
             row_slot, row_order, slot_len, len_add, page_table, pages_per_slot, *k_maps, *v_maps, d,
             heads, out_q, alpha, status);
  return cudaGetLastError();
}

template <int HD>
cudaError_t launch_attn_decode_pt(const float* q, int ldq, int rows, const int32_t* rows_dev,
                                  const int32_t* row_slot, const int32_t* row_order,
                                  const int32_t* slot_len, int len_add, const int32_t* page_table,
                                  int pages_per_slot, int page_tokens, const KvBoxMaps* k_map,
                                  const KvBoxMaps* v_map, int d, int heads, int8_t* out_q,
                                  float alpha, uint32_t* status, cudaStream_t s) {
  switch (page_tokens) {
    case 8: return launch_attn_decode_hd<HD, 8>(q, ldq, rows, rows_dev, row_slot, row_order, slot_len, len_add, page_table, pages_per_slot, k_map, v_map, d, heads, out_q, alpha, status, s);
    case 16: return launch_attn_decode_hd<HD, 16>(q, ldq, rows, rows_dev, row_slot, row_order, slot_len, len_add, page_table, pages_per_slot, k_map, v_map, d, heads, out_q, alpha, status, s);
    case 32: return launch_attn_decode_hd<HD, 32>(q, ldq, rows, rows_dev, row_slot, row_order, slot_len, len_add, page_table, pages_per_slot, k_map, v_map, d, heads, out_q, alpha, status, s);
    default: return cudaErrorInvalidValue;
  }
}

cudaError_t launch_attn_decode(const float* q, int ldq, int rows, const int32_t* rows_dev,
                               const int32_t* row_slot, const int32_t* row_order,
                               const int32_t* slot_len, int len_add, const int32_t* page_table,
                               int pages_per_slot, int page_tokens, const KvBoxMaps* k_map,
                               const KvBoxMaps* v_map, int d, int heads, int8_t* out_q,
                               float alpha, uint32_t* status, cudaStream_t s) {
  if (rows <= 0) return cudaSuccess;
  if (heads % kDecGroup != 0 || d != heads * (d / heads)) return cudaErrorInvalidValue;
  switch (d / heads) {
    case 32: return launch_attn_decode_pt<32>(q, ldq, rows, rows_dev, row_slot, row_order, slot_len, len_add, page_table, pages_per_slot, page_tokens, k_map, v_map, d, heads, out_q, alpha, status, s);
    case 48: return launch_attn_decode_pt<48>(q, ldq, rows, rows_dev, row_slot, row_order, slot_len, len_add, page_table, pages_per_slot, page_tokens, k_map, v_map, d, heads, out_q, alpha, status, s);
    case 64: return launch_attn_decode_pt<64>(q, ldq, rows, rows_dev, row_slot, row_order, slot_len, len_add, page_table, pages_per_slot, page_tokens, k_map, v_map, d, heads, out_q, alpha, status, s);
    default: return cudaErrorInvalidValue;
  }
}

void launch_quantize(const float* x, long long n, float alpha, int8_t* out, uint32_t* status,
                     cudaStream_t s) {
  if (n <= 0) return;
  const long long n4 = n / 4;
  launch_pdl(quantize_kernel, dim3(blocks_for(n4, 256)), dim3(256), 0, s, x, n4, alpha, out, status);
}

void launch_finalize(int rows, const int32_t* rows_dev, const int32_t* row_slot,
                     unsigned long long* best,
                     int32_t* slot_prev, int32_t* slot_step, const int32_t* slot_limit,
                     int32_t* step_tokens, uint8_t* done, uint32_t* status, cudaStream_t s) {
  if (rows <= 0) return;
  launch_pdl(finalize_kernel, dim3(blocks_for(rows, 128)), dim3(128), 0, s, rows, rows_dev, row_slot, best, slot_prev, slot_step,
                                                        slot_limit, step_tokens, done, status);
}

void launch_shortlist_masks(int n, const int32_t* slots, const int32_t* tokens, const int32_t* cu,
                            const int32_t* offsets, const int32_t* targets, int first_num, int vocab,
                            uint32_t* masks, cudaStream_t s) {
  if (n <= 0) return;
  const int words = (vocab + 31) / 32;
  launch_pdl(shortlist_mask_kernel, dim3(n), dim3(256), (size_t)words * 4, s, n, slots, tokens, cu,
             offsets, targets, first_num, vocab, words, masks);
}

void launch_step_rows(int32_t* table, int rmax, const uint8_t* done, const int32_t* join,
                      const int32_t* slot_step, const int32_t* slot_src, int32_t* scratch,
                      uint32_t* status, cudaStream_t s) {
  launch_pdl(step_rows_kernel, dim3(1), dim3(kRowsThreads), 0, s, table, rmax, done, join, slot_step,
             slot_src, scratch, status);
}

void launch_init_slots(int n, const int32_t* slots, const int32_t* limits, const int32_t* force,
                       const int32_t* src_len, int32_t* slot_prev, int32_t* slot_step,
                       int32_t* slot_limit, int32_t* slot_force, int32_t* slot_src,
                       float* ssru_state, int layers, int max_slots, int d,
                       const int32_t* page_rows, int32_t* cross_pages, int32_t* self_pages,
                       int pages_per_slot, cudaStream_t s) {
  if (n <= 0) return;
  launch_pdl(init_slots_kernel, dim3(n), dim3(128), 0, s, n, slots, limits, force, src_len, slot_prev, slot_step,
                                      slot_limit, slot_force, slot_src, ssru_state, layers,
             max_slots, d, page_rows, cross_pages, self_pages, pages_per_slot);
}

}  // namespace mc
