// ops_capi.cu -- operator-level C ABI (device pointers): the Q8 GEMM and the
// status word its kernels report into.
#include <cstring>
#include <mutex>

#include <cmath>

#include "kernels.cuh"
#include "linear_ln.cuh"
#include "marian_cuda.h"
#include "q8_gemm.cuh"

namespace {

std::mutex g_status_mutex;
uint32_t* g_status[64] = {nullptr};

// The operator API's per-device status word (allocated once per device).
uint32_t* op_status_word() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
  std::lock_guard<std::mutex> lock(g_status_mutex);
  if (!g_status[dev]) {
    uint32_t* p = nullptr;
    if (cudaMalloc(&p, sizeof(uint32_t)) != cudaSuccess) return nullptr;
    if (cudaMemset(p, 0, sizeof(uint32_t)) != cudaSuccess) return nullptr;
    g_status[dev] = p;
  }
  return g_status[dev];
}

}  // namespace

extern "C" mc_status mc_q8_gemm(const int8_t* a, const int8_t* w, int32_t m, int32_t n, int32_t k,
                                const float* row_scale, const float* col_scale, const float* bias,
                                const float* residual, int32_t relu, int32_t mode, void* out,
                                void* stream) {
  if (m < 0 || n <= 0 || k <= 0 || (k % 16) != 0 || !a || !w || !out || (mode != 0 && mode != 1) ||
      (mode == 1 && !col_scale))
    return MC_INVALID_INPUT;
  if (m == 0) return MC_OK;
  uint32_t* status = op_status_word();
  if (!status) return MC_CUDA;
  mc::GemmParams p;
  std::memset(&p, 0, sizeof(p));
  const int bn = mc::pick_bn(m, n);
  mc::GemmGroup& g = p.g[0];
  if (!mc::encode_tmap_i8(&g.tmap_a, a, (uint64_t)m, (uint64_t)k, 128) ||
      !mc::encode_tmap_i8(&g.tmap_b, w, (uint64_t)n, (uint64_t)k, (uint32_t)bn))
    return MC_INVALID_INPUT;
  g.col_scale = col_scale;
  g.row_scale = row_scale;
  g.bias = bias;
  g.residual = residual;
  g.ldr = n;
  g.out = out;
  g.n = n;
  g.ldo = n;
  g.col_off = 0;
  g.mode = mode == 0 ? mc::kEpiI32 : mc::kEpiF32;
  g.relu = relu != 0;
  p.m = m;
  p.k = k;
  p.num_groups = 1;
  p.max_n = n;
  p.status = status;
  cudaError_t e = mc::launch_q8_gemm(p, bn, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? MC_OK : MC_CUDA;
}

extern "C" mc_status mc_q8_linear(const float* x, int32_t m, int32_t k, const int8_t* w, int32_t n,
                                  float activation_mult, float weight_mult, const float* bias,
                                  float* y, void* stream) {
  if (m < 0 || n <= 0 || k <= 0 || (k % 16) != 0 || !x || !w || !y ||
      (reinterpret_cast<uintptr_t>(x) & 15) != 0)
    return MC_INVALID_INPUT;
  if (!std::isfinite(activation_mult) || activation_mult <= 0.0f || !std::isfinite(weight_mult) ||
      weight_mult <= 0.0f)
    return MC_INVALID_INPUT;
  const float inverse_scale = 1.0f / (activation_mult * weight_mult);  // q8_gemm.rs:438
  if (!std::isfinite(inverse_scale) || inverse_scale <= 0.0f) return MC_INVALID_INPUT;
  if (m == 0) return MC_OK;
  uint32_t* status = op_status_word();
  if (!status) return MC_CUDA;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // Q8LinearScratch::quantized (q8_gemm.rs:44-49): a stream-ordered buffer
  // for the quantized activations, released when the GEMM is done with it.
  int8_t* q = nullptr;
  if (cudaMallocAsync(reinterpret_cast<void**>(&q), (size_t)m * k, s) != cudaSuccess) return MC_CUDA;
  mc::launch_quantize(x, (long long)m * k, activation_mult, q, status, s);
  mc::GemmParams p;
  std::memset(&p, 0, sizeof(p));
  const int bn = mc::pick_bn(m, n);
  mc::GemmGroup& g = p.g[0];
  mc_status st = MC_OK;
  if (!mc::encode_tmap_i8(&g.tmap_a, q, (uint64_t)m, (uint64_t)k, 128) ||
      !mc::encode_tmap_i8(&g.tmap_b, w, (uint64_t)n, (uint64_t)k, (uint32_t)bn)) {
    st = MC_INVALID_INPUT;
  } else {
    g.uniform_scale = inverse_scale;
    g.bias = bias;
    g.out = y;
    g.n = n;
    g.ldo = n;
    g.mode = mc::kEpiF32;
    p.m = m;
    p.k = k;
    p.num_groups = 1;
    p.max_n = n;
    p.status = status;
    if (mc::launch_q8_gemm(p, bn, s) != cudaSuccess) st = MC_CUDA;
  }
  if (cudaFreeAsync(q, s) != cudaSuccess && st == MC_OK) st = MC_CUDA;
  return st;
}

extern "C" mc_status mc_q8_linear_ln(const float* x, int32_t m, int32_t k, const int8_t* w, int32_t d,
                                     float activation_mult, float weight_mult, const float* bias,
                                     const float* residual, const float* gamma, const float* beta,
                                     float* y, int8_t* y_q, float y_alpha, void* stream) {
  if (m < 0 || k <= 0 || (k % 16) != 0 || !x || !w || !residual || !gamma || !beta || !y ||
      mc::linear_ln_cluster(d) == 0 || (reinterpret_cast<uintptr_t>(x) & 15) != 0 ||
      (reinterpret_cast<uintptr_t>(residual) & 15) != 0 || (reinterpret_cast<uintptr_t>(y) & 15) != 0 ||
      (reinterpret_cast<uintptr_t>(gamma) & 15) != 0 || (reinterpret_cast<uintptr_t>(beta) & 15) != 0 ||
      (y_q && ((reinterpret_cast<uintptr_t>(y_q) & 3) != 0 || !std::isfinite(y_alpha) || y_alpha <= 0.0f)))
    return MC_INVALID_INPUT;
  if (!std::isfinite(activation_mult) || activation_mult <= 0.0f || !std::isfinite(weight_mult) ||
      weight_mult <= 0.0f)
    return MC_INVALID_INPUT;
  const float inverse_scale = 1.0f / (activation_mult * weight_mult);  // q8_gemm.rs:438
  if (!std::isfinite(inverse_scale) || inverse_scale <= 0.0f) return MC_INVALID_INPUT;
  if (m == 0) return MC_OK;
  uint32_t* status = op_status_word();
  if (!status) return MC_CUDA;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int8_t* q = nullptr;
  if (cudaMallocAsync(reinterpret_cast<void**>(&q), (size_t)m * k, s) != cudaSuccess) return MC_CUDA;
  mc::launch_quantize(x, (long long)m * k, activation_mult, q, status, s);
  mc::LinearLnParams p;
  std::memset(&p, 0, sizeof(p));
  mc_status st = MC_OK;
  const int bn = d / mc::linear_ln_cluster(d);
  if (!mc::encode_tmap_i8(&p.tmap_a, q, (uint64_t)m, (uint64_t)k, 128) ||
      !mc::encode_tmap_i8(&p.tmap_b, w, (uint64_t)d, (uint64_t)k, (uint32_t)bn)) {
    st = MC_INVALID_INPUT;
  } else {
    p.uniform_scale = inverse_scale;
    p.bias = bias;
    p.residual = residual;
    p.ldr = d;
    p.gamma = gamma;
    p.beta = beta;
    p.out = y;
    p.q.base = y_q;
    p.q.stride = 0;
    p.q.count = y_q ? 1 : 0;
    p.q.alpha[0] = y_alpha;
    p.cap = m;
    p.k = k;
    p.status = status;
    if (mc::launch_q8_linear_ln(p, d, s) != cudaSuccess) st = MC_CUDA;
  }
  if (cudaFreeAsync(q, s) != cudaSuccess && st == MC_OK) st = MC_CUDA;
  return st;
}

extern "C" mc_status mc_op_status(uint32_t* status_bits) {
  uint32_t* status = op_status_word();
  if (!status || !status_bits) return MC_CUDA;
  if (cudaDeviceSynchronize() != cudaSuccess) return MC_CUDA;
  if (cudaMemcpy(status_bits, status, sizeof(uint32_t), cudaMemcpyDeviceToHost) != cudaSuccess)
    return MC_CUDA;
  if (cudaMemset(status, 0, sizeof(uint32_t)) != cudaSuccess) return MC_CUDA;
  return MC_OK;
}
