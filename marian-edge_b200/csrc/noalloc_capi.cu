// noalloc_capi.cu -- mc_q8_linear_noalloc: the Q8 linear of mc_q8_linear
// (quantize -> tcgen05 int8 GEMM -> dequantize + bias) for callers that
// cannot allocate device memory.
//
// Who needs it: a host application whose memory manager reserves the GPU's
// memory up front for its own pool (a cudaMalloc or cudaMallocAsync from a
// plugin then fails or fragments that pool), and latency-critical request
// paths that cannot afford an allocation's driver call and possible device
// synchronization.  mc_q8_linear allocates its quantized-activation scratch
// with cudaMallocAsync; this entry point uses a fixed device array instead.
//
// The scratch is the file-scope array g_linear_scratch below: 256 bytes for
// this entry point's status word, then MC_Q8_LINEAR_NOALLOC_MAX_ACTIVATIONS
// bytes for the quantized activations.  Every GPU on which the library's
// device code is loaded holds the array until the process exits.  Its device
// address is looked up once per device (cudaGetSymbolAddress, on the first
// call made with that device current); host code never passes the array's
// host-side name to a kernel.  The cached address belongs to the device
// context the first call ran in: a cudaDeviceReset after that call is not
// supported (the array is reloaded elsewhere with the module).  All calls on
// a device share the array: calls whose kernels overlap on the GPU
// (different streams without ordering) race on it.
#include <cmath>
#include <cstring>
#include <mutex>

#include "kernels.cuh"
#include "marian_cuda.h"
#include "q8_gemm.cuh"

namespace {

constexpr size_t kStatusBytes = 256;
constexpr size_t kActivationBytes = MC_Q8_LINEAR_NOALLOC_MAX_ACTIVATIONS;

static __device__ __align__(256) uint8_t g_linear_scratch[kStatusBytes + kActivationBytes];

std::mutex g_scratch_mutex;
uint8_t* g_scratch_addr[64] = {nullptr};  // device address of g_linear_scratch, per device

// One-time set-up per device: the device address of the scratch array.
mc_status scratch_address(uint8_t** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return MC_CUDA;
  std::lock_guard<std::mutex> lock(g_scratch_mutex);
  if (!g_scratch_addr[dev]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_linear_scratch) != cudaSuccess || !p) return MC_CUDA;
    g_scratch_addr[dev] = static_cast<uint8_t*>(p);
  }
  *out = g_scratch_addr[dev];
  return MC_OK;
}

}  // namespace

extern "C" mc_status mc_q8_linear_noalloc(const float* x, int32_t m, int32_t k, const int8_t* w,
                                          int32_t n, float activation_mult, float weight_mult,
                                          const float* bias, float* y, void* stream,
                                          uint32_t* status_bits) {
  if (m < 0 || n <= 0 || k <= 0 || (k % 16) != 0 || !x || !w || !y ||
      (reinterpret_cast<uintptr_t>(x) & 15) != 0)
    return MC_INVALID_INPUT;
  if ((uint64_t)m * (uint64_t)k > (uint64_t)kActivationBytes) return MC_INVALID_INPUT;
  if (!std::isfinite(activation_mult) || activation_mult <= 0.0f || !std::isfinite(weight_mult) ||
      weight_mult <= 0.0f)
    return MC_INVALID_INPUT;
  const float inverse_scale = 1.0f / (activation_mult * weight_mult);  // q8_gemm.rs:438
  if (!std::isfinite(inverse_scale) || inverse_scale <= 0.0f) return MC_INVALID_INPUT;
  uint8_t* base = nullptr;
  mc_status st = scratch_address(&base);
  if (st != MC_OK) return st;
  uint32_t* status = reinterpret_cast<uint32_t*>(base);
  int8_t* q = reinterpret_cast<int8_t*>(base + kStatusBytes);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (m > 0) {
    mc::GemmParams p;
    std::memset(&p, 0, sizeof(p));
    const int bn = mc::pick_bn(m, n);
    mc::GemmGroup& g = p.g[0];
    // Both tensor maps are encoded (and w's alignment checked) before any
    // launch, so an invalid weight pointer returns without touching the
    // scratch or its status word.
    if (!mc::encode_tmap_i8(&g.tmap_a, q, (uint64_t)m, (uint64_t)k, 128) ||
        !mc::encode_tmap_i8(&g.tmap_b, w, (uint64_t)n, (uint64_t)k, (uint32_t)bn))
      return MC_INVALID_INPUT;
    mc::launch_quantize(x, (long long)m * k, activation_mult, q, status, s);
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
    if (mc::launch_q8_gemm(p, bn, s) != cudaSuccess) return MC_CUDA;
  }
  if (status_bits) {
    // Report and clear this entry point's status word (it starts at zero).
    if (cudaMemcpyAsync(status_bits, status, sizeof(uint32_t), cudaMemcpyDeviceToHost, s) != cudaSuccess ||
        cudaMemsetAsync(status, 0, sizeof(uint32_t), s) != cudaSuccess ||
        cudaStreamSynchronize(s) != cudaSuccess)
      return MC_CUDA;
  }
  return MC_OK;
}
