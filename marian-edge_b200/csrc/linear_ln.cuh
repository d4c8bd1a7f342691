// linear_ln.cuh -- host interface of the fused Q8 linear + residual + LayerNorm.
//
// out = LN(dequant(A x W^T) + residual) with gamma/beta, plus the quantized
// copies of out that the next linears read: Q8Linear::run_into
// (crates/marian-cpu/src/q8_gemm.rs:380-448) followed by
// residual_layer_norm_into (tensor.rs:132-155), in one launch.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "kernels.cuh"

namespace mc {

// Tensor maps come first so they keep the 64-byte alignment the TMA unit
// requires of a kernel-parameter map.
struct alignas(64) LinearLnParams {
  CUtensorMap tmap_a;        // A [rows, K] int8, box {128, 128}, 128-byte swizzle
  CUtensorMap tmap_b;        // W [d, K] int8, box {128, d / linear_ln_cluster(d)}
  CUtensorMap tmap_b2;       // proj: W2 [d, d] int8, box {128, d / linear_ln_cluster(d)}
  const float* col_scale;    // [d] per-column dequantization scale, or null
  float uniform_scale;       // used when col_scale is null
  const float* bias;         // [d] or null
  const float* residual;     // [rows, ldr]
  int32_t ldr;
  const float* gamma;        // [d]
  const float* beta;         // [d]
  float* out;                // [rows, d]
  QuantOut q;                // quantized copies of out, row stride d
  int32_t cap;               // rows the grid covers
  const int32_t* m_dev;      // nullable: device row count (clamped to cap)
  int32_t k;                 // inner dimension (multiple of 16)
  int32_t stages;            // shared-memory ring depth (set by the launcher)
  uint32_t* status;          // device status word (error bits)
  // proj != 0: the normalized rows are also the input of a second Q8 linear
  // W2 in the same launch, A2 = quantize(out, alpha2):
  //   proj 1: W2 [d, d] (the decoder's cross-attention query after its first
  //           LayerNorm), out2 = dequant(A2 x W2^T) * scale2 + bias2, f32;
  //   proj 2: W2 [4d, d] (the FFN's first linear after the second
  //           LayerNorm), out2q = quantize(ReLU(dequant(A2 x W2^T) * scale2 +
  //           bias2), alpha3), int8 (d = 128, 256 or 512).
  int32_t proj;
  const float* col_scale2;   // [N2] or null
  float uniform_scale2;
  const float* bias2;        // [N2] or null
  float* out2;               // proj 1: [rows, ldo2] f32
  int8_t* out2q;             // proj 2: [rows, ldo2] int8
  int32_t ldo2;              // elements
  float alpha2;              // W2's activation alpha
  float alpha3;              // proj 2: the next linear's activation alpha
};

// CTAs per cluster for model width d (each owns d / C output columns of a
// 128-row block), or 0 when the fused kernel does not support d.
int linear_ln_cluster(int d);

// Sets the kernels' shared-memory limits on the current device (before any
// stream capture; the launcher does it on first use otherwise).
cudaError_t prepare_q8_linear_ln();

// Launches the fused kernel over p.cap rows (m_dev rows when given).
cudaError_t launch_q8_linear_ln(const LinearLnParams& p, int d, cudaStream_t stream);

}  // namespace mc
