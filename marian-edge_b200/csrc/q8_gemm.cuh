// q8_gemm.cuh -- host interface of the tcgen05 int8 GEMM.
//
// Y[m, n] = epilogue( sum_k A[m, k] * W[n, k] ) with A int8 [M, K] (activations
// already quantized and centred, i.e. the reference's u8 minus 127) and W int8
// [N, K] (canonical [out, in] weights, legacy_q8.rs:82-87).  The int32
// accumulation is exact, as q8_gemm.rs:539-553 requires.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace mc {

enum GemmMode : int32_t {
  kEpiI32 = 0,     // raw int32 accumulators
  kEpiF32 = 1,     // acc*scale + bias (+ReLU) (+residual), q8_gemm.rs:438-446
  kEpiQ8 = 2,      // quantize(relu?(acc*scale + bias), alpha) for the next linear
  kEpiArgmax = 3,  // masked argmax over n of acc*scale + bias (q8_engine.rs:749-790)
};

// One linear of a grouped launch.  Tensor maps come first so they keep the
// 64-byte alignment the TMA unit requires of a kernel-parameter map.
struct alignas(64) GemmGroup {
  CUtensorMap tmap_a;          // A [rows, K] int8, box {128, 128}, 128-byte swizzle
  CUtensorMap tmap_b;          // W [N, K] int8, box {128, BN}, 128-byte swizzle
  const float* col_scale;      // [N]: 1/(alpha_a * w_mult) per output column, or null
                               // to use uniform_scale for every column
  const float* row_scale;      // [M] or null: extra per-row factor (microbench)
  const float* bias;           // [N] or null; kEpiArgmax: [N rounded up to 32] with
                               // -inf at non-candidate ids and past N
  const float* residual;       // [M, ldr] or null (kEpiF32)
  void* out;                   // float / int8 / int32 output base
  const int32_t* row_map;      // [M] destination row per source row, or null
  unsigned long long* argmax;  // [dest rows] packed (value, index) maxima (kEpiArgmax)
  const uint8_t* eos_mask;     // [M] 1 = token 0 excluded for this row (kEpiArgmax)
  const uint32_t* cand_rows;   // kEpiArgmax, nullable: per-slot candidate bitmasks
                               // [slots][cand_words] (lexical shortlist)
  const int32_t* cand_slot;    // [M] slot of each row (indexes cand_rows)
  int32_t cand_words;          // words per candidate bitmask
  int32_t n;                   // output columns of this group
  int32_t ldo;                 // output row stride (elements)
  int32_t col_off;             // first output column of this group
  int32_t ldr;                 // residual row stride
  float alpha;                 // next linear's activation alpha (kEpiQ8)
  int32_t mode;
  int32_t relu;
  float uniform_scale;         // used when col_scale is null (per-tensor scale)
};

constexpr int kMaxGemmGroups = 3;

struct GemmParams {
  GemmGroup g[kMaxGemmGroups];
  int32_t m;           // rows of A actually used (the capacity when m_dev is set)
  const int32_t* m_dev;  // nullable: device row count, read by the kernel and
                         // clamped to m (launches replayed from a CUDA graph)
  int32_t k;           // inner dimension (multiple of 16)
  int32_t num_groups;
  int32_t max_n;       // max over groups of n
  int32_t stages;      // shared-memory ring depth (set by the launcher)
  uint32_t* status;    // device status word (error bits)
};

// Encodes a 2-D int8 tensor map over a row-major [rows, cols] matrix with a
// {128, box_rows} box and the 128-byte swizzle.  Returns false when the
// driver rejects it (alignment, stride or size).
bool encode_tmap_i8(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols,
                    uint32_t box_rows);

// Encodes a 3-D f32 tensor map over a KV-cache pool [rows, d] (row-major)
// for the decode attention: dims {32 floats, rows, d / 32 column blocks}
// (strides d * 4 and 128 bytes), box {32, box_rows, group_cols / 32} --
// box_rows (8, 4, 2 or 1) cache rows' slice of group_cols columns per copy
// (page_tokens, a multiple of 8, keeps a box that starts at a multiple of 8
// inside one page) -- with the 128-byte swizzle, which lands the slice in
// shared memory as [column block][box_rows rows][32 floats], 16-byte chunk
// c of 128-byte line l (l = block * box_rows + row) stored at chunk
// c ^ (l & 7).
bool encode_tmap_kv(CUtensorMap* map, const float* base, uint64_t rows, int d, int page_tokens,
                    int group_cols, int box_rows);

// Picks the N tile (64, 128 or 256) for a launch.
int pick_bn(int m, int max_n);

// Sets the kernels' shared-memory limits on the current device (done before
// any stream capture; launch_q8_gemm does it on first use otherwise).
cudaError_t prepare_q8_gemm();

// Launches the grouped GEMM.  The tensor maps in p must have been encoded with
// box_rows == 128 for A and box_rows == bn for B.
cudaError_t launch_q8_gemm(const GemmParams& p, int bn, cudaStream_t stream);

}  // namespace mc
