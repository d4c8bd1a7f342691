// q8_gemm.cu -- int8 x int8 -> int32 GEMM on the 5th-generation tensor cores.
//
// Replaces Q8Linear::run_into's integer GEMM and dequantizing epilogue
// (crates/marian-cpu/src/q8_gemm.rs:380-448, q8_avx2.rs:125-229) and the
// tied-vocabulary scoring of select_token (q8_engine.rs:749-790).
//
// One CTA computes a 128 x BN output tile:
//   warp 0      TMA producer: A and W tiles (128 K-bytes each) into a
//               STAGES-deep ring of 128-byte-swizzled shared-memory buffers;
//   warp 1      allocates TMEM and issues tcgen05.mma.kind::i8 (K = 32 per
//               instruction) from one elected thread, committing each stage
//               back to the producer and the finished accumulator to the
//               epilogue;
//   warps 2..5  epilogue: tcgen05.ld of the int32 accumulators (one row per
//               thread, lanes = rows), dequantize/bias/ReLU/residual, and
//               either an f32 store, an int8 store quantized for the next
//               linear, or a per-row masked argmax merged with a 64-bit
//               atomicMax.
#include "common.cuh"
#include "q8_gemm.cuh"

#include <cudaTypedefs.h>

namespace mc {

namespace {

constexpr int kBM = 128;
constexpr int kBK = 128;  // bytes of K per stage (= int8 elements)
constexpr int kEpiWarps = 8;  // two warps per TMEM lane quarter, each half the columns
constexpr int kThreads = 64 + 32 * kEpiWarps;

__device__ __forceinline__ unsigned long long pack_argmax(float v, int32_t n) {
  v = v + 0.0f;  // -0 -> +0: equal logits must compare equal (strict '>')
  uint32_t b = __float_as_uint(v);
  uint32_t ord = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
  return (static_cast<unsigned long long>(ord) << 32) | (0xFFFFFFFFu - static_cast<uint32_t>(n));
}

template <int BN>
__device__ __forceinline__ void epilogue_chunk(const GemmGroup& g, const uint32_t (&r)[32],
                                               int row, int dest_row, int nb, float row_scale,
                                               uint32_t* status, float& best, int& best_n) {
  const int n_end = g.n;
  if (g.mode == kEpiI32) {
    int32_t* out = static_cast<int32_t*>(g.out) + (size_t)dest_row * g.ldo + g.col_off;
#pragma unroll
    for (int j = 0; j < 32; ++j)
      if (nb + j < n_end) out[nb + j] = static_cast<int32_t>(r[j]);
    return;
  }
  if (g.mode == kEpiArgmax) {
    const bool mask_eos = g.eos_mask != nullptr && g.eos_mask[row] != 0;
    uint32_t cand = g.cand_bits[nb >> 5];  // nb is a multiple of 32
    if (nb == 0 && mask_eos) cand &= ~1u;
    const float uscale = g.row_scale ? __fmul_rn(row_scale, g.uniform_scale) : g.uniform_scale;
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      const int n = nb + j;
      if (n >= n_end) break;
      if (!((cand >> j) & 1u)) continue;
      float scale = uscale;
      if (g.col_scale) scale = g.row_scale ? __fmul_rn(row_scale, g.col_scale[n]) : g.col_scale[n];
      const float logit = dequant(static_cast<int32_t>(r[j]), scale, g.bias ? g.bias[n] : 0.0f);
      if (logit > best) {  // strict: the lowest index wins ties
        best = logit;
        best_n = n;
      }
    }
    return;
  }
  float v[32];
#pragma unroll
  for (int j = 0; j < 32; ++j) {
    const int n = nb + j;
    if (n < n_end) {
      float scale = g.col_scale ? g.col_scale[n] : g.uniform_scale;
      if (g.row_scale) scale = __fmul_rn(row_scale, scale);
      float x = dequant(static_cast<int32_t>(r[j]), scale, g.bias ? g.bias[n] : 0.0f);
      if (g.relu) x = fmaxf(x, 0.0f);
      if (g.residual) x = __fadd_rn(x, g.residual[(size_t)row * g.ldr + n]);
      v[j] = x;
    } else {
      v[j] = 0.0f;
    }
  }
  const bool full = nb + 32 <= n_end;
  if (g.mode == kEpiF32) {
    float* out = static_cast<float*>(g.out) + (size_t)dest_row * g.ldo + g.col_off + nb;
    if (full && ((reinterpret_cast<uintptr_t>(out) & 15) == 0)) {
      float4* o4 = reinterpret_cast<float4*>(out);
#pragma unroll
      for (int j = 0; j < 8; ++j) o4[j] = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
    } else {
      for (int j = 0; j < 32; ++j)
        if (nb + j < n_end) out[j] = v[j];
    }
  } else {  // kEpiQ8
    int8_t* out = static_cast<int8_t*>(g.out) + (size_t)dest_row * g.ldo + g.col_off + nb;
    int8_t q[32];
#pragma unroll
    for (int j = 0; j < 32; ++j) q[j] = (nb + j < n_end) ? quantize_one(v[j], g.alpha, status) : 0;
    if (full && ((reinterpret_cast<uintptr_t>(out) & 15) == 0)) {
      uint4* o = reinterpret_cast<uint4*>(out);
      const uint4* s = reinterpret_cast<const uint4*>(q);
      o[0] = s[0];
      o[1] = s[1];
    } else {
      for (int j = 0; j < 32; ++j)
        if (nb + j < n_end) out[j] = q[j];
    }
  }
}

template <int BN, int STAGES>
__global__ void __launch_bounds__(kThreads, 1) q8_gemm_kernel(const __grid_constant__ GemmParams p) {
  const GemmGroup& g = p.g[blockIdx.z];
  const int n0 = blockIdx.x * BN;
  const int m0 = blockIdx.y * kBM;
  if (n0 >= g.n) return;  // whole CTA leaves before any barrier

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* smem_a = smem;                           // STAGES x 16 KB
  uint8_t* smem_b = smem + STAGES * kBM * kBK;      // STAGES x BN*128
  __shared__ __align__(8) uint64_t full_bar[STAGES];
  __shared__ __align__(8) uint64_t empty_bar[STAGES];
  __shared__ __align__(8) uint64_t accum_bar;
  __shared__ uint32_t tmem_base_s;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int num_kb = (p.k + kBK - 1) / kBK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    mbar_init(&accum_bar, 1);
    fence_barrier_init();
    tma_prefetch_desc(&g.tmap_a);
    tma_prefetch_desc(&g.tmap_b);
  }
  if (warp == 1) {
    tmem_alloc(&tmem_base_s, BN);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = tmem_base_s;

  if (warp == 0) {
    if (lane == 0) {
      constexpr uint32_t kStageBytes = kBM * kBK + BN * kBK;
      for (int kb = 0; kb < num_kb; ++kb) {
        const int s = kb % STAGES;
        const uint32_t phase = (kb / STAGES) & 1;
        if (!mbar_wait(&empty_bar[s], phase ^ 1, p.status)) break;
        mbar_arrive_expect_tx(&full_bar[s], kStageBytes);
        tma_load_2d(smem_a + s * kBM * kBK, &g.tmap_a, kb * kBK, m0, &full_bar[s]);
        tma_load_2d(smem_b + s * BN * kBK, &g.tmap_b, kb * kBK, n0, &full_bar[s]);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_i8(kBM, BN);
      bool ok = true;
      for (int kb = 0; kb < num_kb && ok; ++kb) {
        const int s = kb % STAGES;
        const uint32_t phase = (kb / STAGES) & 1;
        ok = mbar_wait(&full_bar[s], phase, p.status);
        if (!ok) break;
        tc_fence_after();
        const uint32_t a_addr = smem_u32(smem_a + s * kBM * kBK);
        const uint32_t b_addr = smem_u32(smem_b + s * BN * kBK);
#pragma unroll
        for (int kk = 0; kk < kBK / 32; ++kk) {
          mma_i8(tmem_base, sdesc_k_sw128(a_addr + kk * 32), sdesc_k_sw128(b_addr + kk * 32), idesc,
                 (kb > 0 || kk > 0) ? 1u : 0u);
        }
        mma_commit(&empty_bar[s]);
      }
      mma_commit(&accum_bar);
    }
  } else {
    // Epilogue warps 2..9: warp % 4 selects the TMEM lane quarter (rows),
    // (warp - 2) / 4 the half of the tile's columns.
    const int quarter = warp & 3;
    const int half = (warp - 2) >> 2;
    const int row_in_tile = quarter * 32 + lane;
    const int row = m0 + row_in_tile;
    const bool row_ok = row < p.m;
    // Warp-uniform: tcgen05.ld below is .sync.aligned.
    const bool ready = __all_sync(0xffffffffu, mbar_wait(&accum_bar, 0, p.status));
    tc_fence_after();
    if (ready) {
      const int dest_row = row_ok ? (g.row_map ? g.row_map[row] : row) : 0;
      const float row_scale = (row_ok && g.row_scale) ? g.row_scale[row] : 1.0f;
      float best = -INFINITY;
      int best_n = -1;
      const uint32_t lane_base = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16);
      constexpr int kHalf = BN / 2 >= 32 ? BN / 2 : 32;
#pragma unroll 1
      for (int c0 = half * kHalf; c0 < BN && c0 < (half + 1) * kHalf; c0 += 32) {
        uint32_t r[32];
        tmem_ld_32x32b_x32(lane_base + c0, r);
        tmem_ld_wait();
        if (row_ok && dest_row >= 0 && n0 + c0 < g.n)
          epilogue_chunk<BN>(g, r, row, dest_row, n0 + c0, row_scale, p.status, best, best_n);
      }
      if (g.mode == kEpiArgmax && row_ok && dest_row >= 0 && best_n >= 0)
        atomicMax(&g.argmax[dest_row], pack_argmax(best, best_n));
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, BN);
  }
}

template <int BN, int STAGES>
constexpr int smem_bytes() {
  return STAGES * (kBM * kBK + BN * kBK) + 1024;
}

template <int BN, int STAGES>
cudaError_t launch_impl(const GemmParams& p, cudaStream_t stream) {
  constexpr int smem = smem_bytes<BN, STAGES>();
  auto kern = q8_gemm_kernel<BN, STAGES>;
  static unsigned long long configured = 0;  // one bit per device ordinal
  int dev = 0;
  cudaGetDevice(&dev);
  if (!(configured & (1ull << (dev & 63)))) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    configured |= 1ull << (dev & 63);
  }
  dim3 grid((p.max_n + BN - 1) / BN, (p.m + kBM - 1) / kBM, p.num_groups);
  kern<<<grid, kThreads, smem, stream>>>(p);
  return cudaGetLastError();
}

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    cudaDriverEntryPointQueryResult q;
    void* ptr = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  }
  return fn;
}

}  // namespace

bool encode_tmap_i8(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols,
                    uint32_t box_rows) {
  auto fn = encode_fn();
  if (!fn || !base || rows == 0 || cols == 0 || (cols % 16) != 0 ||
      (reinterpret_cast<uintptr_t>(base) & 15) != 0)
    return false;
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {cols};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(kBK), box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box,
                  estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

int pick_bn(int m, int max_n) {
  // Fill the 148 SMs: prefer the widest tile that still gives one wave.
  const long m_tiles = (m + kBM - 1) / kBM;
  if (m_tiles * ((max_n + 255) / 256) >= 148) return 256;
  if (m_tiles * ((max_n + 127) / 128) >= 148) return 128;
  return 64;
}

cudaError_t launch_q8_gemm(const GemmParams& p, int bn, cudaStream_t stream) {
  if (p.m <= 0 || p.num_groups <= 0) return cudaSuccess;
  switch (bn) {
    case 256: return launch_impl<256, 4>(p, stream);
    case 128: return launch_impl<128, 6>(p, stream);
    default: return launch_impl<64, 8>(p, stream);
  }
}

}  // namespace mc
