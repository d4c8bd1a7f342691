// q8_gemm.cu -- int8 x int8 -> int32 GEMM on the 5th-generation tensor cores.
//
// Replaces Q8Linear::run_into's integer GEMM and dequantizing epilogue
// (crates/marian-cpu/src/q8_gemm.rs:380-448, q8_avx2.rs:125-229) and the
// tied-vocabulary scoring of select_token (q8_engine.rs:749-790).
//
// One CTA computes 128 x BN output tiles (persistent over the tile list):
//   warp 0      TMA producer: A and W tiles (128 K-bytes each) into a
//               STAGES-deep ring of 128-byte-swizzled shared-memory buffers;
//   warp 1      allocates TMEM and issues tcgen05.mma.kind::i8 (K = 32 per
//               instruction) from one elected thread, committing each stage
//               back to the producer and the finished accumulator to the
//               epilogue;
//   warps 2..   EPI epilogue warps (16 for BN 128/256, 8 for BN 64):
//               tcgen05.ld of the int32 accumulators (one row per thread,
//               lanes = rows), dequantize/bias/ReLU/residual, and either an
//               f32 store, an int8 store quantized for the next linear, or a
//               per-row masked argmax merged with a 64-bit atomicMax.
#include "common.cuh"
#include "q8_gemm.cuh"

#include <cudaTypedefs.h>

namespace mc {

namespace {

constexpr int kBM = 128;
constexpr int kBK = 128;  // bytes of K per stage (= int8 elements)

// Epilogue warps per CTA: EPI / 4 per TMEM lane quarter, each taking an
// equal share of the tile's columns.  16 for the one-CTA-per-SM tiles (BN 128
// and 256), 8 for BN 64 (two CTAs per SM).
template <int EPI>
constexpr int threads_for() {
  return 64 + 32 * EPI;
}

__device__ __forceinline__ unsigned long long pack_argmax(float v, int32_t n) {
  v = v + 0.0f;  // -0 -> +0: equal logits must compare equal (strict '>')
  uint32_t b = __float_as_uint(v);
  uint32_t ord = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
  return (static_cast<unsigned long long>(ord) << 32) | (0xFFFFFFFFu - static_cast<uint32_t>(n));
}

// Per-warp staging tile for coalesced stores: 32 rows x stage_ld words.
// With 16 epilogue warps (one CTA per SM) lane i writes row i with 16-byte
// stores; at a stride of 36 words every 8 lanes cover the 32 banks once, so
// each store and each 16-byte read of 4 rows x 128 B takes the minimum 4
// shared-memory wavefronts.  With 8 (two CTAs per SM, where shared memory
// is short) the stride is 33 words and the stores are 4-byte: the odd
// stride keeps both the row-wise writes and the column-wise reads of the 32
// lanes on distinct banks.
template <int EPI>
constexpr int stage_ld() {
  return EPI == 16 ? 36 : 33;
}
template <int EPI>
constexpr int staging_bytes() {
  return EPI * 32 * stage_ld<EPI>() * 4;
}

// Low bytes of four ints -> one word (byte i = q[i]).
__device__ __forceinline__ uint32_t pack4_s8(int q0, int q1, int q2, int q3) {
  const uint32_t lo = __byte_perm((uint32_t)q0, (uint32_t)q1, 0x0040);
  const uint32_t hi = __byte_perm((uint32_t)q2, (uint32_t)q3, 0x0040);
  return __byte_perm(lo, hi, 0x5410);
}

// One 32-column chunk of one tile row per lane.  `ok` is this lane's row
// validity; the call itself is warp-uniform (tcgen05.ld precedes it).
// sbias / sscale: this chunk's 32 bias and column-scale values, staged in
// shared memory before the accumulator was ready (nullptr: none).
template <int BN, int EPI>
__device__ __forceinline__ void epilogue_chunk(const GemmGroup& g, const uint32_t (&r)[32],
                                               bool ok, int row, int dest_row, int nb,
                                               float row_scale, uint32_t* status, float& best,
                                               int& best_n, uint32_t* stage, const float* sbias,
                                               const float* sscale) {
  const int n_end = g.n;
  const int lane = threadIdx.x & 31;
  if (g.mode == kEpiArgmax) {
    // bias is the candidate-masked bias: -inf for ids that are not
    // candidates and past the last column (padded to whole 32-column
    // chunks), so no per-column mask or bounds test is needed.
    if (!ok) return;
    const float uscale = g.row_scale ? __fmul_rn(row_scale, g.uniform_scale) : g.uniform_scale;
    const float4* b4 = reinterpret_cast<const float4*>(sbias);
    float v[32];
#pragma unroll
    for (int j4 = 0; j4 < 8; ++j4) {
      const float4 b = b4[j4];
      v[4 * j4 + 0] = dequant(static_cast<int32_t>(r[4 * j4 + 0]), uscale, b.x);
      v[4 * j4 + 1] = dequant(static_cast<int32_t>(r[4 * j4 + 1]), uscale, b.y);
      v[4 * j4 + 2] = dequant(static_cast<int32_t>(r[4 * j4 + 2]), uscale, b.z);
      v[4 * j4 + 3] = dequant(static_cast<int32_t>(r[4 * j4 + 3]), uscale, b.w);
    }
    if (g.cand_rows) {  // the row's shortlist candidates (shortlist.rs:150-198)
      const uint32_t word = g.cand_rows[(size_t)g.cand_slot[row] * g.cand_words + (nb >> 5)];
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (!((word >> j) & 1u)) v[j] = -INFINITY;
    }
    if (nb == 0 && g.eos_mask != nullptr && g.eos_mask[row] != 0) v[0] = -INFINITY;
    float t16[16];
#pragma unroll
    for (int j = 0; j < 16; ++j) t16[j] = fmaxf(v[j], v[j + 16]);
#pragma unroll
    for (int w = 8; w > 0; w >>= 1)
#pragma unroll
      for (int j = 0; j < w; ++j) t16[j] = fmaxf(t16[j], t16[j + w]);
    const float m = t16[0];
    if (m > best) {  // strict: an earlier chunk keeps ties
      int jj = 31;
#pragma unroll
      for (int j = 30; j >= 0; --j) jj = (v[j] == m) ? j : jj;  // lowest index of the maximum
      best = m;
      best_n = nb + jj;
    }
    return;
  }
  if (g.mode == kEpiI32) {
    if (!ok) return;
    int32_t* out = static_cast<int32_t*>(g.out) + (size_t)dest_row * g.ldo + g.col_off;
#pragma unroll
    for (int j = 0; j < 32; ++j)
      if (nb + j < n_end) out[nb + j] = static_cast<int32_t>(r[j]);
    return;
  }
  float v[32];
  const bool full = nb + 32 <= n_end;
  if (full && !g.residual) {
    // Fast path: per-column scale and bias fetched four at a time, no
    // per-element bounds checks.
    const float us = g.uniform_scale;
#pragma unroll
    for (int j4 = 0; j4 < 8; ++j4) {
      float4 s4 = sscale ? reinterpret_cast<const float4*>(sscale)[j4] : make_float4(us, us, us, us);
      if (g.row_scale) {
        s4.x = __fmul_rn(row_scale, s4.x);
        s4.y = __fmul_rn(row_scale, s4.y);
        s4.z = __fmul_rn(row_scale, s4.z);
        s4.w = __fmul_rn(row_scale, s4.w);
      }
      const float4 b4 = sbias ? reinterpret_cast<const float4*>(sbias)[j4] : make_float4(0.f, 0.f, 0.f, 0.f);
      v[4 * j4 + 0] = dequant(static_cast<int32_t>(r[4 * j4 + 0]), s4.x, b4.x);
      v[4 * j4 + 1] = dequant(static_cast<int32_t>(r[4 * j4 + 1]), s4.y, b4.y);
      v[4 * j4 + 2] = dequant(static_cast<int32_t>(r[4 * j4 + 2]), s4.z, b4.z);
      v[4 * j4 + 3] = dequant(static_cast<int32_t>(r[4 * j4 + 3]), s4.w, b4.w);
    }
    if (g.relu) {
#pragma unroll
      for (int j = 0; j < 32; ++j) v[j] = fmaxf(v[j], 0.0f);
    }
  } else {
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      const int n = nb + j;
      float x = 0.0f;
      if (ok && n < n_end) {
        float scale = g.col_scale ? g.col_scale[n] : g.uniform_scale;
        if (g.row_scale) scale = __fmul_rn(row_scale, scale);
        x = dequant(static_cast<int32_t>(r[j]), scale, g.bias ? g.bias[n] : 0.0f);
        if (g.relu) x = fmaxf(x, 0.0f);
        if (g.residual) x = __fadd_rn(x, g.residual[(size_t)row * g.ldr + n]);
      }
      v[j] = x;
    }
  }
  if (g.mode == kEpiF32) {
    const bool aligned = ((reinterpret_cast<uintptr_t>(g.out) | (uintptr_t)g.ldo * 4 |
                           (uintptr_t)(g.col_off + nb) * 4) & 15) == 0;
    if (full && aligned) {
      // stage the 32x32 block, then each instruction stores 4 rows x 128 B
      constexpr int ld = stage_ld<EPI>();
      if constexpr (ld % 4 == 0) {
        float4* mine = reinterpret_cast<float4*>(stage + lane * ld);
#pragma unroll
        for (int j4 = 0; j4 < 8; ++j4) mine[j4] = make_float4(v[4 * j4], v[4 * j4 + 1], v[4 * j4 + 2], v[4 * j4 + 3]);
      } else {
#pragma unroll
        for (int j = 0; j < 32; ++j) stage[lane * ld + j] = __float_as_uint(v[j]);
      }
      __syncwarp();
      const int sub = lane >> 3, c4 = (lane & 7) * 4;
#pragma unroll
      for (int it = 0; it < 8; ++it) {
        const int rr = it * 4 + sub;
        const int drow = __shfl_sync(0xffffffffu, dest_row, rr);
        const bool rok = __shfl_sync(0xffffffffu, ok ? 1 : 0, rr) != 0;
        const uint32_t* srow = stage + rr * ld + c4;
        float4 val;
        if constexpr (ld % 4 == 0) {
          val = *reinterpret_cast<const float4*>(srow);
        } else {
          val = make_float4(__uint_as_float(srow[0]), __uint_as_float(srow[1]), __uint_as_float(srow[2]),
                            __uint_as_float(srow[3]));
        }
        if (rok) {
          float* o = static_cast<float*>(g.out) + (size_t)drow * g.ldo + g.col_off + nb + c4;
          *reinterpret_cast<float4*>(o) = val;
        }
      }
      __syncwarp();
    } else if (ok) {
      float* out = static_cast<float*>(g.out) + (size_t)dest_row * g.ldo + g.col_off + nb;
      for (int j = 0; j < 32; ++j)
        if (nb + j < n_end) out[j] = v[j];
    }
  } else {  // kEpiQ8
    // quantize(v, alpha) as quantize_one does: rint(v * alpha) clamped to
    // [-127, 127].  v comes from an integer accumulator times a finite scale
    // plus a finite bias (the loader rejects non-finite payloads and
    // scales), so it is finite unless it overflowed to +-inf, which the
    // running |v| maximum detects.  Rows past m and columns past n get
    // values too; the stores below skip them.
    uint32_t q4[8];
    float amax = 0.0f;
    const float al = g.alpha;
    const bool lower = !g.relu;  // after ReLU, v * alpha >= 0
#pragma unroll
    for (int w = 0; w < 8; ++w) {
      int qv[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int j = 4 * w + u;
        amax = fmaxf(amax, fabsf(v[j]));
        float t = fminf(__fmul_rn(v[j], al), 127.0f);
        if (lower) t = fmaxf(t, -127.0f);
        qv[u] = rint_low_byte(t);  // clamping before rounding = rounding before clamping
      }
      q4[w] = pack4_s8(qv[0], qv[1], qv[2], qv[3]);
    }
    const bool finite = amax <= 3.402823466e38f;
    if (!finite && ok) flag_status(status, kStatusNonFinite);
    const bool aligned = ((reinterpret_cast<uintptr_t>(g.out) | (uintptr_t)g.ldo |
                           (uintptr_t)(g.col_off + nb)) & 3) == 0;
    if (full && aligned) {
      // stage 32 rows x 32 bytes (row stride 12 words), then each
      // instruction stores 4 rows x 32 B
      uint4* mine = reinterpret_cast<uint4*>(stage + lane * 12);
      mine[0] = make_uint4(q4[0], q4[1], q4[2], q4[3]);
      mine[1] = make_uint4(q4[4], q4[5], q4[6], q4[7]);
      __syncwarp();
      const int sub = lane >> 3, w = lane & 7;
#pragma unroll
      for (int it = 0; it < 8; ++it) {
        const int rr = it * 4 + sub;
        const int drow = __shfl_sync(0xffffffffu, dest_row, rr);
        const bool rok = __shfl_sync(0xffffffffu, ok ? 1 : 0, rr) != 0;
        if (rok) {
          int8_t* o = static_cast<int8_t*>(g.out) + (size_t)drow * g.ldo + g.col_off + nb + 4 * w;
          *reinterpret_cast<uint32_t*>(o) = stage[rr * 12 + w];
        }
      }
      __syncwarp();
    } else if (ok) {
      int8_t* out = static_cast<int8_t*>(g.out) + (size_t)dest_row * g.ldo + g.col_off + nb;
      for (int j = 0; j < 32; ++j)
        if (nb + j < n_end) out[j] = (int8_t)((q4[j >> 2] >> (8 * (j & 3))) & 0xFF);
    }
  }
}

// Tile order shared by the three roles: tile t -> (group, m tile, n tile),
// n fastest.  Tiles past a group's own N are skipped by every role alike.
struct TileCoord {
  int z, m0, n0;
};

template <int BN>
__device__ __forceinline__ bool tile_coord(const GemmParams& p, int t, int n_tiles, int m_tiles,
                                           TileCoord* c) {
  const int per_group = n_tiles * m_tiles;
  c->z = t / per_group;
  const int rem = t - c->z * per_group;
  c->m0 = (rem / n_tiles) * kBM;
  c->n0 = (rem % n_tiles) * BN;
  return c->n0 < p.g[c->z].n;
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// Persistent: each CTA walks tiles blockIdx.x, blockIdx.x + gridDim.x, ...
// The shared-memory ring continues across tiles, and the accumulator is
// double-buffered in TMEM (2 x BN columns) so the epilogue of one tile
// overlaps the MMAs of the next.
template <int BN, int MAX_STAGES, int EPI>
__global__ void __launch_bounds__(threads_for<EPI>(), EPI == 8 ? 2 : 1) q8_gemm_kernel(
    const __grid_constant__ GemmParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int stages = p.stages;
  uint8_t* smem_a = smem;                           // stages x 16 KB
  uint8_t* smem_b = smem + stages * kBM * kBK;      // stages x BN*128
  uint32_t* staging = reinterpret_cast<uint32_t*>(smem_b + stages * BN * kBK);  // staging_bytes<EPI>()
  __shared__ __align__(8) uint64_t full_bar[MAX_STAGES];
  __shared__ __align__(8) uint64_t empty_bar[MAX_STAGES];
  __shared__ __align__(8) uint64_t tfull_bar[2];
  __shared__ __align__(8) uint64_t tempty_bar[2];
  __shared__ uint32_t tmem_base_s;
  // per epilogue warp: the bias and column scales of its columns of the
  // current tile (at most 64: BN / (EPI / 4))
  __shared__ __align__(16) float s_bias[EPI][64];
  __shared__ __align__(16) float s_scale[EPI][64];

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int num_kb = (p.k + kBK - 1) / kBK;
  const int n_tiles = (p.max_n + BN - 1) / BN;
  pdl_enter();
  // The device row count is loaded before the set-up and used after it, so
  // its latency overlaps the barrier initialization and TMEM allocation.
  const int m_raw = p.m_dev ? *p.m_dev : p.m;

  if (threadIdx.x == 0) {
    for (int s = 0; s < stages; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull_bar[b], 1);
      mbar_init(&tempty_bar[b], EPI);
    }
    fence_barrier_init();
    for (int z = 0; z < p.num_groups; ++z) {
      tma_prefetch_desc(&p.g[z].tmap_a);
      tma_prefetch_desc(&p.g[z].tmap_b);
    }
  }
  if (warp == 1) {
    tmem_alloc(&tmem_base_s, 2 * BN);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = tmem_base_s;
  const int m = max(0, min(m_raw, p.m));
  const int m_tiles = (m + kBM - 1) / kBM;
  const int total = n_tiles * m_tiles * p.num_groups;

  if (warp == 0) {
    if (lane == 0) {
      constexpr uint32_t kStageBytes = kBM * kBK + BN * kBK;
      const uint64_t keep = l2_policy_evict_last();  // weights: reused every step
      int kbg = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < total && ok; t += gridDim.x) {
        TileCoord c;
        if (!tile_coord<BN>(p, t, n_tiles, m_tiles, &c)) continue;
        const GemmGroup& g = p.g[c.z];
        for (int kb = 0; kb < num_kb; ++kb, ++kbg) {
          const int s = kbg % stages;
          const uint32_t phase = (kbg / stages) & 1;
          if (!(ok = mbar_wait(&empty_bar[s], phase ^ 1, p.status))) break;
          mbar_arrive_expect_tx(&full_bar[s], kStageBytes);
          tma_load_2d(smem_a + s * kBM * kBK, &g.tmap_a, kb * kBK, c.m0, &full_bar[s]);
          tma_load_2d_hint(smem_b + s * BN * kBK, &g.tmap_b, kb * kBK, c.n0, &full_bar[s], keep);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_i8(kBM, BN);
      int kbg = 0, it = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < total && ok; t += gridDim.x) {
        TileCoord c;
        if (!tile_coord<BN>(p, t, n_tiles, m_tiles, &c)) continue;
        const int buf = it & 1;
        if (!(ok = mbar_wait(&tempty_bar[buf], ((it >> 1) & 1) ^ 1, p.status))) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + buf * BN;
        for (int kb = 0; kb < num_kb; ++kb, ++kbg) {
          const int s = kbg % stages;
          const uint32_t phase = (kbg / stages) & 1;
          if (!(ok = mbar_wait(&full_bar[s], phase, p.status))) break;
          tc_fence_after();
          const uint32_t a_addr = smem_u32(smem_a + s * kBM * kBK);
          const uint32_t b_addr = smem_u32(smem_b + s * BN * kBK);
#pragma unroll
          for (int kk = 0; kk < kBK / 32; ++kk)
            mma_i8(d_tmem, sdesc_k_sw128(a_addr + kk * 32), sdesc_k_sw128(b_addr + kk * 32), idesc,
                   (kb > 0 || kk > 0) ? 1u : 0u);
          mma_commit(&empty_bar[s]);
        }
        mma_commit(&tfull_bar[buf]);
        ++it;
      }
    }
  } else {
    // Epilogue warps 2 .. EPI + 1: warp % 4 selects the TMEM lane quarter
    // (rows), (warp - 2) / 4 the share of the tile's columns.
    const int quarter = warp & 3;
    const int part = (warp - 2) >> 2;
    uint32_t* stage = staging + (warp - 2) * 32 * stage_ld<EPI>();
    int it = 0;
    for (int t = blockIdx.x; t < total; t += gridDim.x) {
      TileCoord c;
      if (!tile_coord<BN>(p, t, n_tiles, m_tiles, &c)) continue;
      const GemmGroup& g = p.g[c.z];
      const int buf = it & 1;
      constexpr int kShare = BN / (EPI / 4) >= 32 ? BN / (EPI / 4) : 32;
      static_assert(kShare <= 64, "s_bias holds 64 columns per warp");
      // The per-row operands are loaded, and the bias lines of this warp's
      // columns are prefetched into L1, before the accumulator is ready, so
      // their latency overlaps the MMAs.
      const int row = c.m0 + quarter * 32 + lane;
      const bool row_ok = row < m;
      const int dest_row = row_ok ? (g.row_map ? g.row_map[row] : row) : 0;
      const float row_scale = (row_ok && g.row_scale) ? g.row_scale[row] : 1.0f;
      const int c_first = part * kShare;
      const int nb_first = c.n0 + c_first;
      // This warp's bias and column scales are staged in shared memory now:
      // their loads (often DRAM: the KV-cache traffic evicts them from L2)
      // overlap the MMAs instead of following the accumulator.
      float* sb = s_bias[warp - 2];
      float* ss = s_scale[warp - 2];
      const bool has_bias = g.bias != nullptr && g.mode != kEpiI32;
      const bool has_scale = g.col_scale != nullptr && g.mode != kEpiI32;
#pragma unroll
      for (int i = 0; i < kShare / 32; ++i) {
        const int n = nb_first + 32 * i + lane;
        // the argmax bias is padded with -inf to whole 256-column blocks
        const bool in = g.mode == kEpiArgmax || n < g.n;
        if (has_bias) sb[32 * i + lane] = in ? g.bias[n] : 0.0f;
        if (has_scale) ss[32 * i + lane] = n < g.n ? g.col_scale[n] : 0.0f;
      }
      __syncwarp();
      // Warp-uniform: tcgen05.ld below is .sync.aligned.
      const bool ready = __all_sync(0xffffffffu, mbar_wait(&tfull_bar[buf], (it >> 1) & 1, p.status));
      if (!ready) break;
      tc_fence_after();
      float best = -INFINITY;
      int best_n = -1;
      const uint32_t lane_base = tmem_base + buf * BN + (static_cast<uint32_t>(quarter * 32) << 16);
#pragma unroll 1
      for (int c0 = c_first; c0 < BN && c0 < (part + 1) * kShare; c0 += 32) {
        uint32_t r[32];
        tmem_ld_32x32b_x32(lane_base + c0, r);
        tmem_ld_wait();
        if (c.n0 + c0 < g.n)
          epilogue_chunk<BN, EPI>(g, r, row_ok && dest_row >= 0, row, dest_row, c.n0 + c0, row_scale,
                             p.status, best, best_n, stage, has_bias ? sb + (c0 - c_first) : nullptr,
                             has_scale ? ss + (c0 - c_first) : nullptr);
      }
      if (g.mode == kEpiArgmax && row_ok && dest_row >= 0 && best_n >= 0)
        atomicMax(&g.argmax[dest_row], pack_argmax(best, best_n));
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty_bar[buf]);
      ++it;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, 2 * BN);
  }
}

template <int BN>
constexpr int stage_bytes() {
  return kBM * kBK + BN * kBK;
}

int num_sms() {
  static int cached[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  dev &= 63;
  if (!cached[dev]) {
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    cached[dev] = n > 0 ? n : 148;
  }
  return cached[dev];
}

template <int BN, int MAX_STAGES, int EPI>
cudaError_t configure_impl() {
  static unsigned long long configured = 0;  // one bit per device ordinal
  int dev = 0;
  cudaGetDevice(&dev);
  if (!(configured & (1ull << (dev & 63)))) {
    cudaError_t e = cudaFuncSetAttribute(q8_gemm_kernel<BN, MAX_STAGES, EPI>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         MAX_STAGES * stage_bytes<BN>() + staging_bytes<EPI>() + 1024);
    if (e != cudaSuccess) return e;
    configured |= 1ull << (dev & 63);
  }
  return cudaSuccess;
}

template <int BN, int MAX_STAGES, int EPI>
cudaError_t launch_impl(GemmParams p, cudaStream_t stream) {
  auto kern = q8_gemm_kernel<BN, MAX_STAGES, EPI>;
  cudaError_t ce = configure_impl<BN, MAX_STAGES, EPI>();
  if (ce != cudaSuccess) return ce;
  const int num_kb = (p.k + kBK - 1) / kBK;
  const int tiles = ((p.max_n + BN - 1) / BN) * ((p.m + kBM - 1) / kBM) * p.num_groups;
  // Two CTAs per SM for the narrow tile when a 3-stage ring covers short K
  // and the tiles outnumber the SMs; with fewer tiles, one CTA per SM and a
  // ring as deep as K, so every k-block is requested at once (one load
  // round trip instead of two).
  int ctas_per_sm = 1;
  int stages = MAX_STAGES;
  if (BN == 64 && num_kb <= 4) {
    if (tiles > num_sms()) {
      stages = 3;
      ctas_per_sm = 2;
    } else {
      stages = num_kb < 3 ? 3 : num_kb;
    }
  }
  const int grid = tiles < num_sms() * ctas_per_sm ? tiles : num_sms() * ctas_per_sm;
  p.stages = stages;
  launch_pdl(kern, dim3(grid), dim3(threads_for<EPI>()),
             stages * stage_bytes<BN>() + staging_bytes<EPI>() + 1024, stream, p);
  return cudaGetLastError();
}

// ---- the vocabulary argmax, weight-stationary ---------------------------------
// The tied vocabulary projection (N = 32,000) with its masked argmax at
// decode row counts: the generic persistent kernel above loads both
// operands for every 128 x 256 tile (48 KB per k-block), and at 1,000 tiles
// over 148 CTAs that traffic, not the MMAs, sets its time.  Here each CTA
// keeps one 256-id block of the weight table resident in shared memory (all
// of K: 128 KB at d = 512) and streams the activations' 128-row blocks past
// it through a ring of 16 KB k-blocks, so a CTA loads 128 KB of weights and
// the activations once (640 KB in all at 1,024 rows, against ~1.3 MB per
// CTA for the tiled order).  Roles and the epilogue are the generic
// kernel's: warp 0 TMA, warp 1 TMEM + MMA (double-buffered accumulators, so
// one row block's epilogue overlaps the next one's MMAs), 16 epilogue warps
// with the masked-argmax epilogue.
constexpr int kArgBN = 256;
constexpr int kArgEpi = 16;
constexpr int kArgStages = 4;

template <int MAX_KB>
__global__ void __launch_bounds__(threads_for<kArgEpi>(), 1) q8_argmax_kernel(const __grid_constant__ GemmParams p) {
  constexpr int BN = kArgBN, EPI = kArgEpi;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int num_kb = (p.k + kBK - 1) / kBK;  // <= MAX_KB (checked by the launcher)
  uint8_t* smem_b = smem;                          // resident weights: num_kb x BN x 128 B
  uint8_t* smem_a = smem + MAX_KB * BN * kBK;      // activation ring: kArgStages x 16 KB
  __shared__ __align__(8) uint64_t full_bar[kArgStages];
  __shared__ __align__(8) uint64_t empty_bar[kArgStages];
  __shared__ __align__(8) uint64_t bfull_bar, bempty_bar;
  __shared__ __align__(8) uint64_t tfull_bar[2];
  __shared__ __align__(8) uint64_t tempty_bar[2];
  __shared__ uint32_t tmem_base_s;
  __shared__ __align__(16) float s_bias[EPI][64];
  __shared__ __align__(16) float s_scale[EPI][64];

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const GemmGroup& g = p.g[0];
  const int n_tiles = (p.max_n + BN - 1) / BN;
  pdl_enter();
  const int m_raw = p.m_dev ? *p.m_dev : p.m;
  if (threadIdx.x == 0) {
    for (int s = 0; s < kArgStages; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    mbar_init(&bfull_bar, 1);
    mbar_init(&bempty_bar, 1);
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull_bar[b], 1);
      mbar_init(&tempty_bar[b], EPI);
    }
    fence_barrier_init();
    tma_prefetch_desc(&g.tmap_a);
    tma_prefetch_desc(&g.tmap_b);
  }
  if (warp == 1) {
    tmem_alloc(&tmem_base_s, 2 * BN);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = tmem_base_s;
  const int m = max(0, min(m_raw, p.m));
  const int m_tiles = (m + kBM - 1) / kBM;

  if (warp == 0) {
    if (lane == 0) {
      const uint64_t keep = l2_policy_evict_last();  // weights: reused every step
      int kbg = 0, jt = 0;
      bool ok = true;
      for (int j = blockIdx.x; j < n_tiles && ok; j += gridDim.x, ++jt) {
        // the previous block's MMAs are done with the resident weights
        if (!(ok = mbar_wait(&bempty_bar, (jt & 1) ^ 1, p.status))) break;
        mbar_arrive_expect_tx(&bfull_bar, num_kb * BN * kBK);
        for (int kb = 0; kb < num_kb; ++kb)
          tma_load_2d_hint(smem_b + kb * BN * kBK, &g.tmap_b, kb * kBK, j * BN, &bfull_bar, keep);
        for (int mt = 0; mt < m_tiles && ok; ++mt)
          for (int kb = 0; kb < num_kb; ++kb, ++kbg) {
            const int s = kbg % kArgStages;
            const uint32_t phase = (kbg / kArgStages) & 1;
            if (!(ok = mbar_wait(&empty_bar[s], phase ^ 1, p.status))) break;
            mbar_arrive_expect_tx(&full_bar[s], kBM * kBK);
            tma_load_2d(smem_a + s * kBM * kBK, &g.tmap_a, kb * kBK, mt * kBM, &full_bar[s]);
          }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_i8(kBM, BN);
      int kbg = 0, it = 0, jt = 0;
      bool ok = true;
      for (int j = blockIdx.x; j < n_tiles && ok; j += gridDim.x, ++jt) {
        if (!(ok = mbar_wait(&bfull_bar, jt & 1, p.status))) break;
        for (int mt = 0; mt < m_tiles && ok; ++mt, ++it) {
          const int buf = it & 1;
          if (!(ok = mbar_wait(&tempty_bar[buf], ((it >> 1) & 1) ^ 1, p.status))) break;
          tc_fence_after();
          const uint32_t d_tmem = tmem_base + buf * BN;
          for (int kb = 0; kb < num_kb; ++kb, ++kbg) {
            const int s = kbg % kArgStages;
            const uint32_t phase = (kbg / kArgStages) & 1;
            if (!(ok = mbar_wait(&full_bar[s], phase, p.status))) break;
            tc_fence_after();
            const uint32_t a_addr = smem_u32(smem_a + s * kBM * kBK);
            const uint32_t b_addr = smem_u32(smem_b + kb * BN * kBK);
#pragma unroll
            for (int kk = 0; kk < kBK / 32; ++kk)
              mma_i8(d_tmem, sdesc_k_sw128(a_addr + kk * 32), sdesc_k_sw128(b_addr + kk * 32), idesc,
                     (kb > 0 || kk > 0) ? 1u : 0u);
            mma_commit(&empty_bar[s]);
          }
          if (ok) mma_commit(&tfull_bar[buf]);
        }
        if (ok) mma_commit(&bempty_bar);  // every MMA of this block has read the weights
      }
    }
  } else {
    // the generic kernel's epilogue in its argmax mode, per (row block, id block)
    const int quarter = warp & 3;
    const int part = (warp - 2) >> 2;
    constexpr int kShare = BN / (EPI / 4);  // 64 columns per warp
    float* sb = s_bias[warp - 2];
    float* ss = s_scale[warp - 2];
    const bool has_scale = g.col_scale != nullptr;
    int it = 0;
    bool ok = true;
    for (int j = blockIdx.x; j < n_tiles && ok; j += gridDim.x) {
      const int n0 = j * BN;
      const int nb_first = n0 + part * kShare;
      // this block's bias (-inf padded past N) and column scales for the warp
#pragma unroll
      for (int i = 0; i < kShare / 32; ++i) {
        const int n = nb_first + 32 * i + lane;
        sb[32 * i + lane] = g.bias ? g.bias[n] : 0.0f;
        if (has_scale) ss[32 * i + lane] = n < g.n ? g.col_scale[n] : 0.0f;
      }
      __syncwarp();
      for (int mt = 0; mt < m_tiles; ++mt, ++it) {
        const int buf = it & 1;
        const int row = mt * kBM + quarter * 32 + lane;
        const bool row_ok = row < m;
        const bool ready = __all_sync(0xffffffffu, mbar_wait(&tfull_bar[buf], (it >> 1) & 1, p.status));
        if (!ready) {
          ok = false;
          break;
        }
        tc_fence_after();
        float best = -INFINITY;
        int best_n = -1;
        const uint32_t lane_base = tmem_base + buf * BN + (static_cast<uint32_t>(quarter * 32) << 16);
#pragma unroll 1
        for (int c0 = part * kShare; c0 < (part + 1) * kShare; c0 += 32) {
          uint32_t r[32];
          tmem_ld_32x32b_x32(lane_base + c0, r);
          tmem_ld_wait();
          if (n0 + c0 < g.n)
            epilogue_chunk<BN, EPI>(g, r, row_ok, row, row, n0 + c0, 1.0f, p.status, best, best_n, nullptr,
                               g.bias ? sb + (c0 - part * kShare) : nullptr,
                               has_scale ? ss + (c0 - part * kShare) : nullptr);
        }
        if (row_ok && best_n >= 0) atomicMax(&g.argmax[row], pack_argmax(best, best_n));
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&tempty_bar[buf]);
      }
      __syncwarp();  // the staged bias is rewritten for the next block
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, 2 * BN);
  }
}

template <int MAX_KB>
constexpr int argmax_smem_bytes() {
  return MAX_KB * kArgBN * kBK + kArgStages * kBM * kBK + 1024;
}

template <int MAX_KB>
cudaError_t configure_argmax() {
  static unsigned long long configured = 0;  // one bit per device ordinal
  int dev = 0;
  cudaGetDevice(&dev);
  if (!(configured & (1ull << (dev & 63)))) {
    cudaError_t e = cudaFuncSetAttribute(q8_argmax_kernel<MAX_KB>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         argmax_smem_bytes<MAX_KB>());
    if (e != cudaSuccess) return e;
    configured |= 1ull << (dev & 63);
  }
  return cudaSuccess;
}

cudaError_t launch_argmax(const GemmParams& p, cudaStream_t stream) {
  constexpr int MAX_KB = 4;
  cudaError_t e = configure_argmax<MAX_KB>();
  if (e != cudaSuccess) return e;
  const int n_tiles = (p.max_n + kArgBN - 1) / kArgBN;
  const int grid = n_tiles < num_sms() ? n_tiles : num_sms();
  launch_pdl(q8_argmax_kernel<MAX_KB>, dim3(grid), dim3(threads_for<kArgEpi>()), argmax_smem_bytes<MAX_KB>(),
             stream, p);
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

bool encode_tmap_kv(CUtensorMap* map, const float* base, uint64_t rows, int d, int page_tokens,
                    int group_cols, int box_rows) {
  auto fn = encode_fn();
  if (!fn || !base || rows == 0 || d % 32 != 0 || group_cols % 32 != 0 || page_tokens <= 0 ||
      page_tokens % 8 != 0 || group_cols / 32 > 256 || (reinterpret_cast<uintptr_t>(base) & 15) != 0 ||
      (box_rows != 8 && box_rows != 4 && box_rows != 2 && box_rows != 1))
    return false;
  cuuint64_t dims[3] = {32, rows, static_cast<cuuint64_t>(d / 32)};
  cuuint64_t strides[2] = {static_cast<cuuint64_t>(d) * 4, 128};
  cuuint32_t box[3] = {32, static_cast<cuuint32_t>(box_rows), static_cast<cuuint32_t>(group_cols / 32)};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, const_cast<float*>(base), dims, strides, box,
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

cudaError_t prepare_q8_gemm() {
  num_sms();
  cudaError_t e = configure_impl<256, 3, 16>();
  if (e == cudaSuccess) e = configure_impl<128, 4, 16>();
  if (e == cudaSuccess) e = configure_impl<64, 7, 8>();
  if (e == cudaSuccess) e = configure_argmax<4>();
  return e;
}

cudaError_t launch_q8_gemm(const GemmParams& p, int bn, cudaStream_t stream) {
  if (p.m <= 0 || p.num_groups <= 0) return cudaSuccess;
  // a single vocabulary argmax with K <= 512: the weight-stationary kernel
  // (its tensor map has the BN = 256 box)
  if (bn == 256 && p.num_groups == 1 && p.g[0].mode == kEpiArgmax && p.k <= 4 * kBK && !p.g[0].row_map &&
      !p.g[0].row_scale)
    return launch_argmax(p, stream);
  switch (bn) {
    case 256: return launch_impl<256, 3, 16>(p, stream);
    case 128: return launch_impl<128, 4, 16>(p, stream);
    default: return launch_impl<64, 7, 8>(p, stream);
  }
}

}  // namespace mc
