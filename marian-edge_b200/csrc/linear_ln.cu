// linear_ln.cu -- a Q8 linear fused with the residual add and the LayerNorm
// that follow it in every Transformer sub-layer: Q8Linear::run_into
// (crates/marian-cpu/src/q8_gemm.rs:380-448) writes acc * scale + bias, and
// residual_layer_norm_into (tensor.rs:132-155, normalize_row 372-385) forms
// x = linear + residual, mean = sum(x) / d, var = sum((x - mean)^2) / d with
// both sums left to right, and (x - mean) * (1 / sqrt(var + eps)) * gamma +
// beta.  The quantized copies of the result for the next linears
// (quantize_symmetric_u8_into, q8_gemm.rs:609-617) are written too.
//
// The LayerNorm needs whole rows, and its two sums are serial chains over
// all d columns, so the work is split by rows AND columns: a cluster of C
// CTAs (8 for d = 512) owns one 128-row block, CTA j computing output
// columns [j * d / C, (j + 1) * d / C) on the tensor cores:
//   warp 0      TMA producer (A and W k-blocks into a ring, 128-byte
//               swizzle), started before the TMEM allocation;
//   warp 1      TMEM allocation and tcgen05.mma.kind::i8 from one thread;
//   warps 2..9  epilogue, two per TMEM lane quarter (one row per thread,
//               alternate 32-column chunks): x = (acc * scale + bias) +
//               residual, the residual values having been loaded into
//               registers while the MMAs ran.
// Each CTA also owns 128 / C rows of the block for the normalization.  The
// epilogue writes each row's x segment either into the CTA's own exchange
// buffer (its own rows) or, grouped by owner, into the idle TMA ring; one
// bulk copy per owner (cp.async.bulk shared::cta -> shared::cluster) then
// moves each group into the owner's exchange buffer and completes its bytes
// on the owner's mbarrier.  Once all d columns of its rows have arrived, one
// thread per row runs the two ordered sums, and every warp of the CTA
// normalizes the rows with coalesced row-wise stores of the f32 result and
// its int8 copies.  Every mbarrier wait is bounded; the cluster barriers are
// passed by every thread of every CTA on every path.
#include "common.cuh"
#include "linear_ln.cuh"
#include "q8_gemm.cuh"

namespace mc {

namespace {

constexpr int kLlBM = 128;        // rows per cluster
constexpr int kLlBK = 128;        // K bytes per stage
constexpr int kLlEpiWarps = 8;    // two per TMEM lane quarter

// Threads per CTA: the producer, MMA and 8 epilogue warps, plus warps that
// only join the row passes (latency-bound: more warps in flight help);
// 384 for d = 384, whose epilogue needs more registers per thread.
template <int D>
__host__ __device__ constexpr int ll_threads() {
  return D == 384 ? 384 : 512;
}
constexpr int kLlMaxStages = 6;
constexpr float kLlEps = 1.0e-6f;  // tensor.rs:3

__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

// All threads of all CTAs of the cluster (release / acquire at cluster scope).
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile(
      "barrier.cluster.arrive.release.aligned;\n\t"
      "barrier.cluster.wait.acquire.aligned;" ::
          : "memory");
}

// This CTA's shared-memory address -> the same offset in CTA `rank`.
__device__ __forceinline__ uint32_t map_shared_rank(uint32_t addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
  return r;
}

// Bounded wait with acquire semantics at cluster scope: the bytes that
// completed the phase were written by other CTAs of the cluster.
__device__ __forceinline__ bool mbar_wait_cluster(uint64_t* bar, uint32_t phase, uint32_t* status) {
  for (uint32_t i = 0; i < kSpinLimit; ++i) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(phase)
        : "memory");
    if (ok) return true;
  }
  flag_status(status, kStatusWaitTimeout);
  return false;
}

// quantize_one (common.cuh) for four values and every copy, the result in
// the low byte; a non-finite value is reported once for the four.
__device__ __forceinline__ int quant_s8(float v, float alpha) {
  return quantize_low_byte(v, alpha);
}

__device__ __forceinline__ void store_copies(const QuantOut& q, long long elem, float4 v,
                                             uint32_t* status) {
  constexpr float kMax = 3.402823466e38f;
  if (!(fabsf(v.x) <= kMax) || !(fabsf(v.y) <= kMax) || !(fabsf(v.z) <= kMax) || !(fabsf(v.w) <= kMax))
    flag_status(status, kStatusNonFinite);
  for (int i = 0; i < q.count; ++i) {
    const float al = q.alpha[i];
    const uint32_t lo = __byte_perm((uint32_t)quant_s8(v.x, al), (uint32_t)quant_s8(v.y, al), 0x0040);
    const uint32_t hi = __byte_perm((uint32_t)quant_s8(v.z, al), (uint32_t)quant_s8(v.w, al), 0x0040);
    *reinterpret_cast<uint32_t*>(q.base + i * q.stride + elem) = __byte_perm(lo, hi, 0x5410);
  }
}

template <int D, int C>
struct LlShape {
  static constexpr int BN = D / C;           // output columns per CTA
  static constexpr int R = kLlBM / C;        // rows each CTA normalizes
  static constexpr int SLD = BN + 4;         // row stride of a column segment (floats)
  static constexpr int XSEG = R * SLD;       // one CTA's columns of R rows (floats)
  static constexpr int TCOLS = BN <= 32 ? 32 : (BN <= 64 ? 64 : 128);  // TMEM columns
  static constexpr int STAGE = kLlBM * kLlBK + BN * kLlBK;
  static constexpr int XBYTES = C * XSEG * 4;       // the incoming rows
  static constexpr int STAGING = C * XSEG * 4;      // outgoing segments (in the ring)
  static constexpr int MIN_STAGES = (STAGING + STAGE - 1) / STAGE;
  // second linear (proj): its A operand, the block's 128 normalized rows
  // quantized, K = d in 128-byte k-blocks ([k-block][128 rows][128 B],
  // 128-byte swizzle), and this CTA's rows of it staged for the peers
  // ([k-block][R rows][128 B]) -- both in the idle ring after the outgoing
  // segments; W2's [k-block][BN rows][128 B] after the exchange buffer.
  static constexpr int KB2 = D / 128;
  static constexpr int A2_OFF = (STAGING + 1023) / 1024 * 1024;
  static constexpr int OUT_OFF = A2_OFF + KB2 * 16384;
  static constexpr int PROJ_END = OUT_OFF + KB2 * R * 128;
  static constexpr int MIN_STAGES_PROJ = (PROJ_END + STAGE - 1) / STAGE;
  static constexpr int XBYTES_AL = (XBYTES + 1023) / 1024 * 1024;
  static_assert(D % 128 == 0 && BN % 32 == 0 && BN <= 128 && kLlBM % C == 0 && R <= 32 && R >= 8,
                "unsupported fused LayerNorm shape");
  static_assert((XSEG * 4) % 16 == 0, "bulk copies move 16-byte multiples");
};

// Second-linear variants: PK = 0 none, 1 a d-wide f32 linear (the
// cross-attention query), 2 the FFN's first linear (4d wide, ReLU, int8
// output quantized for the second).
template <int D, int C, int PK>
struct LlPlan {
  using S = LlShape<D, C>;
  static constexpr int BN2 = PK == 2 ? 4 * S::BN : S::BN;     // second-linear columns per CTA
  static constexpr int CHUNK = BN2 * 128;                     // one k-block of its weights
  // resident weight k-blocks: all of them (PK 1); two, with k-block 2 loaded
  // into the exchange buffer once it is read and k-block 3 into the ring's
  // outgoing segments once they are delivered (PK 2)
  static constexpr int B2_RES = PK == 0 ? 0 : (PK == 1 ? S::KB2 * CHUNK : 2 * CHUNK);
  static constexpr int TC1 = S::TCOLS;
  static constexpr int TCOLS = PK == 0 ? TC1 : (S::BN + BN2 <= 64 ? 64 : (S::BN + BN2 <= 128 ? 128 : (S::BN + BN2 <= 256 ? 256 : 512)));
  static_assert(PK != 2 || (S::KB2 <= 4 && BN2 <= 256 && S::XBYTES_AL >= CHUNK && S::STAGING >= CHUNK),
                "FFN projection shape");
};

template <int D, int C, int PK>
constexpr int ll_smem_bytes(int stages) {
  using S = LlShape<D, C>;
  return stages * S::STAGE + S::XBYTES_AL + LlPlan<D, C, PK>::B2_RES + 1024;
}

// Ring depth: up to kLlMaxStages within the dynamic shared memory that the
// static arrays leave of the 227 KB per-CTA limit.
template <int D, int C, int PK>
constexpr int ll_max_stages() {
  using S = LlShape<D, C>;
  constexpr int budget = (PK == 2 ? 220 : 218) * 1024;
  constexpr int fit = (budget - S::XBYTES_AL - LlPlan<D, C, PK>::B2_RES - 1024) / S::STAGE;
  return fit < kLlMaxStages ? fit : kLlMaxStages;
}

template <int D, int C, int PK>
constexpr int ll_min_stages() {
  using S = LlShape<D, C>;
  return PK != 0 && S::MIN_STAGES_PROJ > S::MIN_STAGES ? S::MIN_STAGES_PROJ : S::MIN_STAGES;
}

// Bulk copy of `bytes` from this CTA's shared memory to a cluster peer's,
// completing them on the peer's mbarrier (both peer addresses from mapa).
__device__ __forceinline__ void bulk_copy_to_peer(uint32_t dst, const void* src, uint32_t bytes,
                                                  uint32_t bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.shared::cta.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
      "r"(smem_u32(src)), "r"(bytes), "r"(bar)
      : "memory");
}

// A row's left-to-right sum over the C column segments of a buffer laid out
// [segment][row][SLD]: batches of eight 16-byte loads and their 32
// dependent adds, four batches unrolled so the loads of the next batches
// are issued while the adds run (4.4 cycles per add on B200, against 4.2
// for a chain held in registers).
// The same order over the centred squares (x - mean) * (x - mean), the
// reference's `var += c * c` with two roundings (about 6 cycles per add:
// the subtract and multiply issue between the dependent adds).
template <int D, int C>
__device__ __forceinline__ float ordered_sq_sum(const float* seg0, float mean) {
  using S = LlShape<D, C>;
  constexpr int kPerSeg = S::BN / 32;
  float sum = 0.0f;
#pragma unroll 4
  for (int bt = 0; bt < D / 32; ++bt) {
    const float4* r4 = reinterpret_cast<const float4*>(seg0 + (bt / kPerSeg) * S::XSEG) + 8 * (bt % kPerSeg);
    float4 v[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) v[u] = r4[u];
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const float c0 = __fsub_rn(v[u].x, mean), c1 = __fsub_rn(v[u].y, mean);
      const float c2 = __fsub_rn(v[u].z, mean), c3 = __fsub_rn(v[u].w, mean);
      sum = __fadd_rn(sum, __fmul_rn(c0, c0));
      sum = __fadd_rn(sum, __fmul_rn(c1, c1));
      sum = __fadd_rn(sum, __fmul_rn(c2, c2));
      sum = __fadd_rn(sum, __fmul_rn(c3, c3));
    }
  }
  return sum;
}

template <int D, int C>
__device__ __forceinline__ float ordered_row_sum(const float* seg0) {
  using S = LlShape<D, C>;
  constexpr int kPerSeg = S::BN / 32;  // 8-float4 batches per segment
  float sum = 0.0f;
#pragma unroll 4
  for (int bt = 0; bt < D / 32; ++bt) {
    const float4* r4 = reinterpret_cast<const float4*>(seg0 + (bt / kPerSeg) * S::XSEG) + 8 * (bt % kPerSeg);
    float4 v[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) v[u] = r4[u];
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      sum = __fadd_rn(sum, v[u].x);
      sum = __fadd_rn(sum, v[u].y);
      sum = __fadd_rn(sum, v[u].z);
      sum = __fadd_rn(sum, v[u].w);
    }
  }
  return sum;
}

template <int D, int C, int PK>
__global__ void __launch_bounds__(ll_threads<D>(), 1) q8_linear_ln_kernel(const __grid_constant__ LinearLnParams p) {
  using S = LlShape<D, C>;
  using P = LlPlan<D, C, PK>;
  constexpr bool PROJ = PK != 0;
  constexpr int TCOLS = P::TCOLS;  // the second linear's accumulator at column BN
  constexpr int BN2 = P::BN2;
  constexpr int BN = S::BN, R = S::R, SLD = S::SLD, XSEG = S::XSEG;
  constexpr int kLlThreads = ll_threads<D>();
  constexpr int CHUNKS = BN / 32;                 // 32-column TMEM chunks per tile row
  constexpr int MY_CHUNKS = (CHUNKS + 1) / 2;     // per epilogue warp (two warps per lane quarter)
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int stages = p.stages;
  uint8_t* smem_a = smem;                              // stages x 16 KB
  uint8_t* smem_b = smem + stages * kLlBM * kLlBK;     // stages x BN * 128
  // After the last MMA the ring holds the outgoing segments [owner][R][SLD].
  float* staging = reinterpret_cast<float*>(smem);
  // Incoming rows [source CTA][R][SLD].
  float* xbuf = reinterpret_cast<float*>(smem_b + stages * BN * kLlBK);
  uint8_t* a2 = smem + S::A2_OFF;                       // proj: its A operand
  uint8_t* a2_out = smem + S::OUT_OFF;                  // proj: this CTA's rows of it
  uint8_t* b2 = reinterpret_cast<uint8_t*>(xbuf) + S::XBYTES_AL;  // proj: W2's resident k-blocks
  // k-block kb of the second linear's weights (PK 2: k-block 2 reuses the
  // exchange buffer, k-block 3 the ring's outgoing segments)
  auto b2_chunk = [&](int kb) -> uint8_t* {
    if (PK == 2 && kb == 2) return reinterpret_cast<uint8_t*>(xbuf);
    if (PK == 2 && kb == 3) return smem;
    return b2 + kb * P::CHUNK;
  };
  __shared__ __align__(8) uint64_t full_bar[kLlMaxStages];
  __shared__ __align__(8) uint64_t empty_bar[kLlMaxStages];
  __shared__ __align__(8) uint64_t tfull_bar;
  __shared__ __align__(8) uint64_t x_bar;
  __shared__ __align__(8) uint64_t b2_bar[4], a2_bar, t2_bar;  // proj
  __shared__ uint32_t tmem_base_s;
  __shared__ __align__(16) float s_bias[BN];
  __shared__ __align__(16) float s_scale[BN];
  __shared__ __align__(16) float s_gamma[D];
  __shared__ __align__(16) float s_beta[D];
  __shared__ float s_mean[R];
  __shared__ float s_inv[R];
  __shared__ __align__(16) float s_bias2[PROJ ? BN2 : 1];
  __shared__ __align__(16) float s_scale2[PK == 1 ? BN2 : 1];  // PK 2: read from global when per column

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const int n0 = static_cast<int>(rank) * BN;
  const int row0 = blockIdx.y * kLlBM;

  // Weights are never written by a kernel: staged before the dependency wait.
  for (int i = threadIdx.x; i < D; i += kLlThreads) {
    s_gamma[i] = p.gamma[i];
    s_beta[i] = p.beta[i];
  }
  if (threadIdx.x < BN) {
    s_bias[threadIdx.x] = p.bias ? p.bias[n0 + threadIdx.x] : 0.0f;
    s_scale[threadIdx.x] = p.col_scale ? p.col_scale[n0 + threadIdx.x] : p.uniform_scale;
  }
  const int n0_2 = static_cast<int>(rank) * BN2;  // the second linear's first column
  if constexpr (PROJ) {
    for (int i = threadIdx.x; i < BN2; i += kLlThreads) {
      s_bias2[i] = p.bias2 ? p.bias2[n0_2 + i] : 0.0f;
      if constexpr (PK == 1) s_scale2[i] = p.col_scale2 ? p.col_scale2[n0_2 + i] : p.uniform_scale2;
    }
  }
  if (threadIdx.x == 0) {
    for (int s = 0; s < stages; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    mbar_init(&tfull_bar, 1);
    mbar_init(&x_bar, 1);
    // the owner's own arrival: the phase completes when the other C - 1
    // CTAs' segments of its R rows have landed (its own are plain stores)
    mbar_arrive_expect_tx(&x_bar, static_cast<uint32_t>((C - 1) * XSEG * 4));
    if constexpr (PROJ) {
      for (int i = 0; i < 4; ++i) mbar_init(&b2_bar[i], 1);
      mbar_init(&a2_bar, 1);
      // the other C - 1 CTAs' R quantized rows of every k-block
      mbar_arrive_expect_tx(&a2_bar, static_cast<uint32_t>((C - 1) * S::KB2 * R * 128));
      mbar_init(&t2_bar, 1);
      tma_prefetch_desc(&p.tmap_b2);
    }
    fence_barrier_init();
    tma_prefetch_desc(&p.tmap_a);
    tma_prefetch_desc(&p.tmap_b);
  }
  // Every CTA's exchange barrier is initialized before any peer can write.
  cluster_sync_all();
  pdl_enter();
  const int m = max(0, min(p.m_dev ? *p.m_dev : p.cap, p.cap));
  if (row0 >= m) return;  // the whole cluster shares row0 and leaves together

  const int num_kb = (p.k + kLlBK - 1) / kLlBK;
  if (warp == 0) {
    // TMA producer: needs only the ring's barriers, so it starts while the
    // other warps allocate TMEM and load their residual values.
    if (lane == 0) {
      const uint64_t keep = l2_policy_evict_last();  // weights: reused every step
      for (int kb = 0; kb < num_kb; ++kb) {
        const int s = kb % stages;
        const uint32_t phase = (kb / stages) & 1;
        if (!mbar_wait(&empty_bar[s], phase ^ 1, p.status)) break;
        mbar_arrive_expect_tx(&full_bar[s], S::STAGE);
        tma_load_2d(smem_a + s * kLlBM * kLlBK, &p.tmap_a, kb * kLlBK, row0, &full_bar[s]);
        tma_load_2d_hint(smem_b + s * BN * kLlBK, &p.tmap_b, kb * kLlBK, n0, &full_bar[s], keep);
      }
      if constexpr (PROJ) {  // the second linear's resident k-blocks, needed after the LayerNorm
        for (int kb = 0; kb < (PK == 2 ? (S::KB2 < 2 ? S::KB2 : 2) : S::KB2); ++kb) {
          mbar_arrive_expect_tx(&b2_bar[kb], P::CHUNK);
          tma_load_2d_hint(b2_chunk(kb), &p.tmap_b2, kb * kLlBK, n0_2, &b2_bar[kb], keep);
        }
      }
    }
  }

  uint32_t tmem_base = 0;
  if (warp != 0) {
    if (warp == 1) {
      tmem_alloc(&tmem_base_s, TCOLS);
      tmem_relinquish();
    }
    tc_fence_before();
    asm volatile("bar.sync 1, %0;" ::"n"(kLlThreads - 32) : "memory");  // every warp but 0
    tc_fence_after();
    tmem_base = tmem_base_s;
  }

  // Epilogue warps 2..9: tile row t (TMEM lane t); the warp's half h takes
  // the 32-column chunks h, h + 2, ... of the row.  Its residual values are
  // loaded while the MMAs run (after the barrier above, which would
  // otherwise wait for them).
  const bool epi = warp >= 2 && warp < 2 + kLlEpiWarps;
  const int quarter = warp & 3;
  const int half = (warp - 2) >> 2;
  const int t = quarter * 32 + lane;
  const int row = row0 + t;
  const bool row_ok = epi && row < m;
  float res[MY_CHUNKS * 32];
  if (epi) {
    const float* rp = p.residual + (size_t)(row_ok ? row : 0) * p.ldr + n0;
#pragma unroll
    for (int i = 0; i < MY_CHUNKS; ++i) {
      const int c0 = 32 * (half + 2 * i);
#pragma unroll
      for (int j4 = 0; j4 < 8; ++j4) {
        const float4 v = (row_ok && c0 < BN) ? *reinterpret_cast<const float4*>(rp + c0 + 4 * j4)
                                             : make_float4(0.f, 0.f, 0.f, 0.f);
        res[32 * i + 4 * j4 + 0] = v.x;
        res[32 * i + 4 * j4 + 1] = v.y;
        res[32 * i + 4 * j4 + 2] = v.z;
        res[32 * i + 4 * j4 + 3] = v.w;
      }
    }
  }
  bool ready = true;

  if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_i8(kLlBM, BN);
      bool ok = true;
      for (int kb = 0; kb < num_kb; ++kb) {
        const int s = kb % stages;
        const uint32_t phase = (kb / stages) & 1;
        if (!(ok = mbar_wait(&full_bar[s], phase, p.status))) break;
        tc_fence_after();
        const uint32_t a_addr = smem_u32(smem_a + s * kLlBM * kLlBK);
        const uint32_t b_addr = smem_u32(smem_b + s * BN * kLlBK);
#pragma unroll
        for (int kk = 0; kk < kLlBK / 32; ++kk)
          mma_i8(tmem_base, sdesc_k_sw128(a_addr + kk * 32), sdesc_k_sw128(b_addr + kk * 32), idesc,
                 (kb > 0 || kk > 0) ? 1u : 0u);
        mma_commit(&empty_bar[s]);
      }
      if (ok) mma_commit(&tfull_bar);
    }
  } else if (epi) {
    // ---- x = (acc * scale + bias) + residual for row t, by owner ----
    // Row t belongs to owner t / R: this CTA's own rows go straight into
    // its exchange buffer, the others into the (now idle) ring, one
    // contiguous segment per owner, sent below with one bulk copy each.
    const int owner = t / R;
    float* dst = (owner == static_cast<int>(rank) ? xbuf + rank * XSEG : staging + owner * XSEG) + (t % R) * SLD;
    ready = __all_sync(0xffffffffu, mbar_wait(&tfull_bar, 0, p.status));
    if (ready) {
      tc_fence_after();
      fence_proxy_async_smem();  // the ring was last written by TMA
      const uint32_t lane_base = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16);
#pragma unroll
      for (int i = 0; i < MY_CHUNKS; ++i) {
        const int c0 = 32 * (half + 2 * i);
        if (c0 >= BN) break;
        uint32_t r[32];
        tmem_ld_32x32b_x32(lane_base + c0, r);
        tmem_ld_wait();
#pragma unroll
        for (int j4 = 0; j4 < 8; ++j4) {
          float x[4];
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            const int j = 4 * j4 + u;
            x[u] = __fadd_rn(dequant(static_cast<int32_t>(r[j]), s_scale[c0 + j], s_bias[c0 + j]), res[32 * i + j]);
          }
          *reinterpret_cast<float4*>(dst + c0 + 4 * j4) = make_float4(x[0], x[1], x[2], x[3]);
        }
      }
      fence_proxy_async_smem();  // the segments are read by the bulk copies
    }
    // The two warps of this lane quarter (halves 0 and 1) have written their
    // rows' segments; the half-0 warp sends the quarter's remote ones.
    asm volatile("bar.sync %0, 64;" ::"r"(2 + quarter) : "memory");
    if (half == 0 && lane == 0 && ready) {
      for (int o = (quarter * 32) / R; o <= (quarter * 32 + 31) / R; ++o) {
        if (o == static_cast<int>(rank)) continue;
        const uint32_t peer_dst = map_shared_rank(smem_u32(xbuf + rank * XSEG), o);
        const uint32_t peer_bar = map_shared_rank(smem_u32(&x_bar), o);
        bulk_copy_to_peer(peer_dst, staging + o * XSEG, XSEG * 4, peer_bar);
      }
    }
  }
  // ---- owner: the R rows [rank * R, rank * R + R) of the block ----
  // Every warp: the CTA's own segment of its rows is in place; the others
  // are visible to every thread once it has observed the phase.
  __syncthreads();
  const bool got = mbar_wait_cluster(&x_bar, 0, p.status) && ready;
  // Everything bound for this CTA has arrived: its peers may leave once
  // every CTA has said so (the matching wait ends the kernel), so no bulk
  // copy ever reads from or writes to an exited CTA.  (With a projection
  // the quantized rows arrive later; the arrival waits for them.)
  if constexpr (!PROJ) asm volatile("barrier.cluster.arrive.relaxed;" ::: "memory");
  constexpr int kVec = D / 4;
  constexpr int SEGV = BN / 4;  // float4 per row segment
  const float fd = static_cast<float>(D);
  const int rows_here = max(0, min(R, m - (row0 + static_cast<int>(rank) * R)));
  if (warp == 2 && lane < R)  // normalize_row's first left-to-right sum, one thread per row
    s_mean[lane] = ordered_row_sum<D, C>(xbuf + lane * SLD) / fd;
  __syncthreads();
  if (warp == 2 && lane < R) {  // the second sum: var = sum((x - mean)^2) / d
    const float var = ordered_sq_sum<D, C>(xbuf + lane * SLD, s_mean[lane]) / fd;
    s_inv[lane] = 1.0f / sqrtf(var + kLlEps);
  }
  __syncthreads();
  if (got) {
    // thread -> one float4 column, rows i0, i0 + kGroups, ...
    constexpr int kGroups = kLlThreads / kVec;
    static_assert(kLlThreads % kVec == 0, "row pass assumes whole row groups");
    const int c4 = threadIdx.x % kVec;
    const int i0 = threadIdx.x / kVec;
    const int coff = (c4 / SEGV) * XSEG + 4 * (c4 % SEGV);
    const float4 g = reinterpret_cast<const float4*>(s_gamma)[c4];
    const float4 b = reinterpret_cast<const float4*>(s_beta)[c4];
#pragma unroll 2
    for (int i = i0; i < rows_here; i += kGroups) {
      const int grow = row0 + static_cast<int>(rank) * R + i;
      const float inv = s_inv[i], mean = s_mean[i];
      const float4 xv = *reinterpret_cast<const float4*>(xbuf + coff + i * SLD);
      const float4 c = make_float4(__fsub_rn(xv.x, mean), __fsub_rn(xv.y, mean), __fsub_rn(xv.z, mean),
                                   __fsub_rn(xv.w, mean));
      float4 v;
      v.x = __fadd_rn(__fmul_rn(__fmul_rn(c.x, inv), g.x), b.x);
      v.y = __fadd_rn(__fmul_rn(__fmul_rn(c.y, inv), g.y), b.y);
      v.z = __fadd_rn(__fmul_rn(__fmul_rn(c.z, inv), g.z), b.z);
      v.w = __fadd_rn(__fmul_rn(__fmul_rn(c.w, inv), g.w), b.w);
      const long long elem = (long long)grow * D + 4 * c4;
      *reinterpret_cast<float4*>(p.out + elem) = v;
      store_copies(p.q, elem, v, p.status);
      if constexpr (PROJ) {
        // quantize_one for W2 (finiteness reported by store_copies' test
        // when q has copies, else here), into A2 row rank * R + i and the
        // staged copy for the peers, both 128-byte swizzled
        if (p.q.count == 0 && (!(fabsf(v.x) <= 3.402823466e38f) || !(fabsf(v.y) <= 3.402823466e38f) ||
                               !(fabsf(v.z) <= 3.402823466e38f) || !(fabsf(v.w) <= 3.402823466e38f)))
          flag_status(p.status, kStatusNonFinite);
        const uint32_t lo = __byte_perm((uint32_t)quant_s8(v.x, p.alpha2), (uint32_t)quant_s8(v.y, p.alpha2), 0x0040);
        const uint32_t hi = __byte_perm((uint32_t)quant_s8(v.z, p.alpha2), (uint32_t)quant_s8(v.w, p.alpha2), 0x0040);
        const uint32_t word = __byte_perm(lo, hi, 0x5410);
        const int byte = 4 * c4, kb = byte >> 7, cc = byte & 127;
        const int t2 = static_cast<int>(rank) * R + i;  // the row in the block
        *reinterpret_cast<uint32_t*>(a2 + kb * 16384 + t2 * 128 + ((((cc >> 4) ^ (t2 & 7))) << 4) + (cc & 15)) = word;
        *reinterpret_cast<uint32_t*>(a2_out + kb * (R * 128) + i * 128 + ((((cc >> 4) ^ (i & 7))) << 4) + (cc & 15)) =
            word;
      }
    }
  }
  if constexpr (PROJ) {
    // ---- the second linear: exchange the quantized rows, MMA, epilogue ----
    fence_proxy_async_smem();  // A2, the staged rows and the read exchange buffer
    __syncthreads();
    // one thread per (peer, k-block) piece issues its bulk copy
    constexpr int kPieces = (C - 1) * S::KB2;
    static_assert(kPieces < kLlThreads, "one thread per outgoing piece");
    if (threadIdx.x < kPieces && got) {
      const int j = threadIdx.x / S::KB2, kb = threadIdx.x % S::KB2;
      const int o = j < static_cast<int>(rank) ? j : j + 1;
      bulk_copy_to_peer(map_shared_rank(smem_u32(a2 + kb * 16384 + static_cast<int>(rank) * R * 128), o),
                        a2_out + kb * (R * 128), R * 128, map_shared_rank(smem_u32(&a2_bar), o));
    }
    const uint64_t keep = l2_policy_evict_last();
    if (PK == 2 && S::KB2 > 2 && threadIdx.x == kPieces) {
      // the exchange buffer has been read: weight k-block 2 goes there
      mbar_arrive_expect_tx(&b2_bar[2], P::CHUNK);
      tma_load_2d_hint(b2_chunk(2), &p.tmap_b2, 2 * kLlBK, n0_2, &b2_bar[2], keep);
    }
    const bool got2 = mbar_wait_cluster(&a2_bar, 0, p.status) && got;
    asm volatile("barrier.cluster.arrive.relaxed;" ::: "memory");  // see above
    if (PK == 2 && S::KB2 > 3 && threadIdx.x == kPieces) {
      // every peer has received this CTA's outgoing segments (they sent
      // their quantized rows after that): weight k-block 3 goes there
      mbar_arrive_expect_tx(&b2_bar[3], P::CHUNK);
      tma_load_2d_hint(b2_chunk(3), &p.tmap_b2, 3 * kLlBK, n0_2, &b2_bar[3], keep);
    }
    if (warp == 1 && lane == 0 && got2) {
      constexpr uint32_t idesc = idesc_i8(kLlBM, BN2);
      bool ok = true;
      for (int kb = 0; kb < S::KB2 && ok; ++kb) {
        if (!(ok = mbar_wait(&b2_bar[kb], 0, p.status))) break;
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < kLlBK / 32; ++kk)
          mma_i8(tmem_base + BN, sdesc_k_sw128(smem_u32(a2 + kb * 16384) + kk * 32),
                 sdesc_k_sw128(smem_u32(b2_chunk(kb)) + kk * 32), idesc, (kb > 0 || kk > 0) ? 1u : 0u);
      }
      if (ok) mma_commit(&t2_bar);
    }
    if (epi) {
      const bool ready2 = __all_sync(0xffffffffu, mbar_wait(&t2_bar, 0, p.status));
      if (ready2) {
        tc_fence_after();
        const uint32_t lane_base = tmem_base + BN + (static_cast<uint32_t>(quarter * 32) << 16);
        if constexpr (PK == 1) {
          float* orow = p.out2 + (size_t)(row_ok ? row : 0) * p.ldo2 + n0_2;
#pragma unroll
          for (int i = 0; i < MY_CHUNKS; ++i) {
            const int c0 = 32 * (half + 2 * i);
            if (c0 >= BN2) break;
            uint32_t r[32];
            tmem_ld_32x32b_x32(lane_base + c0, r);
            tmem_ld_wait();
            if (row_ok) {
#pragma unroll
              for (int j4 = 0; j4 < 8; ++j4) {
                float y[4];
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                  const int j = 4 * j4 + u;
                  y[u] = dequant(static_cast<int32_t>(r[j]), s_scale2[c0 + j], s_bias2[c0 + j]);
                }
                *reinterpret_cast<float4*>(orow + c0 + 4 * j4) = make_float4(y[0], y[1], y[2], y[3]);
              }
            }
          }
        } else {
          // the FFN's first linear: bias, ReLU, quantized with the second
          // linear's alpha (the GEMM's int8 epilogue); half h of the
          // quarter takes columns [h * BN2 / 2, (h + 1) * BN2 / 2)
          int8_t* orow = p.out2q + (size_t)(row_ok ? row : 0) * p.ldo2 + n0_2;
          float amax = 0.0f;
#pragma unroll 1
          for (int c0 = half * (BN2 / 2); c0 < (half + 1) * (BN2 / 2); c0 += 32) {
            uint32_t r[32];
            tmem_ld_32x32b_x32(lane_base + c0, r);
            tmem_ld_wait();
            uint32_t w[8];
#pragma unroll
            for (int j4 = 0; j4 < 8; ++j4) {
              int qv[4];
#pragma unroll
              for (int u = 0; u < 4; ++u) {
                const int j = 4 * j4 + u;
                const float sc = p.col_scale2 ? p.col_scale2[n0_2 + c0 + j] : p.uniform_scale2;
                const float v = fmaxf(dequant(static_cast<int32_t>(r[j]), sc, s_bias2[c0 + j]), 0.0f);
                amax = fmaxf(amax, v);
                qv[u] = quant_s8(v, p.alpha3);
              }
              w[j4] = __byte_perm(__byte_perm((uint32_t)qv[0], (uint32_t)qv[1], 0x0040),
                                  __byte_perm((uint32_t)qv[2], (uint32_t)qv[3], 0x0040), 0x5410);
            }
            if (row_ok) {
              *reinterpret_cast<uint4*>(orow + c0) = make_uint4(w[0], w[1], w[2], w[3]);
              *reinterpret_cast<uint4*>(orow + c0 + 16) = make_uint4(w[4], w[5], w[6], w[7]);
            }
          }
          if (row_ok && !(amax <= 3.402823466e38f)) flag_status(p.status, kStatusNonFinite);
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, TCOLS);
  }
  asm volatile("barrier.cluster.wait.acquire;" ::: "memory");
}

template <int D, int C, int PK>
cudaError_t configure_ll() {
  static unsigned long long configured = 0;  // one bit per device ordinal
  int dev = 0;
  cudaGetDevice(&dev);
  if (!(configured & (1ull << (dev & 63)))) {
    cudaError_t e = cudaFuncSetAttribute(q8_linear_ln_kernel<D, C, PK>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         ll_smem_bytes<D, C, PK>(ll_max_stages<D, C, PK>()));
    if (e != cudaSuccess) return e;
    configured |= 1ull << (dev & 63);
  }
  return cudaSuccess;
}

template <int D, int C, int PK>
cudaError_t launch_ll(LinearLnParams p, cudaStream_t stream) {
  static_assert(ll_min_stages<D, C, PK>() <= ll_max_stages<D, C, PK>(), "shared memory plan");
  cudaError_t e = configure_ll<D, C, PK>();
  if (e != cudaSuccess) return e;
  const int num_kb = (p.k + kLlBK - 1) / kLlBK;
  // as deep as K (within the budget), and deep enough to hold the outgoing
  // segments (and, with a second linear, its operand) after the last MMA
  int stages = num_kb < ll_max_stages<D, C, PK>() ? num_kb : ll_max_stages<D, C, PK>();
  if (stages < ll_min_stages<D, C, PK>()) stages = ll_min_stages<D, C, PK>();
  p.stages = stages;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(C, (p.cap + kLlBM - 1) / kLlBM);
  cfg.blockDim = dim3(ll_threads<D>());
  cfg.dynamicSmemBytes = ll_smem_bytes<D, C, PK>(p.stages);
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = C;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = kProgrammaticLaunch ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  e = cudaLaunchKernelEx(&cfg, q8_linear_ln_kernel<D, C, PK>, p);
  return e != cudaSuccess ? e : cudaGetLastError();
}

// The FFN variant (PK 2) exists for d = 128, 256 and 512 (its 4d-wide
// columns per CTA must fit one MMA: 4 * d / C <= 256).
template <int D, int C>
constexpr bool ll_has_ffn() {
  return 4 * (D / C) <= 256 && LlShape<D, C>::KB2 <= 4;
}

template <int D, int C>
cudaError_t launch_ll_any(const LinearLnParams& p, cudaStream_t stream) {
  if (p.proj == 1) return launch_ll<D, C, 1>(p, stream);
  if (p.proj == 2) {
    if constexpr (ll_has_ffn<D, C>()) return launch_ll<D, C, 2>(p, stream);
    return cudaErrorInvalidValue;
  }
  return launch_ll<D, C, 0>(p, stream);
}

template <int D, int C>
cudaError_t configure_ll_all() {
  cudaError_t e = configure_ll<D, C, 0>();
  if (e == cudaSuccess) e = configure_ll<D, C, 1>();
  if constexpr (ll_has_ffn<D, C>())
    if (e == cudaSuccess) e = configure_ll<D, C, 2>();
  return e;
}

}  // namespace

int linear_ln_cluster(int d) {
  switch (d) {
    case 128: return 4;
    case 256: return 8;
    case 384: return 4;
    case 512: return 8;
    default: return 0;
  }
}

cudaError_t prepare_q8_linear_ln() {
  cudaError_t e = configure_ll_all<128, 4>();
  if (e == cudaSuccess) e = configure_ll_all<256, 8>();
  if (e == cudaSuccess) e = configure_ll_all<384, 4>();
  if (e == cudaSuccess) e = configure_ll_all<512, 8>();
  return e;
}

cudaError_t launch_q8_linear_ln(const LinearLnParams& p, int d, cudaStream_t stream) {
  if (p.cap <= 0) return cudaSuccess;
  if (p.k <= 0 || p.k % 16 != 0 || p.q.count < 0 || p.q.count > kMaxQuantOut ||
      (p.proj == 1 && (!p.out2 || p.ldo2 < d)) || (p.proj == 2 && (!p.out2q || p.ldo2 < 4 * d)) ||
      p.proj < 0 || p.proj > 2)
    return cudaErrorInvalidValue;
  switch (d) {
    case 128: return launch_ll_any<128, 4>(p, stream);
    case 256: return launch_ll_any<256, 8>(p, stream);
    case 384: return launch_ll_any<384, 4>(p, stream);
    case 512: return launch_ll_any<512, 8>(p, stream);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace mc
