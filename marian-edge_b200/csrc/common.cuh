// common.cuh -- shared device helpers for the sm_100a kernels of marian_cuda.
//
// Inline PTX wrappers for mbarriers, TMA tiled loads, and tcgen05 (TMEM
// allocation, MMA, commit, TMEM loads).  Every wait on an mbarrier is bounded:
// after kSpinLimit polls it records an error bit in the kernel's status word
// and returns false, so a broken pipeline ends the kernel instead of hanging
// the GPU.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace mc {

// Status bits written by kernels into the engine's device status word.
enum : uint32_t {
  kStatusNonFinite = 1u << 0,      // a quantizer saw NaN/Inf (reference: error)
  kStatusWaitTimeout = 1u << 1,    // an mbarrier wait gave up
  kStatusBadIndex = 1u << 2,       // an index failed its bounds check
};

constexpr uint32_t kSpinLimit = 1u << 24;

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void flag_status(uint32_t* status, uint32_t bits) {
  if (status) atomicOr(status, bits);
}

// ---- programmatic dependent launch ------------------------------------------
// Every engine kernel is written for programmatic stream serialization: it
// may start while its predecessor on the stream is still running and waits
// in pdl_wait() until that grid has completed and its writes are visible.
// Nothing touches global memory written or read by other kernels before
// pdl_wait().  No kernel triggers its successor early
// (griddepcontrol.launch_dependents): the successor launches as the last
// CTAs of its predecessor exit, which hides the launch gap between the two
// grids without letting waiting CTAs hold shared memory and TMEM for a
// whole kernel.  Measured end to end on the benchmark stream (decode and
// concurrent encoder streams): +3.6% over no programmatic launch, while a
// trigger at kernel entry was 3-5% slower than none.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

__device__ __forceinline__ void pdl_enter() { pdl_wait(); }

// ---- mbarrier ---------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t phase) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(phase)
      : "memory");
  return ok != 0;
}

// Bounded wait.  Returns false (and flags the status word) on timeout.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t phase, uint32_t* status) {
  for (uint32_t i = 0; i < kSpinLimit; ++i) {
    if (mbar_try_wait(bar, phase)) return true;
  }
  flag_status(status, kStatusWaitTimeout);
  return false;
}

// ---- TMA ----------------------------------------------------------------------
__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// 2-D tiled load of box {x (inner), y} into shared memory, completing on bar.
// x must be a multiple of 16 bytes for the element type (callers pass K
// offsets that are multiples of 128 bytes).
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int32_t x,
                                            int32_t y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

// L2 eviction priorities for TMA loads (a cache-policy operand): weights are
// re-read by every decode step and should stay in L2; the KV-cache pages
// stream through once per step and should leave first.
__device__ __forceinline__ uint64_t l2_policy_evict_last() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}
__device__ __forceinline__ uint64_t l2_policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}

// tma_load_2d with an L2 cache-policy hint.
__device__ __forceinline__ void tma_load_2d_hint(void* dst, const CUtensorMap* map, int32_t x, int32_t y,
                                                 uint64_t* bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%2, %3}], [%4], %5;" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}

// tma_load_3d with an L2 cache-policy hint.
__device__ __forceinline__ void tma_load_3d_hint(void* dst, const CUtensorMap* map, int32_t x, int32_t y,
                                                 int32_t z, uint64_t* bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%2, %3, %4}], [%5], %6;" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}

// 3-D tiled load of box {x, y, z} (x innermost) into shared memory.
__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, int32_t x,
                                            int32_t y, int32_t z, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar))
      : "memory");
}

// ---- tcgen05 -------------------------------------------------------------------
__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}

__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D[tmem] (+)= A[smem] x B[smem]^T, int8 x int8 -> int32.
__device__ __forceinline__ void mma_i8(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                       uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive on bar once every MMA issued so far by this thread has completed.
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_u32(bar))
      : "memory");
}

// 32 lanes x 32 consecutive 32-bit columns: thread i gets lane (base+i).
__device__ __forceinline__ void tmem_ld_32x32b_x32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
        "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]),
        "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]),
        "=r"(r[31])
      : "r"(taddr));
}

__device__ __forceinline__ void tmem_ld_wait() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// Shared-memory matrix descriptor for a K-major tile stored with the 128-byte
// swizzle: rows of 128 bytes, 8-row atoms 1024 bytes apart (stride byte
// offset), layout type 2 (SWIZZLE_128B), descriptor version 1 (sm_100).
__device__ __forceinline__ uint64_t sdesc_k_sw128(uint32_t smem_addr) {
  uint64_t d = 0;
  d |= (uint64_t)((smem_addr >> 4) & 0x3FFF);
  d |= (uint64_t)1 << 16;                 // leading byte offset (unused for SW128 K-major)
  d |= (uint64_t)(1024 >> 4) << 32;       // stride byte offset: 8 rows x 128 B
  d |= (uint64_t)1 << 46;                 // version
  d |= (uint64_t)2 << 61;                 // SWIZZLE_128B
  return d;
}

// Instruction descriptor: kind::i8, s8 x s8 -> s32, both K-major.
__host__ __device__ constexpr uint32_t idesc_i8(int m, int n) {
  return (2u << 4)            // D format: S32
         | (1u << 7)          // A: signed 8-bit
         | (1u << 10)         // B: signed 8-bit
         | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}

// ---- Q8 arithmetic shared by every kernel (q8_gemm.rs:569-590, 438-446) ------
// Quantize one activation: round-half-even, clamp to [-127, 127].  The value
// is stored centred (signed), i.e. the reference's u8 minus its zero point.
// rint(t) for t in [-127, 127], in the low byte of the result (two's
// complement): t + 1.5 * 2^23 lies in [2^23, 2^24), where adjacent floats
// are 1 apart, so the round-to-nearest-even addition rounds t to an integer
// and the sum's bit pattern is 0x4B400000 + rint(t).  One full-rate
// floating-point addition instead of a rounding and a conversion, which
// share one narrow pipe.
__device__ __forceinline__ int rint_low_byte(float t) {
  return __float_as_int(__fadd_rn(t, 12582912.0f));
}

// rint(v * alpha) clamped to [-127, 127] in the low byte (clamping first and
// rounding after gives the same value); a non-finite v gives an unspecified
// byte, so callers report it.
__device__ __forceinline__ int quantize_low_byte(float v, float alpha) {
  return rint_low_byte(fminf(fmaxf(__fmul_rn(v, alpha), -127.0f), 127.0f));
}

__device__ __forceinline__ int8_t quantize_one(float v, float alpha, uint32_t* status) {
  if (!isfinite(v)) {
    flag_status(status, kStatusNonFinite);
    return 0;
  }
  return static_cast<int8_t>(quantize_low_byte(v, alpha));
}

// acc as f32 * scale + bias, two roundings (no fused multiply-add).
__device__ __forceinline__ float dequant(int32_t acc, float scale, float bias) {
  return __fadd_rn(__fmul_rn(__int2float_rn(acc), scale), bias);
}

constexpr bool kProgrammaticLaunch = true;

#ifdef __CUDACC__
template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                              cudaStream_t stream, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = kProgrammaticLaunch ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}
#endif

}  // namespace mc
