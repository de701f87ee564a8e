// Shared device helpers for the sm_100a decode engine: GGUF type ids, TMA
// bulk copies into shared memory with mbarrier completion, bounded waits and
// programmatic-dependent-launch controls.
#pragma once
#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <stdint.h>

namespace inf {

// ggml type ids (GGUF spec; Inferno.jl src/GGUF.jl:25-60)
enum GgmlType : int {
  T_F32 = 0, T_F16 = 1, T_Q8_0 = 8, T_Q4_K = 12, T_Q5_K = 13, T_Q6_K = 14, T_IQ2_XXS = 16,
  // engine-internal: Q6_K bytes regrouped per 16 rows for the tensor-core
  // GEMV (gemv_mma.cuh); same size, never visible at the C ABI
  T_Q6_KR = 114
};

__host__ __device__ constexpr int qk_of(int t) { return t == T_Q8_0 ? 32 : (t == T_F32 || t == T_F16) ? 1 : 256; }
__host__ __device__ constexpr int bb_of(int t) {
  return t == T_F32 ? 4 : t == T_F16 ? 2 : t == T_Q8_0 ? 34 : t == T_Q4_K ? 144 : t == T_Q5_K ? 176
       : (t == T_Q6_K || t == T_Q6_KR) ? 210 : t == T_IQ2_XXS ? 66 : 0;
}
inline bool type_supported(int t) {
  return t == T_F32 || t == T_Q8_0 || t == T_Q4_K || t == T_Q5_K || t == T_Q6_K || t == T_IQ2_XXS;
}

// Device-side error word: kernels never trap; a wait that runs out of budget
// records a code here and the kernel returns.  The host reads it after sync.
enum DevErr : int { DERR_NONE = 0, DERR_MBAR_TIMEOUT = 1, DERR_BAD_ARG = 2 };

// ---------------------------------------------------------------------------
// PTX wrappers
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait: gives up after ~2^26 polls (seconds), records DERR_MBAR_TIMEOUT
// and returns false so the caller can leave the kernel.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int* err) {
  for (uint32_t i = 0; i < (1u << 26); ++i)
    if (mbar_try_wait(bar, parity)) return true;
  if (err) atomicExch(err, DERR_MBAR_TIMEOUT);
  return false;
}

// 1-D TMA bulk copy global -> shared, completion counted on `bar` in bytes.
// dst, src and bytes must be multiples of 16.
__device__ __forceinline__ void tma_load_1d(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// Same, with an L2 cache policy (e.g. evict_first for weights streamed once
// per token, so they do not push code, activations and recurrent state out of
// L2).
__device__ __forceinline__ uint64_t l2_policy_evict_first() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}
__device__ __forceinline__ void tma_load_1d_hint(void* dst, const void* src, uint32_t bytes, uint64_t* bar,
                                                 uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}

__device__ __forceinline__ unsigned long long gtimer() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

// Kernel timeline stamps, compiled in only with -DINFERNO_KTRACE=1 (they sit
// on the latency-critical path).  With INFERNO_B200_TRACE set at engine
// creation every launch of a token gets 8 u64 slots (`trace`); thread 0 of
// every CTA folds its %globaltimer into them with atomicMax, earliest-of
// stamps stored complemented so that one zeroed buffer serves both:
//   0 kernel kind, 1 ~first CTA entry, 2 ~first CTA past griddepcontrol.wait,
//   3 last CTA past the wait, 4 last prologue done, 5 last first weight tile,
//   6 last CTA exit.
#ifndef INFERNO_KTRACE
#define INFERNO_KTRACE 0
#endif
enum KtKind : int { KT_GEMV = 1, KT_GEMV_MMA = 2, KT_GDN = 3, KT_ATTN = 4 };
#define KT_FIRST(tr, s) \
  do { if (INFERNO_KTRACE && (tr)) atomicMax((tr) + (s), ~gtimer()); } while (0)
#define KT_LAST(tr, s) \
  do { if (INFERNO_KTRACE && (tr)) atomicMax((tr) + (s), gtimer()); } while (0)
#define KT_KIND(tr, k) \
  do { if (INFERNO_KTRACE && (tr) && blockIdx.x == 0 && blockIdx.y == 0) (tr)[0] = (k); } while (0)

// Programmatic dependent launch (no-ops when the launch did not enable it).
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

__device__ __forceinline__ void named_bar_sync(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// ---------------------------------------------------------------------------
// small math helpers
// ---------------------------------------------------------------------------
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
__device__ __forceinline__ float h2f_bits(uint16_t h) { return __half2float(__ushort_as_half(h)); }

// byte k (0..3) of w as an exact float, via the 2^23 magic exponent:
// bits 0x4B0000bb == 8388608 + bb; subtract (8388608 + off) to get bb - off.
template <int K>
__device__ __forceinline__ float byte_as_float(uint32_t w, float magic_minus_off) {
  return __uint_as_float(__byte_perm(w, 0x4B000000u, 0x7650u | K)) - magic_minus_off;
}

// 32-bit load from a shared-memory byte address of any alignment (reads the
// two enclosing aligned words).
__device__ __forceinline__ uint32_t lds_u32_any(const uint8_t* p) {
  uintptr_t a = (uintptr_t)p;
  const uint32_t* q = (const uint32_t*)(a & ~(uintptr_t)3);
  uint32_t sh = (uint32_t)(a & 3) * 8u;
  uint32_t w0 = q[0], w1 = q[1];
  return __funnelshift_r(w0, w1, sh);
}
__device__ __forceinline__ uint16_t lds_u16_any(const uint8_t* p) {
  return (uint16_t)(p[0] | (p[1] << 8));
}

// order-preserving float -> uint32 (for atomicMax-based argmax)
__device__ __forceinline__ uint32_t float_ordered(float f) {
  uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__host__ __device__ inline float ordered_to_float(uint32_t o) {
  uint32_t u = (o & 0x80000000u) ? (o & 0x7fffffffu) : ~o;
  union { uint32_t u; float f; } c;
  c.u = u;
  return c.f;
}

}  // namespace inf
