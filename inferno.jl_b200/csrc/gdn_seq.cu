// Gated delta-rule recurrence over a sequence of T steps (the state update of
// GatedDeltaNetCPU, Inferno.jl src/ModelCPU.jl:640-674, without the
// projections): for every head h and step t
//     S_h = S_h * exp(g[t,h])
//     S_h += beta[t,h] * (v[t,h] - S_h k[t,h]) k[t,h]^T
//     y[t,h] = S_h q[t,h]
// with q, k as given (already normalised by the caller).  Layouts: q, k
// [T][H][dk]; v, y [T][H][dv]; beta, g [T][H]; S [H][dv][dk] row-major fp32.
//
// One launch runs all T steps.  A CTA owns GS_ROWS rows of one head's state
// and keeps them in registers for the whole sequence (a warp per row, four
// fp32 per lane): state traffic is one read and one write in total instead of
// one per step.  The per-step inputs of the head (q, k: 1 KB; v rows, beta,
// g) are staged chunk by chunk into shared memory with cp.async, the next
// chunk in flight while the current one is consumed.  Rows are independent
// given q and k, so CTAs never synchronise with each other.
#include "internal.h"
#include "common.cuh"
#include "../../include/inferno_b200.h"

namespace inf {

constexpr int GS_DK = 128;
constexpr int GS_ROWS = 16;              // state rows per CTA (2 per warp)
constexpr int GS_WARPS = 8;
constexpr int GS_THREADS = GS_WARPS * 32;
constexpr int GS_CHUNK = 32;             // steps per staged chunk

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(smem)), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async4(void* smem, const void* gmem) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_u32(smem)), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_1() { asm volatile("cp.async.wait_group 1;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_0() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }

struct GsBuf {
  float4 q[GS_CHUNK][GS_DK / 4];
  float4 k[GS_CHUNK][GS_DK / 4];
  float v[GS_CHUNK][GS_ROWS];
  float beta[GS_CHUNK];
  float g[GS_CHUNK];
};

__device__ void gs_stage(GsBuf& b, int t0, int T, int H, int h, int dv, int r0, const float* q, const float* k,
                         const float* v, const float* beta, const float* g) {
  const int tid = threadIdx.x;
  const int n = min(GS_CHUNK, T - t0);
  // q, k: n steps x 32 float4 each
  for (int i = tid; i < n * (GS_DK / 4) * 2; i += GS_THREADS) {
    const int which = i / (n * (GS_DK / 4)), r = i % (n * (GS_DK / 4));
    const int s = r / (GS_DK / 4), c = r % (GS_DK / 4);
    const float* src = (which ? k : q) + ((size_t)(t0 + s) * H + h) * GS_DK + 4 * c;
    cp_async16(which ? &b.k[s][c] : &b.q[s][c], src);
  }
  for (int i = tid; i < n * GS_ROWS; i += GS_THREADS) {
    const int s = i / GS_ROWS, rr = i % GS_ROWS;
    cp_async4(&b.v[s][rr], v + ((size_t)(t0 + s) * H + h) * dv + r0 + rr);
  }
  for (int i = tid; i < n; i += GS_THREADS) {
    cp_async4(&b.beta[i], beta + (size_t)(t0 + i) * H + h);
    cp_async4(&b.g[i], g + (size_t)(t0 + i) * H + h);
  }
}

__global__ void __launch_bounds__(GS_THREADS) gdn_seq_kernel(int T, int H, int dv, const float* __restrict__ q,
                                                             const float* __restrict__ k,
                                                             const float* __restrict__ v,
                                                             const float* __restrict__ beta,
                                                             const float* __restrict__ g, float* S, float* y) {
  extern __shared__ __align__(16) uint8_t gs_smem[];
  GsBuf* buf = (GsBuf*)gs_smem;          // [2]
  const int h = blockIdx.x, r0 = blockIdx.y * GS_ROWS;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  constexpr int RPW = GS_ROWS / GS_WARPS;   // rows per warp
  float4 s[RPW];
#pragma unroll
  for (int j = 0; j < RPW; ++j)
    s[j] = *((const float4*)(S + ((size_t)h * dv + r0 + warp + GS_WARPS * j) * GS_DK) + lane);
  const int nchunks = (T + GS_CHUNK - 1) / GS_CHUNK;
  gs_stage(buf[0], 0, T, H, h, dv, r0, q, k, v, beta, g);
  cp_async_commit();
  for (int c = 0; c < nchunks; ++c) {
    const int t0 = c * GS_CHUNK;
    if (c + 1 < nchunks) gs_stage(buf[(c + 1) & 1], t0 + GS_CHUNK, T, H, h, dv, r0, q, k, v, beta, g);
    cp_async_commit();
    cp_async_wait_1();                   // chunk c landed (c + 1 may be in flight)
    __syncthreads();
    const GsBuf& b = buf[c & 1];
    const int n = min(GS_CHUNK, T - t0);
    for (int st = 0; st < n; ++st) {
      const float4 k4 = b.k[st][lane], q4 = b.q[st][lane];
      const float dec = expf(b.g[st]), bt = b.beta[st];
#pragma unroll
      for (int j = 0; j < RPW; ++j) {
        const int rr = warp + GS_WARPS * j;
        float4 x = s[j];
        x.x *= dec; x.y *= dec; x.z *= dec; x.w *= dec;
        const float sk = warp_sum(x.x * k4.x + x.y * k4.y + x.z * k4.z + x.w * k4.w);
        const float d = bt * (b.v[st][rr] - sk);
        x.x += d * k4.x; x.y += d * k4.y; x.z += d * k4.z; x.w += d * k4.w;
        const float o = warp_sum(x.x * q4.x + x.y * q4.y + x.z * q4.z + x.w * q4.w);
        s[j] = x;
        if (lane == 0) y[((size_t)(t0 + st) * H + h) * dv + r0 + rr] = o;
      }
    }
    __syncthreads();                     // buffer c & 1 is restaged two chunks later
  }
  cp_async_wait_0();
#pragma unroll
  for (int j = 0; j < RPW; ++j)
    *((float4*)(S + ((size_t)h * dv + r0 + warp + GS_WARPS * j) * GS_DK) + lane) = s[j];
}

int launch_gdn_seq(int T, int n_heads, int dv, const float* q, const float* k, const float* v, const float* beta,
                   const float* g, float* S, float* y, cudaStream_t st) {
  const size_t smem = 2 * sizeof(GsBuf);
  static DeviceOnce once;
  cudaError_t ea = once.run([] {
    return cudaFuncSetAttribute(gdn_seq_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
  });
  if (ea != cudaSuccess) return set_error(INFERNO_ECUDA, "gdn_recurrence: %s", cudaGetErrorString(ea));
  gdn_seq_kernel<<<dim3(n_heads, dv / GS_ROWS), GS_THREADS, smem, st>>>(T, n_heads, dv, q, k, v, beta, g, S, y);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? 0 : set_error(INFERNO_ECUDA, "gdn_recurrence launch: %s", cudaGetErrorString(e));
}

}  // namespace inf

using namespace inf;

/* Gated delta-rule recurrence over T steps on device pointers (see the
 * header). */
extern "C" int inferno_gdn_recurrence(int T, int n_heads, int dk, int dv, const float* q, const float* k,
                                      const float* v, const float* beta, const float* g, float* S, float* y,
                                      void* stream) {
  if (T <= 0 || n_heads <= 0 || !q || !k || !v || !beta || !g || !S || !y)
    return set_error(INFERNO_EINVAL, "gdn_recurrence: bad arguments");
  if (dk != GS_DK || dv % GS_ROWS)
    return set_error(INFERNO_EINVAL, "gdn_recurrence: dk must be %d and dv a multiple of %d", GS_DK, GS_ROWS);
  if (((uintptr_t)q | (uintptr_t)k | (uintptr_t)S) & 15)
    return set_error(INFERNO_EINVAL, "gdn_recurrence: q, k and S must be 16-byte aligned");
  return launch_gdn_seq(T, n_heads, dv, q, k, v, beta, g, S, y, (cudaStream_t)stream);
}
