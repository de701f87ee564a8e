// Chunked (WY / UT-transform) form of the gated delta-rule recurrence for
// prefill: the same map as gdn_seq.cu (src/ModelCPU.jl:640-674 for every
// token: S = S*exp(g); S += beta*(v - S k) k^T; y = S q), reorganised so that
// most of the work is dense matrix products over chunks of C = 64 tokens.
//
// Within a chunk (tokens t = 0..C-1, state S_0 on entry, G_t = g_0+..+g_t):
//   S_t = e^{G_t} S_0 + sum_{j<=t} e^{G_t - G_j} d_j k_j^T, and the residuals
//   d_t = beta_t (v_t - e^{G_t} S_0 k_t - sum_{j<t} e^{G_t-G_j} (k_j.k_t) d_j)
// solve the unit lower-triangular system (I + A) D = diag(beta)(V - diag(e^G) K S_0^T),
// A[t][j] = beta_t e^{G_t-G_j} k_t.k_j (j < t).  With T = (I + A)^-1 diag(beta):
//   D = U - W S_0^T,   U = T V,   W = T diag(e^G) K            (no S_0: parallel)
//   Y = diag(e^G) Q S_0^T + (Q K^T o E) D,   E[t][j] = e^{G_t-G_j} (j <= t)
//   S_C = e^{G_{C-1}} S_0 + D^T diag(e^{G_{C-1}-G}) K
// Kernel 1 (grid chunks x heads) builds W, U and P = Q K^T o E per chunk;
// kernel 2 (grid heads x 16-row blocks of S) walks the chunks in order with
// its rows of S in shared memory.  The decay ratios are formed as
// e^{G_t - G_j} (never e^{G_t} / e^{G_j}), so strong decays underflow to 0
// instead of producing 0/0.
#include <algorithm>
#include "internal.h"
#include "common.cuh"
#include "../../include/inferno_b200.h"

namespace inf {

constexpr int WY_C = 64;          // tokens per chunk
constexpr int WY_DK = 128;
constexpr int WY_THREADS = 256;
constexpr int WY_ROWS = 16;       // state rows per CTA of kernel 2

struct WyScratch {
  float* W;   // [nch][H][C][dk]
  float* U;   // [nch][H][C][dv]
  float* P;   // [nch][H][C][C]
  float* G;   // [nch][H][C]
};

// [C][dk] rows of a token-major tensor (row t at ((t0+t)*H + h)*dk, zero past
// n) into padded shared rows [C][KP]: every thread issues its eight 16-byte
// loads before the first store, so a chunk costs one load round trip
template <int KP>
__device__ __forceinline__ void wy_load_rows(float* dst, const float* src, int t0, int n, int H, int h, int tid) {
  constexpr int NV = WY_C * WY_DK / 4 / WY_THREADS;
  float4 r[NV];
#pragma unroll
  for (int u = 0; u < NV; ++u) {
    const int e = 4 * (tid + u * WY_THREADS), t = e / WY_DK, d = e % WY_DK;
    r[u] = t < n ? *(const float4*)&src[((size_t)(t0 + t) * H + h) * WY_DK + d] : make_float4(0.f, 0.f, 0.f, 0.f);
  }
#pragma unroll
  for (int u = 0; u < NV; ++u) {
    const int e = 4 * (tid + u * WY_THREADS), t = e / WY_DK, d = e % WY_DK;
    float* o = dst + t * KP + d;
    o[0] = r[u].x;
    o[1] = r[u].y;
    o[2] = r[u].z;
    o[3] = r[u].w;
  }
}

// smem: K, Q [C][dk+1] (padded rows), V [C][dv], A/T [C][C+1], G, beta
__global__ void __launch_bounds__(WY_THREADS) gdn_wy_prep_kernel(int T, int H, int dv, const float* __restrict__ q,
                                                                 const float* __restrict__ k,
                                                                 const float* __restrict__ v,
                                                                 const float* __restrict__ beta,
                                                                 const float* __restrict__ g, WyScratch o) {
  extern __shared__ float wsm[];
  constexpr int KP = WY_DK + 1, AP = WY_C + 1;
  float* Ks = wsm;                       // [C][KP]
  float* Qs = Ks + WY_C * KP;            // [C][KP]
  float* Vs = Qs + WY_C * KP;            // [C][dv]
  float* As = Vs + WY_C * dv;            // [C][AP]  A, then T
  float* Gs = As + WY_C * AP;            // [C]
  float* Bs = Gs + WY_C;                 // [C]
  float* Es = Bs + WY_C;                 // [C] e^{G_t}
  const int c = blockIdx.x, h = blockIdx.y, tid = threadIdx.x;
  const int t0 = c * WY_C, n = min(WY_C, T - t0);
  wy_load_rows<KP>(Ks, k, t0, n, H, h, tid);
  wy_load_rows<KP>(Qs, q, t0, n, H, h, tid);
  for (int i = tid; i < WY_C * dv; i += WY_THREADS) {
    const int t = i / dv, e = i % dv;
    Vs[i] = t < n ? v[((size_t)(t0 + t) * H + h) * dv + e] : 0.f;
  }
  if (tid < WY_C) {
    const bool ok = tid < n;
    Gs[tid] = ok ? g[(size_t)(t0 + tid) * H + h] : 0.f;
    Bs[tid] = ok ? beta[(size_t)(t0 + tid) * H + h] : 0.f;
  }
  __syncthreads();
  // inclusive prefix sum of g (one warp, two tokens per lane)
  if (tid < 32) {
    float a = Gs[2 * tid], b = Gs[2 * tid + 1];
    b += a;
    float s = b;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const float u = __shfl_up_sync(0xffffffffu, s, off);
      if (tid >= off) s += u;
    }
    const float excl = s - b;
    Gs[2 * tid] = excl + a;
    Gs[2 * tid + 1] = s;
  }
  __syncthreads();
  if (tid < WY_C) Es[tid] = expf(Gs[tid]);
  // A (strictly lower) and P = (Q K^T) o E (lower incl. diagonal)
  float* Pg = o.P + ((size_t)c * H + h) * WY_C * WY_C;
  for (int i = tid; i < WY_C * WY_C; i += WY_THREADS) {
    const int t = i / WY_C, j = i % WY_C;
    float a = 0.f, p = 0.f;
    if (j <= t) {
      float kk = 0.f, qk = 0.f;
      for (int d = 0; d < WY_DK; ++d) {
        const float kj = Ks[j * KP + d];
        kk = fmaf(Ks[t * KP + d], kj, kk);
        qk = fmaf(Qs[t * KP + d], kj, qk);
      }
      const float e = expf(Gs[t] - Gs[j]);
      p = qk * e;
      if (j < t) a = Bs[t] * e * kk;
    }
    As[t * AP + j] = a;
    Pg[i] = p;
  }
  __syncthreads();
  // T = (I + A)^-1 diag(beta), row by row in place over A's storage:
  // X[t][:] = beta_t e_t - sum_{j<t} A[t][j] X[j][:]  (X[j] only has columns <= j)
  // Thread = column; row t's old entries are read before the row is rewritten.
  for (int t = 0; t < WY_C; ++t) {
    float x = 0.f;
    if (tid < WY_C && tid <= t) {
      x = tid == t ? Bs[t] : 0.f;
      for (int j = tid; j < t; ++j) x = fmaf(-As[t * AP + j], As[j * AP + tid], x);
    }
    __syncthreads();
    if (tid < WY_C) As[t * AP + tid] = tid <= t ? x : 0.f;
    __syncthreads();
  }
  // W = T diag(e^G) K, U = T V
  float* Wg = o.W + ((size_t)c * H + h) * WY_C * WY_DK;
  float* Ug = o.U + ((size_t)c * H + h) * WY_C * dv;
  for (int i = tid; i < WY_C * WY_DK; i += WY_THREADS) {
    const int t = i / WY_DK, d = i % WY_DK;
    float w = 0.f;
    for (int j = 0; j <= t; ++j) w = fmaf(As[t * AP + j] * Es[j], Ks[j * KP + d], w);
    Wg[i] = w;
  }
  for (int i = tid; i < WY_C * dv; i += WY_THREADS) {
    const int t = i / dv, e = i % dv;
    float u = 0.f;
    for (int j = 0; j <= t; ++j) u = fmaf(As[t * AP + j], Vs[j * dv + e], u);
    Ug[i] = u;
  }
  if (tid < WY_C) o.G[((size_t)c * H + h) * WY_C + tid] = Gs[tid];
}

// Grid (H, dv / 16), 256 threads.  Rows r0..r0+15 of S_h live in shared
// memory across the chunks, transposed (St[d][i]) so that a thread reads four
// rows' values of one column as one 16-byte load.  Register tiles: in the D
// and Y products a thread owns token t and rows i0..i0+3; in the S update
// column d and eight rows.
__global__ void __launch_bounds__(WY_THREADS) gdn_wy_state_kernel(int T, int H, int dv, const float* __restrict__ q,
                                                                  const float* __restrict__ k, float* S, float* y,
                                                                  WyScratch o) {
  extern __shared__ __align__(16) float wsm[];
  constexpr int KP = WY_DK + 1;
  float* St = wsm;                          // [dk][16]
  float* Ws = St + WY_DK * WY_ROWS;         // [C][KP]
  float* Ks = Ws + WY_C * KP;               // [C][KP]
  float* Qs = Ks + WY_C * KP;               // [C][KP]
  float* Ds = Qs + WY_C * KP;               // [C][16]  D rows of this CTA
  float* Ps = Ds + WY_C * WY_ROWS;          // [C][C]
  float* Gs = Ps + WY_C * WY_C;             // [C]
  float* EGs = Gs + WY_C;                   // [C] e^{G_t}
  float* DEs = EGs + WY_C;                  // [C] e^{G_last - G_j}
  const int h = blockIdx.x, r0 = blockIdx.y * WY_ROWS, tid = threadIdx.x;
  for (int i = tid; i < WY_ROWS * WY_DK; i += WY_THREADS) {
    const int r = i / WY_DK, d = i % WY_DK;
    St[d * WY_ROWS + r] = S[((size_t)h * dv + r0 + r) * WY_DK + d];
  }
  // D / Y tile: token tt, rows i0..i0+3; S tile: column sd, rows si0..si0+7
  const int tt = tid >> 2, i0 = (tid & 3) * 4;
  const int sd = tid & (WY_DK - 1), si0 = (tid >> 7) * 8;
  const int nch = (T + WY_C - 1) / WY_C;
  for (int c = 0; c < nch; ++c) {
    const int t0 = c * WY_C, n = min(WY_C, T - t0);
    __syncthreads();
    const float* Wg = o.W + ((size_t)c * H + h) * WY_C * WY_DK;
    wy_load_rows<KP>(Ws, Wg, 0, WY_C, 1, 0, tid);     // W is chunk-major [C][dk]
    wy_load_rows<KP>(Ks, k, t0, n, H, h, tid);
    wy_load_rows<KP>(Qs, q, t0, n, H, h, tid);
    const float* Pg = o.P + ((size_t)c * H + h) * WY_C * WY_C;
    {
      float4 pr[WY_C * WY_C / 4 / WY_THREADS];
#pragma unroll
      for (int u = 0; u < WY_C * WY_C / 4 / WY_THREADS; ++u) pr[u] = ((const float4*)Pg)[tid + u * WY_THREADS];
#pragma unroll
      for (int u = 0; u < WY_C * WY_C / 4 / WY_THREADS; ++u) ((float4*)Ps)[tid + u * WY_THREADS] = pr[u];
    }
    if (tid < WY_C) {
      const float gt = o.G[((size_t)c * H + h) * WY_C + tid];
      const float glast = o.G[((size_t)c * H + h) * WY_C + (n - 1)];
      Gs[tid] = gt;
      EGs[tid] = expf(gt);
      DEs[tid] = tid < n ? expf(glast - gt) : 0.f;
    }
    __syncthreads();
    // D[t][i] = U[t][i] - W[t] . S[i]
    {
      const float* Ug = o.U + ((size_t)c * H + h) * WY_C * dv + (size_t)tt * dv + r0 + i0;
      float a0 = Ug[0], a1 = Ug[1], a2 = Ug[2], a3 = Ug[3];
      const float* wr = Ws + tt * KP;
#pragma unroll 8
      for (int d = 0; d < WY_DK; ++d) {
        const float w = wr[d];
        const float4 s4 = *(const float4*)&St[d * WY_ROWS + i0];
        a0 = fmaf(-w, s4.x, a0);
        a1 = fmaf(-w, s4.y, a1);
        a2 = fmaf(-w, s4.z, a2);
        a3 = fmaf(-w, s4.w, a3);
      }
      *(float4*)&Ds[tt * WY_ROWS + i0] = make_float4(a0, a1, a2, a3);
    }
    __syncthreads();
    // Y[t][i] = e^{G_t} Q[t] . S[i] + sum_{j<=t} P[t][j] D[j][i]
    if (tt < n) {
      float q0 = 0.f, q1 = 0.f, q2 = 0.f, q3 = 0.f;
      const float* qr = Qs + tt * KP;
#pragma unroll 8
      for (int d = 0; d < WY_DK; ++d) {
        const float qv = qr[d];
        const float4 s4 = *(const float4*)&St[d * WY_ROWS + i0];
        q0 = fmaf(qv, s4.x, q0);
        q1 = fmaf(qv, s4.y, q1);
        q2 = fmaf(qv, s4.z, q2);
        q3 = fmaf(qv, s4.w, q3);
      }
      const float eg = EGs[tt];
      float a0 = eg * q0, a1 = eg * q1, a2 = eg * q2, a3 = eg * q3;
      const float* pr = Ps + tt * WY_C;
      for (int j = 0; j <= tt; ++j) {
        const float pv = pr[j];
        const float4 d4 = *(const float4*)&Ds[j * WY_ROWS + i0];
        a0 = fmaf(pv, d4.x, a0);
        a1 = fmaf(pv, d4.y, a1);
        a2 = fmaf(pv, d4.z, a2);
        a3 = fmaf(pv, d4.w, a3);
      }
      float* yo = y + ((size_t)(t0 + tt) * H + h) * dv + r0 + i0;
      yo[0] = a0;
      yo[1] = a1;
      yo[2] = a2;
      yo[3] = a3;
    }
    __syncthreads();
    // S[i][d] = e^{G_last} S[i][d] + sum_j e^{G_last - G_j} D[j][i] K[j][d]
    {
      const float egl = EGs[n - 1];
      float acc[8];
      const float4 sa = *(const float4*)&St[sd * WY_ROWS + si0], sb = *(const float4*)&St[sd * WY_ROWS + si0 + 4];
      acc[0] = egl * sa.x; acc[1] = egl * sa.y; acc[2] = egl * sa.z; acc[3] = egl * sa.w;
      acc[4] = egl * sb.x; acc[5] = egl * sb.y; acc[6] = egl * sb.z; acc[7] = egl * sb.w;
      for (int j = 0; j < n; ++j) {
        const float kk = Ks[j * KP + sd], de = DEs[j];
        const float4 da = *(const float4*)&Ds[j * WY_ROWS + si0], db = *(const float4*)&Ds[j * WY_ROWS + si0 + 4];
        acc[0] = fmaf(de * da.x, kk, acc[0]);
        acc[1] = fmaf(de * da.y, kk, acc[1]);
        acc[2] = fmaf(de * da.z, kk, acc[2]);
        acc[3] = fmaf(de * da.w, kk, acc[3]);
        acc[4] = fmaf(de * db.x, kk, acc[4]);
        acc[5] = fmaf(de * db.y, kk, acc[5]);
        acc[6] = fmaf(de * db.z, kk, acc[6]);
        acc[7] = fmaf(de * db.w, kk, acc[7]);
      }
      *(float4*)&St[sd * WY_ROWS + si0] = make_float4(acc[0], acc[1], acc[2], acc[3]);
      *(float4*)&St[sd * WY_ROWS + si0 + 4] = make_float4(acc[4], acc[5], acc[6], acc[7]);
    }
  }
  __syncthreads();
  for (int i = tid; i < WY_ROWS * WY_DK; i += WY_THREADS) {
    const int r = i / WY_DK, d = i % WY_DK;
    S[((size_t)h * dv + r0 + r) * WY_DK + d] = St[d * WY_ROWS + r];
  }
}

size_t gdn_wy_scratch_bytes(int T, int H, int dv) {
  const size_t nch = (size_t)(T + WY_C - 1) / WY_C;
  return nch * H * WY_C * ((size_t)WY_DK + dv + WY_C + 1) * 4 + 1024;
}

int launch_gdn_wy(int T, int H, int dv, const float* q, const float* k, const float* v, const float* beta,
                  const float* g, float* S, float* y, void* scratch, cudaStream_t st) {
  if (T <= 0) return 0;
  if (dv % WY_ROWS || dv > WY_DK) return set_error(INFERNO_EINVAL, "gdn chunked: dv %d", dv);
  const size_t nch = (size_t)(T + WY_C - 1) / WY_C;
  float* base = (float*)(((uintptr_t)scratch + 255) & ~(uintptr_t)255);
  WyScratch o;
  o.W = base;
  o.U = o.W + nch * H * WY_C * WY_DK;
  o.P = o.U + nch * H * WY_C * dv;
  o.G = o.P + nch * H * WY_C * WY_C;
  const size_t smem1 = ((size_t)2 * WY_C * (WY_DK + 1) + (size_t)WY_C * dv + (size_t)WY_C * (WY_C + 1) + 3 * WY_C) * 4;
  const size_t smem2 = ((size_t)WY_ROWS * WY_DK + 3 * (size_t)WY_C * (WY_DK + 1) + (size_t)WY_C * WY_ROWS +
                        (size_t)WY_C * WY_C + 3 * WY_C) * 4;
  static DeviceOnce once;
  cudaError_t ea = once.run([] {
    cudaError_t e = cudaFuncSetAttribute(gdn_wy_prep_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
    if (e != cudaSuccess) return e;
    return cudaFuncSetAttribute(gdn_wy_state_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
  });
  if (ea != cudaSuccess) return set_error(INFERNO_ECUDA, "gdn chunked attribute: %s", cudaGetErrorString(ea));
  gdn_wy_prep_kernel<<<dim3((unsigned)nch, H), WY_THREADS, smem1, st>>>(T, H, dv, q, k, v, beta, g, o);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_error(INFERNO_ECUDA, "gdn chunked prep: %s", cudaGetErrorString(e));
  gdn_wy_state_kernel<<<dim3(H, dv / WY_ROWS), WY_THREADS, smem2, st>>>(T, H, dv, q, k, S, y, o);
  e = cudaGetLastError();
  return e == cudaSuccess ? 0 : set_error(INFERNO_ECUDA, "gdn chunked state: %s", cudaGetErrorString(e));
}

}  // namespace inf

using namespace inf;

/* The recurrence of inferno_gdn_recurrence in its chunked (WY) form, chunks
 * of 64 tokens; stream-ordered scratch of gdn_wy_scratch_bytes(). */
extern "C" int inferno_gdn_chunked(int T, int n_heads, int dk, int dv, const float* q, const float* k,
                                   const float* v, const float* beta, const float* g, float* S, float* y, int chunk,
                                   void* stream) {
  if (T <= 0 || n_heads <= 0 || !q || !k || !v || !beta || !g || !S || !y)
    return set_error(INFERNO_EINVAL, "gdn_chunked: bad arguments");
  if (dk != WY_DK || dv % WY_ROWS || dv > WY_DK || chunk != WY_C)
    return set_error(INFERNO_EINVAL, "gdn_chunked: dk must be %d, dv a multiple of %d up to %d, chunk %d", WY_DK,
                     WY_ROWS, WY_DK, WY_C);
  cudaStream_t st = (cudaStream_t)stream;
  void* scratch = nullptr;
  INF_CUDA_TRY(cudaMallocAsync(&scratch, gdn_wy_scratch_bytes(T, n_heads, dv), st));
  const int rc = launch_gdn_wy(T, n_heads, dv, q, k, v, beta, g, S, y, scratch, st);
  cudaError_t ef = cudaFreeAsync(scratch, st);
  if (rc) return rc;
  return ef == cudaSuccess ? 0 : set_error(INFERNO_ECUDA, "gdn_chunked: %s", cudaGetErrorString(ef));
}
