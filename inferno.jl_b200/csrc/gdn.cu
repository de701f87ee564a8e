// Fused Gated DeltaNet decode step (one launch per GDN layer and token).
//
// Replaces the body of GatedDeltaNetCPU (Inferno.jl src/ModelCPU.jl:531-700)
// after the in_proj / attn_gate GEMVs:
//   * alpha / beta projections of RMSNorm(x) (F32 [nv x H], :571-575), with the
//     input RMSNorm recomputed per CTA (src/ModelCPU.jl:110-122);
//   * causal conv1d over a K-slot ring of past in_proj outputs + SiLU (:541-564);
//   * per-head L2 norm of q, k with the 1/sqrt(dk) query scale (:593-616);
//   * gates in Float64 as the reference computes them (:618-636);
//   * the delta-rule update S = S*decay; S += beta*(v - S k)k^T; y = S q
//     (:640-674) with the fp32 state resident in HBM, one warp per state row.
// The per-head output RMSNorm and SiLU(z) gate (:682-692) are fused into the
// prologue of the following ssm_out GEMV.
//
// Grid: (nv heads, dv / GDN_ROWS row-blocks).  Each CTA recomputes the conv
// and norms of its head's q/k group (modulo head map h % nk, :587) and owns
// GDN_ROWS rows of the head's state.  State layout [nv][dv][dk] row-major.
// The conv ring holds the last K inputs: input of step t lives in slot t % K;
// the step counter is per layer and advanced by the last CTA to finish.
#include "internal.h"
#include "common.cuh"
#include "params.h"
#include "../../include/inferno_b200.h"

namespace inf {

constexpr int GDN_THREADS = 128;
constexpr int GDN_ROWS = 16;
constexpr int GDN_DK = 128;



__device__ __forceinline__ float block_sum128(float v, float* red) {
  v = warp_sum(v);
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  return red[0] + red[1] + red[2] + red[3];
}

__global__ void __launch_bounds__(GDN_THREADS) gdn_step_kernel(const __grid_constant__ GdnParams p) {
  __shared__ float qn[GDN_DK], kn[GDN_DK], vrow[GDN_ROWS];
  __shared__ float red[4];
  __shared__ float gate_s[2];
  pdl_trigger();
  pdl_wait();
  const int h = blockIdx.x, r0 = blockIdx.y * GDN_ROWS, tid = threadIdx.x;
  const int g = h % p.nk;
  const int t = *p.step;
  const int K = p.K, C = p.C;
  const int cur = t % K;

  // ---- RMSNorm(x) folded into the alpha/beta dots ----
  float ss = 0.f;
  for (int i = tid; i < p.H; i += GDN_THREADS) ss += p.x[i] * p.x[i];
  ss = block_sum128(ss, red);
  const float scale = 1.0f / sqrtf(ss / (float)p.H + p.eps);
  float da = 0.f, dbv = 0.f;
  const float* wa = p.w_alpha + (long long)h * p.H;
  const float* wb = p.w_beta + (long long)h * p.H;
  for (int i = tid; i < p.H; i += GDN_THREADS) {
    float xn = p.x[i] * scale * p.in_norm[i];
    da = fmaf(wa[i], xn, da);
    dbv = fmaf(wb[i], xn, dbv);
  }
  float alpha = block_sum128(da, red);
  float beta_raw = block_sum128(dbv, red);

  // ---- conv1d + SiLU for this head's q, k (group g) and v rows ----
  auto conv = [&](int c, bool write) -> float {
    float nv = p.qkv[c];
    float v = 0.f;
    for (int k = 0; k < K - 1; ++k) {
      int slot = (t - (K - 1) + k) % K;
      if (slot < 0) slot += K;
      v += p.ring[(long long)slot * C + c] * p.conv_w[(long long)c * K + k];
    }
    v += nv * p.conv_w[(long long)c * K + K - 1];
    if (write) p.ring[(long long)cur * C + c] = nv;
    return v / (1.0f + expf(-v));
  };
  const bool qk_owner = (h == g) && blockIdx.y == 0;   // first head of group g
  float qv = 0.f, kv = 0.f;
  if (tid < GDN_DK) {
    qv = conv(g * GDN_DK + tid, qk_owner);
    kv = conv(p.nk * GDN_DK + g * GDN_DK + tid, qk_owner);
  }
  if (tid < GDN_ROWS) vrow[tid] = conv(2 * p.nk * GDN_DK + h * p.dv + r0 + tid, true);

  // ---- L2 norms (src/ModelCPU.jl:597-616) ----
  float qs = block_sum128(qv * qv, red);
  float ks = block_sum128(kv * kv, red);
  const float eps6 = 1.0e-6f;
  const float qscale = 1.0f / sqrtf((float)GDN_DK);
  const float qnv = 1.0f / (sqrtf(qs) + eps6) * qscale;
  const float knv = 1.0f / (sqrtf(ks) + eps6);
  if (tid < GDN_DK) {
    qn[tid] = qv * qnv;
    kn[tid] = kv * knv;
  }
  // ---- gates in Float64 (src/ModelCPU.jl:618-636) ----
  if (tid == 0) {
    double a = (double)alpha + (double)p.dt_bias[h];
    a = fmin(20.0, fmax(-20.0, a));
    double sp = log(1.0 + exp(a));
    float decay = (float)((double)p.ssm_a[h] * sp);
    gate_s[0] = expf(decay);
    double bv = fmin(20.0, fmax(-20.0, (double)beta_raw));
    gate_s[1] = (float)(1.0 / (1.0 + exp(-bv)));
  }
  __syncthreads();
  const float dec = gate_s[0], bg = gate_s[1];

  // ---- delta rule, one warp per state row, 4 fp32 per lane ----
  const int warp = tid >> 5, lane = tid & 31;
  const float4 k4 = *(const float4*)&kn[lane * 4];
  const float4 q4 = *(const float4*)&qn[lane * 4];
  for (int rr = warp; rr < GDN_ROWS; rr += GDN_THREADS / 32) {
    const int i = r0 + rr;
    float4* Srow = (float4*)(p.S + ((long long)h * p.dv + i) * GDN_DK) + lane;
    float4 s = *Srow;
    s.x *= dec; s.y *= dec; s.z *= dec; s.w *= dec;
    float sk = warp_sum(s.x * k4.x + s.y * k4.y + s.z * k4.z + s.w * k4.w);
    float d = bg * (vrow[rr] - sk);
    s.x += d * k4.x; s.y += d * k4.y; s.z += d * k4.z; s.w += d * k4.w;
    float yv = warp_sum(s.x * q4.x + s.y * q4.y + s.z * q4.z + s.w * q4.w);
    *Srow = s;
    if (lane == 0) p.y[h * p.dv + i] = yv;
  }

  // ---- advance the layer's step counter once all CTAs have read it ----
  __syncthreads();
  if (tid == 0) {
    __threadfence();
    int total = gridDim.x * gridDim.y;
    int prev = atomicAdd(p.done, 1);
    if (prev == total - 1) {
      *p.done = 0;
      *p.step = t + 1;
      __threadfence();
    }
  }
}

int launch_gdn_step(const GdnParams& p, cudaStream_t st, bool pdl) {
  if (p.dv % GDN_ROWS || p.K < 1 || p.K > 8)
    return set_error(INFERNO_EINVAL, "gdn: unsupported dims (dv=%d, K=%d)", p.dv, p.K);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(p.nv, p.dv / GDN_ROWS);
  cfg.blockDim = dim3(GDN_THREADS);
  cfg.stream = st;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = pdl ? 1 : 0;
  cudaError_t e = cudaLaunchKernelEx(&cfg, gdn_step_kernel, p);
  return e == cudaSuccess ? 0 : set_error(INFERNO_ECUDA, "gdn launch: %s", cudaGetErrorString(e));
}

}  // namespace inf
