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
//
// Latency structure: everything that does not depend on the preceding
// kernel (state rows, ring slots, conv / alpha / beta / norm weights) is
// loaded before griddepcontrol.wait; after it only x and the in_proj output
// are read, followed by two block reductions.  Every engine kernel triggers
// its dependents only after its own wait, so data written two or more
// launches earlier is complete when this pre-wait code runs.
#include "internal.h"
#include "common.cuh"
#include "params.h"
#include "../../include/inferno_b200.h"

namespace inf {

constexpr int GDN_THREADS = 128;
constexpr int GDN_ROWS = 16;
constexpr int GDN_DK = 128;
constexpr int GDN_MAXK = 4;          // conv taps held in registers
constexpr int GDN_MAX_H = 8192;      // hidden size (smem for the alpha/beta weights)

template <int NV>
__device__ __forceinline__ void block_sum_n(float (&v)[NV], float (*red)[4]) {
#pragma unroll
  for (int i = 0; i < NV; ++i) v[i] = warp_sum(v[i]);
  if ((threadIdx.x & 31) == 0)
#pragma unroll
    for (int i = 0; i < NV; ++i) red[i][threadIdx.x >> 5] = v[i];
  __syncthreads();
#pragma unroll
  for (int i = 0; i < NV; ++i) v[i] = (red[i][0] + red[i][1]) + (red[i][2] + red[i][3]);
}

__global__ void __launch_bounds__(GDN_THREADS) gdn_step_kernel(const __grid_constant__ GdnParams p) {
  extern __shared__ __align__(16) float gsm[];     // [3][H]: w_alpha row, w_beta row, in_norm
  __shared__ __align__(16) float qn[GDN_DK], kn[GDN_DK];
  __shared__ float vrow[GDN_ROWS];
  __shared__ float red[5][4];
  __shared__ float gate_s[2];
  const int h = blockIdx.x, r0 = blockIdx.y * GDN_ROWS, tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31;
  const int g = h % p.nk;
  const int K = p.K, C = p.C, H = p.H;
  if (tid == 0) {
    KT_KIND(p.trace, KT_GDN);
    KT_FIRST(p.trace, 1);
  }

  // ---------------- pre-wait: state and constants ----------------
  const int t = *p.step;            // written by this layer's previous step
  const int cur = t % K;
  float* wa_s = gsm;
  float* wb_s = gsm + H;
  float* wn_s = gsm + 2 * H;
  for (int i = tid * 4; i < H; i += GDN_THREADS * 4) {
    *(float4*)&wa_s[i] = *(const float4*)&p.w_alpha[(long long)h * H + i];
    *(float4*)&wb_s[i] = *(const float4*)&p.w_beta[(long long)h * H + i];
    *(float4*)&wn_s[i] = *(const float4*)&p.in_norm[i];
  }
  // conv taps and past inputs for this thread's channels
  const int cq = g * GDN_DK + tid, ck = p.nk * GDN_DK + g * GDN_DK + tid;
  const int cv = 2 * p.nk * GDN_DK + h * p.dv + r0 + tid;     // valid for tid < GDN_ROWS
  float wq[GDN_MAXK], wk[GDN_MAXK], wv[GDN_MAXK], hq[GDN_MAXK], hk[GDN_MAXK], hv[GDN_MAXK];
#pragma unroll
  for (int k = 0; k < GDN_MAXK; ++k) {
    wq[k] = wk[k] = wv[k] = hq[k] = hk[k] = hv[k] = 0.f;
    if (k < K) {
      int slot = (t - (K - 1) + k) % K;
      if (slot < 0) slot += K;
      wq[k] = p.conv_w[(long long)cq * K + k];
      wk[k] = p.conv_w[(long long)ck * K + k];
      if (k < K - 1) {
        hq[k] = p.ring[(long long)slot * C + cq];
        hk[k] = p.ring[(long long)slot * C + ck];
      }
      if (tid < GDN_ROWS) {
        wv[k] = p.conv_w[(long long)cv * K + k];
        if (k < K - 1) hv[k] = p.ring[(long long)slot * C + cv];
      }
    }
  }
  // this warp's state rows (4 fp32 per lane per row)
  constexpr int RPW = GDN_ROWS / (GDN_THREADS / 32);
  float4 srow[RPW];
#pragma unroll
  for (int j = 0; j < RPW; ++j)
    srow[j] = *((const float4*)(p.S + ((long long)h * p.dv + r0 + warp + 4 * j) * GDN_DK) + lane);
  const float a_h = p.ssm_a[h], dt_h = p.dt_bias[h];

  pdl_wait();
  pdl_trigger();
  if (tid == 0) {
    KT_FIRST(p.trace, 2);
    KT_LAST(p.trace, 3);
  }

  // ---------------- alpha / beta of RMSNorm(x) ----------------
  // alpha = sum_i Wa[i] * (x[i]*scale*w[i]) = scale * sum_i Wa[i]*w[i]*x[i]
  // Every load that depends on the preceding kernel is issued here, before
  // the first barrier, so their L2 round trips overlap.
  const float nq = p.qkv[cq], nk_ = p.qkv[ck];
  const float nv_ = tid < GDN_ROWS ? p.qkv[cv] : 0.f;
  constexpr int XPT = 8;                 // x elements per thread per batch
  float xr[XPT];
#pragma unroll
  for (int j = 0; j < XPT; ++j) {
    const int i = tid + j * GDN_THREADS;
    xr[j] = i < H ? p.x[i] : 0.f;
  }
  __syncthreads();   // smem weights visible
  float acc3[3] = {0.f, 0.f, 0.f};
  for (int i0 = 0; i0 < H; i0 += XPT * GDN_THREADS) {
    if (i0) {
#pragma unroll
      for (int j = 0; j < XPT; ++j) {
        const int i = i0 + tid + j * GDN_THREADS;
        xr[j] = i < H ? p.x[i] : 0.f;
      }
    }
#pragma unroll
    for (int j = 0; j < XPT; ++j) {
      const int i = i0 + tid + j * GDN_THREADS;
      if (i < H) {
        const float xv = xr[j], xw = xv * wn_s[i];
        acc3[0] = fmaf(xv, xv, acc3[0]);
        acc3[1] = fmaf(wa_s[i], xw, acc3[1]);
        acc3[2] = fmaf(wb_s[i], xw, acc3[2]);
      }
    }
  }
  // conv1d + SiLU on this thread's channels (newest input last, :555-564)
  float vq = 0.f, vk = 0.f, vvv = 0.f;
#pragma unroll
  for (int k = 0; k < GDN_MAXK; ++k) {
    if (k < K - 1) {
      vq += hq[k] * wq[k];
      vk += hk[k] * wk[k];
      vvv += hv[k] * wv[k];
    } else if (k == K - 1) {
      vq += nq * wq[k];
      vk += nk_ * wk[k];
      vvv += nv_ * wv[k];
    }
  }
  const float qv = vq / (1.0f + expf(-vq));
  const float kv = vk / (1.0f + expf(-vk));
  if (tid < GDN_ROWS) vrow[tid] = vvv / (1.0f + expf(-vvv));
  // ring update (owners only; no CTA reads slot `cur` in this step)
  if (h == g && blockIdx.y == 0) {
    p.ring[(long long)cur * C + cq] = nq;
    p.ring[(long long)cur * C + ck] = nk_;
  }
  if (tid < GDN_ROWS) p.ring[(long long)cur * C + cv] = nv_;

  // one block reduction for the RMSNorm statistics, alpha / beta and the
  // q / k L2 norms
  float acc5[5] = {acc3[0], acc3[1], acc3[2], qv * qv, kv * kv};
  block_sum_n<5>(acc5, red);
  if (tid == 0) KT_LAST(p.trace, 4);
  const float scale = 1.0f / sqrtf(acc5[0] / (float)H + p.eps);
  const float alpha = acc5[1] * scale, beta_raw = acc5[2] * scale;
  // gates in Float64 (src/ModelCPU.jl:618-636): decay and beta on threads of
  // two different warps, so their double-precision chains run side by side
  if (tid == 0) {
    double a = (double)alpha + (double)dt_h;
    a = fmin(20.0, fmax(-20.0, a));
    const double sp = log(1.0 + exp(a));
    const float decay = (float)((double)a_h * sp);
    gate_s[0] = expf(decay);
  } else if (tid == 32) {
    const double bv = fmin(20.0, fmax(-20.0, (double)beta_raw));
    gate_s[1] = (float)(1.0 / (1.0 + exp(-bv)));
  }
  // ---------------- L2 norms (src/ModelCPU.jl:597-616) ----------------
  const float qk2[2] = {acc5[3], acc5[4]};
  const float qscale = 1.0f / sqrtf((float)GDN_DK);
  const float qnv = 1.0f / (sqrtf(qk2[0]) + 1.0e-6f) * qscale;
  const float knv = 1.0f / (sqrtf(qk2[1]) + 1.0e-6f);
  qn[tid] = qv * qnv;
  kn[tid] = kv * knv;
  __syncthreads();
  if (tid == 0) KT_LAST(p.trace, 5);
  const float dec = gate_s[0], bg = gate_s[1];

  // ---------------- delta rule ----------------
  const float4 k4 = *(const float4*)&kn[lane * 4];
  const float4 q4 = *(const float4*)&qn[lane * 4];
#pragma unroll
  for (int j = 0; j < RPW; ++j) {
    const int rr = warp + 4 * j, i = r0 + rr;
    float4 s = srow[j];
    s.x *= dec; s.y *= dec; s.z *= dec; s.w *= dec;
    const float sk = warp_sum(s.x * k4.x + s.y * k4.y + s.z * k4.z + s.w * k4.w);
    const float d = bg * (vrow[rr] - sk);
    s.x += d * k4.x; s.y += d * k4.y; s.z += d * k4.z; s.w += d * k4.w;
    const float yv = warp_sum(s.x * q4.x + s.y * q4.y + s.z * q4.z + s.w * q4.w);
    *((float4*)(p.S + ((long long)h * p.dv + i) * GDN_DK) + lane) = s;
    if (lane == 0) p.y[h * p.dv + i] = yv;
  }

  // ---------------- advance the layer's step counter ----------------
  if (!p.self_advance) {
    if (tid == 0) KT_LAST(p.trace, 6);
    return;
  }
  __syncthreads();
  if (tid == 0) KT_LAST(p.trace, 7);
  if (tid == 0) {
    __threadfence();
    const int total = gridDim.x * gridDim.y;
    const int prev = atomicAdd(p.done, 1);
    if (prev == total - 1) {
      *p.done = 0;
      *p.step = t + 1;
      __threadfence();
    }
    KT_LAST(p.trace, 6);
  }
}

// ---------------------------------------------------------------------------
// Whole-head variant: one CTA per value head (512 threads) owns the head's
// dv x 128 state, so the per-head output RMSNorm and SiLU(z) gate
// (src/ModelCPU.jl:682-692) happen here and the ssm_out GEMV reads a plain
// input.  Thread (warp w, lane l) holds 32 state values: row w*8 + l/4,
// columns 32*(l%4)..+31; row dot products are 32 FMAs plus two shuffles.
// Channels: threads 0..127 q (group g = h % nk), 128..255 k, 256..256+dv v.
// The step counter is left to the token's finalize kernel.
// ---------------------------------------------------------------------------
constexpr int GH_THREADS = 512;

__global__ void __launch_bounds__(GH_THREADS, 1) gdn_head_kernel(const __grid_constant__ GdnParams p) {
  extern __shared__ __align__(16) float gsm[];     // [3][H]: w_alpha row, w_beta row, in_norm
  __shared__ __align__(16) float qn[GDN_DK], kn[GDN_DK];
  __shared__ float vrow[GDN_DK];
  __shared__ float red[5][GH_THREADS / 32];
  __shared__ float red2[GH_THREADS / 32];
  __shared__ float gate_s[2];
  const int h = blockIdx.x, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int sb = blockIdx.y;                       // sequence (batched decode)
  const float* X = p.x + sb * p.xs;
  const float* QKV = p.qkv + sb * p.qkvs;
  const float* Z = p.z + sb * p.zys;
  float* Y = p.y + sb * p.zys;
  float* SS = p.S + sb * p.Ss;
  float* RING = p.ring + sb * p.rings;
  const int* STEP = p.step + sb * p.steps_stride;
  const int g = h % p.nk, K = p.K, C = p.C, H = p.H, dv = p.dv;
  if (tid == 0) {
    KT_KIND(p.trace, KT_GDN);
    KT_FIRST(p.trace, 1);
  }
  // ---------------- pre-wait: state, weights, conv history ----------------
  const int t = *STEP;
  const int cur = t % K;
  float* wa_s = gsm;
  float* wb_s = gsm + H;
  float* wn_s = gsm + 2 * H;
  for (int i = tid * 4; i < H; i += GH_THREADS * 4) {
    *(float4*)&wa_s[i] = *(const float4*)&p.w_alpha[(long long)h * H + i];
    *(float4*)&wb_s[i] = *(const float4*)&p.w_beta[(long long)h * H + i];
    *(float4*)&wn_s[i] = *(const float4*)&p.in_norm[i];
  }
  const int row = warp * 8 + (lane >> 2), seg = lane & 3;    // state row / 32-column segment
  const bool row_ok = row < dv;
  float4 s[8];
  const float4* srow = (const float4*)(SS + ((long long)h * dv + (row_ok ? row : 0)) * GDN_DK + 32 * seg);
#pragma unroll
  for (int j = 0; j < 8; ++j) s[j] = row_ok ? srow[j] : make_float4(0.f, 0.f, 0.f, 0.f);
  // this thread's conv channel (q, k or v) and its history
  int ch = -1;
  if (tid < GDN_DK) ch = g * GDN_DK + tid;
  else if (tid < 2 * GDN_DK) ch = p.nk * GDN_DK + g * GDN_DK + (tid - GDN_DK);
  else if (tid < 2 * GDN_DK + dv) ch = 2 * p.nk * GDN_DK + h * dv + (tid - 2 * GDN_DK);
  float cw[GDN_MAXK], hist[GDN_MAXK];
#pragma unroll
  for (int k = 0; k < GDN_MAXK; ++k) {
    cw[k] = hist[k] = 0.f;
    if (ch >= 0 && k < K) {
      cw[k] = p.conv_w[(long long)ch * K + k];
      if (k < K - 1) {
        int slot = (t - (K - 1) + k) % K;
        if (slot < 0) slot += K;
        hist[k] = RING[(long long)slot * C + ch];
      }
    }
  }
  const float nw = (row_ok && seg == 0) ? p.out_norm[row] : 0.f;
  const float a_h = p.ssm_a[h], dt_h = p.dt_bias[h];

  pdl_wait();
  pdl_trigger();
  __syncthreads();   // the shared-memory weight rows (other threads' stores) are visible
  if (tid == 0) {
    KT_FIRST(p.trace, 2);
    KT_LAST(p.trace, 3);
  }
  // ---------------- everything that depends on the previous kernels ----------------
  const float xin = ch >= 0 ? QKV[ch] : 0.f;
  const float zr = (row_ok && seg == 0) ? Z[h * dv + row] : 0.f;
  constexpr int XPT = GDN_MAX_H / GH_THREADS;   // x elements per thread (H <= 8192)
  float acc[5] = {0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
  for (int j = 0; j < XPT; ++j) {
    const int i = tid + j * GH_THREADS;
    if (i < H) {
      const float xv = X[i], xw = xv * wn_s[i];
      acc[0] = fmaf(xv, xv, acc[0]);
      acc[1] = fmaf(wa_s[i], xw, acc[1]);
      acc[2] = fmaf(wb_s[i], xw, acc[2]);
    }
  }
  // conv1d + SiLU (newest input last, :555-564)
  float cv = 0.f;
#pragma unroll
  for (int k = 0; k < GDN_MAXK; ++k) {
    if (k < K - 1) cv += hist[k] * cw[k];
    else if (k == K - 1) cv += xin * cw[k];
  }
  const float act = cv / (1.0f + expf(-cv));
  if (tid < GDN_DK) acc[3] = act * act;
  else if (tid < 2 * GDN_DK) acc[4] = act * act;
  else if (ch >= 0) vrow[tid - 2 * GDN_DK] = act;
  // ring update (q / k channels by the group's first head only; no CTA reads slot `cur` in this step)
  if (ch >= 0 && (tid >= 2 * GDN_DK || h == g)) RING[(long long)cur * C + ch] = xin;
#pragma unroll
  for (int i = 0; i < 5; ++i) acc[i] = warp_sum(acc[i]);
  if (lane == 0)
#pragma unroll
    for (int i = 0; i < 5; ++i) red[i][warp] = acc[i];
  __syncthreads();
  float tot[5] = {0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
  for (int w = 0; w < GH_THREADS / 32; ++w)
#pragma unroll
    for (int i = 0; i < 5; ++i) tot[i] += red[i][w];
  if (tid == 0) {
    // gates in Float64 (src/ModelCPU.jl:618-636)
    const float scale = 1.0f / sqrtf(tot[0] / (float)H + p.eps);
    const float alpha = tot[1] * scale, beta_raw = tot[2] * scale;
    double a = (double)alpha + (double)dt_h;
    a = fmin(20.0, fmax(-20.0, a));
    const double sp = log(1.0 + exp(a));
    gate_s[0] = expf((float)((double)a_h * sp));
    const double bv = fmin(20.0, fmax(-20.0, (double)beta_raw));
    gate_s[1] = (float)(1.0 / (1.0 + exp(-bv)));
  }
  // L2 norms (src/ModelCPU.jl:597-616)
  if (tid < GDN_DK) qn[tid] = act * (1.0f / (sqrtf(tot[3]) + 1.0e-6f) * (1.0f / sqrtf((float)GDN_DK)));
  else if (tid < 2 * GDN_DK) kn[tid - GDN_DK] = act * (1.0f / (sqrtf(tot[4]) + 1.0e-6f));
  __syncthreads();
  const float dec = gate_s[0], bg = gate_s[1];
  // ---------------- delta rule on this thread's 32 state values ----------------
  const float4* k4 = (const float4*)&kn[32 * seg];
  const float4* q4 = (const float4*)&qn[32 * seg];
  float sk = 0.f;
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    s[j].x *= dec; s[j].y *= dec; s[j].z *= dec; s[j].w *= dec;
    const float4 kk = k4[j];
    sk = fmaf(s[j].x, kk.x, fmaf(s[j].y, kk.y, fmaf(s[j].z, kk.z, fmaf(s[j].w, kk.w, sk))));
  }
  sk += __shfl_xor_sync(0xffffffffu, sk, 1);
  sk += __shfl_xor_sync(0xffffffffu, sk, 2);
  const float d = bg * ((row_ok ? vrow[row] : 0.f) - sk);
  float y = 0.f;
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const float4 kk = k4[j], qq = q4[j];
    s[j].x = fmaf(d, kk.x, s[j].x); s[j].y = fmaf(d, kk.y, s[j].y);
    s[j].z = fmaf(d, kk.z, s[j].z); s[j].w = fmaf(d, kk.w, s[j].w);
    y = fmaf(s[j].x, qq.x, fmaf(s[j].y, qq.y, fmaf(s[j].z, qq.z, fmaf(s[j].w, qq.w, y))));
  }
  y += __shfl_xor_sync(0xffffffffu, y, 1);
  y += __shfl_xor_sync(0xffffffffu, y, 2);
  if (row_ok) {
    float4* so = (float4*)(SS + ((long long)h * dv + row) * GDN_DK + 32 * seg);
#pragma unroll
    for (int j = 0; j < 8; ++j) so[j] = s[j];
  }
  // ---------------- per-head RMSNorm x SiLU(z) (:682-692) ----------------
  float y2 = (row_ok && seg == 0) ? y * y : 0.f;
  y2 = warp_sum(y2);
  if (lane == 0) red2[warp] = y2;
  __syncthreads();
  float ys = 0.f;
#pragma unroll
  for (int w = 0; w < GH_THREADS / 32; ++w) ys += red2[w];
  if (row_ok && seg == 0) {
    const float sc = 1.0f / sqrtf(ys / (float)dv + p.eps);
    const float v = y * sc * nw;
    Y[h * dv + row] = v * zr * (1.0f / (1.0f + expf(-zr)));
  }
  if (tid == 0) KT_LAST(p.trace, 6);
}

int launch_gdn_head(const GdnParams& p, cudaStream_t st, bool pdl, int nseq) {
  if (p.dv > GDN_DK || p.dv % 8 || p.K < 1 || p.K > GDN_MAXK || p.H % 4 || p.H > GDN_MAX_H || !p.z || !p.out_norm)
    return set_error(INFERNO_EINVAL, "gdn head: unsupported dims (dv=%d, K=%d, H=%d)", p.dv, p.K, p.H);
  static DeviceOnce once;
  cudaError_t ea = once.run([] {
    return cudaFuncSetAttribute(gdn_head_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 3 * GDN_MAX_H * 4);
  });
  if (ea != cudaSuccess) return set_error(INFERNO_ECUDA, "GDN head attribute: %s", cudaGetErrorString(ea));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(p.nv, nseq);
  cfg.blockDim = dim3(GH_THREADS);
  cfg.dynamicSmemBytes = (size_t)3 * p.H * 4;
  cfg.stream = st;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = pdl ? 1 : 0;
  cudaError_t e = cudaLaunchKernelEx(&cfg, gdn_head_kernel, p);
  return e == cudaSuccess ? 0 : set_error(INFERNO_ECUDA, "gdn head launch: %s", cudaGetErrorString(e));
}

int launch_gdn_step(const GdnParams& p, cudaStream_t st, bool pdl) {
  if (p.dv % GDN_ROWS || p.K < 1 || p.K > GDN_MAXK || p.H % 4 || p.H > GDN_MAX_H)
    return set_error(INFERNO_EINVAL, "gdn: unsupported dims (dv=%d, K=%d, H=%d)", p.dv, p.K, p.H);
  static DeviceOnce once;
  cudaError_t ea = once.run([] {
    cudaError_t e = cudaFuncSetAttribute(gdn_step_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 3 * GDN_MAX_H * 4);
    if (e != cudaSuccess) return e;
    return cudaFuncSetAttribute(gdn_step_kernel, cudaFuncAttributePreferredSharedMemoryCarveout,
                                cudaSharedmemCarveoutMaxShared);
  });
  if (ea != cudaSuccess) return set_error(INFERNO_ECUDA, "GDN step attribute: %s", cudaGetErrorString(ea));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(p.nv, p.dv / GDN_ROWS);
  cfg.blockDim = dim3(GDN_THREADS);
  cfg.dynamicSmemBytes = (size_t)3 * p.H * 4;
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
