// Gated full-attention decode step: Q/K RMSNorm + partial RoPE, KV append,
// split-K attention over the HBM KV cache and the sigmoid output gate.
//
// Replaces FullAttentionCPU after its q/k/v GEMVs (Inferno.jl
// src/ModelCPU.jl:756-851): rmsnorm_rotary! (:187-231), update_kv_cache!
// (:245-258), flash_attention_cpu! (src/FlashAttention.jl:16-74, blocked GQA
// head map kv = h / (nq/nkv)) and the gate (:846-851).
//
// Grid (n_kv heads, n_split).  A CTA owns one KV head and one split of
// `split_len` positions and serves all nq/nkv query heads of that KV head, so
// each K/V row is read from HBM once per token.  Softmax is exact per split
// (max, sum of exp) and the last CTA of a KV head (atomic ticket) merges the
// splits: o = sum_s e^{m_s-M} o_s / sum_s e^{m_s-M} l_s, then o *= sigmoid(g).
// The new K/V row at `pos` is normalised/rotated in the CTA whose split holds
// `pos`, used from shared memory and written to the cache by that CTA; no
// other CTA reads position `pos` in the same launch.
//
// Cache layout: [ctx][n_kv][head_dim] fp32 (the reference's (hd, nkv, seq)
// column-major array, element (d, h, p) at d + hd*(h + nkv*p)).
#include "internal.h"
#include "common.cuh"
#include "params.h"
#include "../../include/inferno_b200.h"

namespace inf {

constexpr int ATT_HD = 256;          // head_dim (one thread per dim)
constexpr int ATT_THREADS = 256;
constexpr int ATT_MAX_GQA = 8;
constexpr int ATT_MAX_SPLIT = 256;   // positions per split (scores in smem)



// RMSNorm over 256 dims (one value per thread) + half-split RoPE on the
// first rd dims, in place in smem row `x` (src/ModelCPU.jl:187-231).
__device__ __forceinline__ void norm_rope(float* x, const float* w, float eps, const float* c, const float* s,
                                          int rd, float* red) {
  const int d = threadIdx.x;
  float v = x[d];
  float ss = warp_sum(v * v);
  if ((d & 31) == 0) red[d >> 5] = ss;
  __syncthreads();
  float tot = 0.f;
#pragma unroll
  for (int i = 0; i < ATT_THREADS / 32; ++i) tot += red[i];
  const float inv = 1.0f / sqrtf(tot / (float)ATT_HD + eps);
  v = v * inv * w[d];
  __syncthreads();
  x[d] = v;
  __syncthreads();
  const int half = rd / 2;
  if (d < half) {
    float x1 = x[d], x2 = x[d + half];
    x[d] = x1 * c[d] - x2 * s[d];
    x[d + half] = x1 * s[d] + x2 * c[d];
  }
  __syncthreads();
}

__global__ void __launch_bounds__(ATT_THREADS) attn_decode_kernel(const __grid_constant__ AttnParams p) {
  __shared__ __align__(16) float qs[ATT_MAX_GQA][ATT_HD];
  __shared__ __align__(16) float knew[ATT_HD], vnew[ATT_HD];
  __shared__ float sc[ATT_MAX_GQA][ATT_MAX_SPLIT];
  __shared__ float red[ATT_THREADS / 32];
  __shared__ float ml[ATT_MAX_GQA][2];
  __shared__ int ticket;
  pdl_trigger();
  pdl_wait();
  const int kvh = blockIdx.x, s = blockIdx.y, d = threadIdx.x;
  const int warp = d >> 5, lane = d & 31;
  const int gqa = p.nh / p.nkv;
  const int pos = *p.pos;
  if (pos < 0 || pos >= p.ctx) {
    if (d == 0 && s == 0 && kvh == 0) atomicExch(p.err, DERR_BAD_ARG);
    return;
  }
  const int L = pos + 1;
  const int nact = (L + p.split_len - 1) / p.split_len;
  if (s >= nact) return;
  const int j0 = s * p.split_len, j1 = min(j0 + p.split_len, L);
  const int nj = j1 - j0;
  const int half = p.rd / 2;
  const float* cs = p.rope_cos + (long long)pos * half;
  const float* sn = p.rope_sin + (long long)pos * half;
  const float scale = 1.0f / sqrtf((float)ATT_HD);

  // query heads of this KV head (blocked GQA, src/ModelCPU.jl:790-795)
  for (int i = 0; i < gqa; ++i) {
    const int qh = kvh * gqa + i;
    qs[i][d] = p.qg[(long long)qh * 2 * ATT_HD + d];
    __syncthreads();
    norm_rope(qs[i], p.q_norm, p.eps, cs, sn, p.rd, red);
  }
  const bool has_new = (pos >= j0 && pos < j1);
  if (has_new) {
    knew[d] = p.k[kvh * ATT_HD + d];
    vnew[d] = p.v[kvh * ATT_HD + d];
    __syncthreads();
    norm_rope(knew, p.k_norm, p.eps, cs, sn, p.rd, red);
    long long off = ((long long)pos * p.nkv + kvh) * ATT_HD + d;
    p.kc[off] = knew[d];
    p.vc[off] = vnew[d];
  }

  // scores: one warp per key, 8 dims per lane
#pragma unroll 4
  for (int jj = warp; jj < nj; jj += ATT_THREADS / 32) {
    const int j = j0 + jj;
    const float* kr = (j == pos) ? knew : p.kc + ((long long)j * p.nkv + kvh) * ATT_HD;
    const float4 k0 = *(const float4*)(kr + lane * 8), k1 = *(const float4*)(kr + lane * 8 + 4);
    for (int i = 0; i < gqa; ++i) {
      const float4 q0 = *(const float4*)(&qs[i][lane * 8]), q1 = *(const float4*)(&qs[i][lane * 8 + 4]);
      float a = q0.x * k0.x + q0.y * k0.y + q0.z * k0.z + q0.w * k0.w + q1.x * k1.x + q1.y * k1.y +
                q1.z * k1.z + q1.w * k1.w;
      a = warp_sum(a);
      if (lane == 0) sc[i][jj] = a * scale;
    }
  }
  __syncthreads();
  // per-head softmax statistics of this split (warp i owns head i)
  for (int i = warp; i < gqa; i += ATT_THREADS / 32) {
    float m = -INFINITY;
    for (int jj = lane; jj < nj; jj += 32) m = fmaxf(m, sc[i][jj]);
    m = warp_max(m);
    float l = 0.f;
    for (int jj = lane; jj < nj; jj += 32) {
      float e = expf(sc[i][jj] - m);
      sc[i][jj] = e;
      l += e;
    }
    l = warp_sum(l);
    if (lane == 0) { ml[i][0] = m; ml[i][1] = l; }
  }
  __syncthreads();
  // o[i][d] = sum_j p[i][j] v[j][d]
  float o[ATT_MAX_GQA];
#pragma unroll
  for (int i = 0; i < ATT_MAX_GQA; ++i) o[i] = 0.f;
#pragma unroll 8
  for (int jj = 0; jj < nj; ++jj) {
    const int j = j0 + jj;
    const float vv = (j == pos) ? vnew[d] : p.vc[((long long)j * p.nkv + kvh) * ATT_HD + d];
#pragma unroll
    for (int i = 0; i < ATT_MAX_GQA; ++i)
      if (i < gqa) o[i] = fmaf(sc[i][jj], vv, o[i]);
  }
#pragma unroll
  for (int i = 0; i < ATT_MAX_GQA; ++i) {
    if (i >= gqa) break;
    const int qh = kvh * gqa + i;
    p.part_o[((long long)qh * p.nsplit + s) * ATT_HD + d] = o[i];
    if (d == 0) {
      p.part_ml[((long long)qh * p.nsplit + s) * 2 + 0] = ml[i][0];
      p.part_ml[((long long)qh * p.nsplit + s) * 2 + 1] = ml[i][1];
    }
  }

  // ---- last CTA of this KV head merges the splits ----
  __threadfence();
  __syncthreads();
  if (d == 0) ticket = atomicAdd(&p.counters[kvh], 1);
  __syncthreads();
  if (ticket != nact - 1) return;
  __threadfence();
  if (d == 0) p.counters[kvh] = 0;
  for (int i = 0; i < gqa; ++i) {
    const int qh = kvh * gqa + i;
    const float* mlp = p.part_ml + (long long)qh * p.nsplit * 2;
    float M = -INFINITY;
    for (int t = 0; t < nact; ++t) M = fmaxf(M, __ldcg(mlp + 2 * t));
    float num = 0.f, den = 0.f;
    for (int t = 0; t < nact; ++t) {
      const float w = expf(__ldcg(mlp + 2 * t) - M);
      num = fmaf(w, __ldcg(p.part_o + ((long long)qh * p.nsplit + t) * ATT_HD + d), num);
      den = fmaf(w, __ldcg(mlp + 2 * t + 1), den);
    }
    const float g = p.qg[(long long)qh * 2 * ATT_HD + ATT_HD + d];
    const float gate = 1.0f / (1.0f + expf(-g));
    p.out[(long long)qh * ATT_HD + d] = (num / den) * gate;
  }
}

int launch_attn_decode(const AttnParams& p, cudaStream_t st, bool pdl) {
  if (p.nh % p.nkv || p.nh / p.nkv > ATT_MAX_GQA || p.split_len > ATT_MAX_SPLIT || p.split_len < 1 ||
      p.rd > ATT_HD || p.rd % 2)
    return set_error(INFERNO_EINVAL, "attention: unsupported shape (nh=%d nkv=%d split=%d rd=%d)", p.nh, p.nkv,
                     p.split_len, p.rd);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(p.nkv, p.nsplit);
  cfg.blockDim = dim3(ATT_THREADS);
  cfg.stream = st;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = pdl ? 1 : 0;
  cudaError_t e = cudaLaunchKernelEx(&cfg, attn_decode_kernel, p);
  return e == cudaSuccess ? 0 : set_error(INFERNO_ECUDA, "attention launch: %s", cudaGetErrorString(e));
}

}  // namespace inf
