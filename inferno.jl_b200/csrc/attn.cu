// Gated full-attention decode step: Q/K RMSNorm + partial RoPE, KV append,
// split-K attention over the HBM KV cache and the sigmoid output gate.
//
// Replaces FullAttentionCPU after its q/k/v GEMVs (Inferno.jl
// src/ModelCPU.jl:756-851): rmsnorm_rotary! (:187-231), update_kv_cache!
// (:245-258), flash_attention_cpu! (src/FlashAttention.jl:16-74, blocked GQA
// head map kv = h / (nq/nkv)) and the gate (:846-851).
//
// Grid (n_heads, n_split), 256 threads (one per head dim).  A CTA owns one
// query head and one split of `split_len` positions, processed in chunks of
// 32 keys: 8 threads per key compute the q.k partial dots, the chunk's
// softmax statistics are folded into a running (max, sum, o) online softmax,
// and each thread accumulates one output dim from the V rows.  The last CTA
// of a head (atomic ticket) merges the splits,
//   o = sum_s e^{m_s-M} o_s / sum_s e^{m_s-M} l_s,  then  o *= sigmoid(g).
// The first chunk's K/V rows (all positions < pos) are loaded before
// griddepcontrol.wait; the new row at `pos` is normalised / rotated from the
// q/k/v GEMV output, used from shared memory and written to the cache by one
// CTA per KV head.
//
// Cache layout: [ctx][n_kv][head_dim] fp32 (the reference's (hd, nkv, seq)
// column-major array, element (d, h, p) at d + hd*(h + nkv*p)).
#include <cmath>
#include <vector>
#include "internal.h"
#include "common.cuh"
#include "params.h"
#include "../../include/inferno_b200.h"

namespace inf {

constexpr int ATT_HD = 256;          // head_dim (one thread per dim)
constexpr int ATT_THREADS = 256;
constexpr int ATT_CHUNK = 32;        // keys per pass (8 threads per key)

__device__ __forceinline__ void load_chunk(const AttnParams& p, const float* KC, const float* VC, int kvh, int j0,
                                           int jend, int pos, float4 (&kreg)[8], float (&vreg)[ATT_CHUNK]) {
  const int t = threadIdx.x, kk = t >> 3, part = t & 7;
  const int j = j0 + kk;
  if (j < jend && j != pos) {
    const float4* kr = (const float4*)(KC + ((long long)j * p.nkv + kvh) * ATT_HD + part * 32);
#pragma unroll
    for (int i = 0; i < 8; ++i) kreg[i] = kr[i];
  } else {
#pragma unroll
    for (int i = 0; i < 8; ++i) kreg[i] = make_float4(0.f, 0.f, 0.f, 0.f);
  }
#pragma unroll
  for (int q = 0; q < ATT_CHUNK; ++q) {
    const int jj = j0 + q;
    vreg[q] = (jj < jend && jj != pos) ? VC[((long long)jj * p.nkv + kvh) * ATT_HD + t] : 0.f;
  }
}

__global__ void __launch_bounds__(ATT_THREADS) attn_decode_kernel(const __grid_constant__ AttnParams p) {
  __shared__ __align__(16) float qs[ATT_HD], knew[ATT_HD], vnew[ATT_HD];
  __shared__ float qraw[ATT_HD], kraw[ATT_HD];
  __shared__ float sc[ATT_CHUNK];
  __shared__ float red[2][ATT_THREADS / 32];
  __shared__ int ticket;
  const int h = blockIdx.x, s = blockIdx.y, d = threadIdx.x;
  const int sq = blockIdx.z;                       // sequence (batched decode)
  float* KC = p.kc + sq * p.caches;
  float* VC = p.vc + sq * p.caches;
  const float* QG = p.qg + sq * p.qgs;
  const float* KN = p.k + sq * p.kvs;
  const float* VN = p.v + sq * p.kvs;
  float* PO = p.part_o + (long long)sq * p.nh * p.nsplit * ATT_HD;
  float* PML = p.part_ml + (long long)sq * p.nh * p.nsplit * 2;
  int* CNT = p.counters + (long long)sq * p.nh;
  const int kvh = h / (p.nh / p.nkv);
  const int lane = d & 31, warp = d >> 5;
  if (d == 0) {
    KT_KIND(p.trace, KT_ATTN);
    KT_FIRST(p.trace, 1);
  }

  // ---------------- pre-wait: position and the first K/V chunk ----------------
  const int pos = p.pos[sq];     // written by the previous step's finalize
  if (pos < 0 || pos >= p.ctx) {
    pdl_wait();
    pdl_trigger();
    if (d == 0 && s == 0 && h == 0) atomicExch(p.err, DERR_BAD_ARG);
    return;
  }
  const int L = pos + 1;
  const int nact = (L + p.split_len - 1) / p.split_len;
  const int j0 = s * p.split_len, j1 = min(j0 + p.split_len, L);
  float4 kreg[8];
  float vreg[ATT_CHUNK];
  if (s < nact) load_chunk(p, KC, VC, kvh, j0, min(j0 + ATT_CHUNK, j1), pos, kreg, vreg);
  // constants of the norm + RoPE of this thread's dim d and its rotation
  // partner (d +- rd/2), loaded before the wait
  const int half = p.rd / 2;
  const bool rot = d < 2 * half;
  const int pd = d < half ? d + half : d - half;
  const float wq_d = p.q_norm[d], wk_d = p.k_norm[d];
  const float wq_p = rot ? p.q_norm[pd] : 0.f, wk_p = rot ? p.k_norm[pd] : 0.f;
  const int ri = d < half ? d : pd;
  const float rc = rot ? p.rope_cos[(long long)pos * half + ri] : 1.f;
  const float rs = rot ? p.rope_sin[(long long)pos * half + ri] : 0.f;
  pdl_wait();
  pdl_trigger();
  if (d == 0) {
    KT_FIRST(p.trace, 2);
    KT_LAST(p.trace, 3);
  }
  if (s >= nact) return;

  // ---------------- q (and the new k) : RMSNorm + RoPE ----------------
  const bool has_new = (pos >= j0 && pos < j1);
  const float qv = QG[(long long)h * 2 * ATT_HD + d];
  const float kv = has_new ? KN[kvh * ATT_HD + d] : 0.f;
  if (has_new) vnew[d] = VN[kvh * ATT_HD + d];
  qraw[d] = qv;
  kraw[d] = kv;
  float a = warp_sum(qv * qv), b = warp_sum(kv * kv);
  if (lane == 0) { red[0][warp] = a; red[1][warp] = b; }
  __syncthreads();
  a = 0.f;
  b = 0.f;
#pragma unroll
  for (int i = 0; i < ATT_THREADS / 32; ++i) { a += red[0][i]; b += red[1][i]; }
  const float iq = 1.0f / sqrtf(a / (float)ATT_HD + p.eps);
  const float ik = 1.0f / sqrtf(b / (float)ATT_HD + p.eps);
  // normalised values of d and of its partner, rotated (x1 = first half,
  // x2 = second half: x1' = x1 c - x2 s, x2' = x1 s + x2 c)
  {
    const float nq = qv * iq * wq_d, nk = kv * ik * wk_d;
    float qo = nq, ko = nk;
    if (rot) {
      const float pq = qraw[pd] * iq * wq_p, pk = kraw[pd] * ik * wk_p;
      if (d < half) {
        qo = nq * rc - pq * rs;
        ko = nk * rc - pk * rs;
      } else {
        qo = pq * rs + nq * rc;
        ko = pk * rs + nk * rc;
      }
    }
    qs[d] = qo;
    if (has_new) knew[d] = ko;
  }
  __syncthreads();
  if (has_new && (h % (p.nh / p.nkv)) == 0) {
    const long long off = ((long long)pos * p.nkv + kvh) * ATT_HD + d;
    KC[off] = knew[d];
    VC[off] = vnew[d];
  }

  if (d == 0) KT_LAST(p.trace, 4);
  // ---------------- online softmax over 32-key chunks ----------------
  const float scale = 1.0f / sqrtf((float)ATT_HD);
  const int kk = d >> 3, part = d & 7;
  float4 q8[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) q8[i] = *(const float4*)&qs[part * 32 + 4 * i];
  float m = -INFINITY, l = 0.f, o = 0.f;
  float4 kreg2[8];
  float vreg2[ATT_CHUNK];
  for (int c0 = j0; c0 < j1; c0 += ATT_CHUNK) {
    const int cend = min(c0 + ATT_CHUNK, j1);
    if (c0 != j0) {
#pragma unroll
      for (int i = 0; i < 8; ++i) kreg[i] = kreg2[i];
#pragma unroll
      for (int q = 0; q < ATT_CHUNK; ++q) vreg[q] = vreg2[q];
    }
    // the next chunk's K/V rows are in flight while this chunk is computed
    if (c0 + ATT_CHUNK < j1) load_chunk(p, KC, VC, kvh, c0 + ATT_CHUNK, min(c0 + 2 * ATT_CHUNK, j1), pos, kreg2, vreg2);
    // the new row at pos comes from shared memory
    if (c0 + kk == pos) {
#pragma unroll
      for (int i = 0; i < 8; ++i) kreg[i] = *(const float4*)&knew[part * 32 + 4 * i];
    }
    float dot = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i)
      dot += q8[i].x * kreg[i].x + q8[i].y * kreg[i].y + q8[i].z * kreg[i].z + q8[i].w * kreg[i].w;
    dot += __shfl_xor_sync(0xffffffffu, dot, 4);
    dot += __shfl_xor_sync(0xffffffffu, dot, 2);
    dot += __shfl_xor_sync(0xffffffffu, dot, 1);
    __syncthreads();   // previous chunk's sc[] consumed
    if (part == 0) sc[kk] = (c0 + kk < cend) ? dot * scale : -INFINITY;
    __syncthreads();
    float cm = -INFINITY;
#pragma unroll
    for (int q = 0; q < ATT_CHUNK; ++q) cm = fmaxf(cm, sc[q]);
    const float mn = fmaxf(m, cm);
    const float corr = expf(m - mn);        // 0 on the first chunk (m = -inf)
    l *= corr;
    o *= corr;
#pragma unroll
    for (int q = 0; q < ATT_CHUNK; ++q) {
      const float e = expf(sc[q] - mn);
      l += e;
      const float vv = (c0 + q == pos) ? vnew[d] : vreg[q];
      o = fmaf(e, vv, o);
    }
    m = mn;
  }
  if (d == 0) KT_LAST(p.trace, 5);
  PO[((long long)h * p.nsplit + s) * ATT_HD + d] = o;
  if (d == 0) {
    PML[((long long)h * p.nsplit + s) * 2 + 0] = m;
    PML[((long long)h * p.nsplit + s) * 2 + 1] = l;
  }

  // ---------------- last CTA of this head merges the splits ----------------
  __threadfence();
  __syncthreads();
  if (d == 0) ticket = atomicAdd(&CNT[h], 1);
  __syncthreads();
  if (d == 0) KT_LAST(p.trace, 6);
  if (ticket != nact - 1) return;
  __threadfence();
  if (d == 0) CNT[h] = 0;
  const float* mlp = PML + (long long)h * p.nsplit * 2;
  float M = -INFINITY;
#pragma unroll 8
  for (int t = 0; t < nact; ++t) M = fmaxf(M, __ldcg(mlp + 2 * t));
  float num = 0.f, den = 0.f;
#pragma unroll 8
  for (int t = 0; t < nact; ++t) {
    const float w = expf(__ldcg(mlp + 2 * t) - M);
    num = fmaf(w, __ldcg(PO + ((long long)h * p.nsplit + t) * ATT_HD + d), num);
    den = fmaf(w, __ldcg(mlp + 2 * t + 1), den);
  }
  const float g = QG[(long long)h * 2 * ATT_HD + ATT_HD + d];
  p.out[sq * p.outs + (long long)h * ATT_HD + d] = (num / den) * (1.0f / (1.0f + expf(-g)));
  if (d == 0) KT_LAST(p.trace, 6);
}

// GQA-grouped variant: one CTA per (KV head, split, sequence) serves the G
// query heads of that KV head (blocked map h = kvh * G + gi), so every K/V row
// of the split is read once per KV head instead of once per query head.  Per
// head the arithmetic is that of attn_decode_kernel (same dots, same online
// softmax, same merge), so both produce the same bits.
template <int G>
__global__ void __launch_bounds__(ATT_THREADS) attn_decode_group_kernel(const __grid_constant__ AttnParams p) {
  __shared__ __align__(16) float qs[G][ATT_HD];
  __shared__ __align__(16) float knew[ATT_HD], vnew[ATT_HD];
  __shared__ float qraw[G][ATT_HD], kraw[ATT_HD];
  __shared__ float sc[G][ATT_CHUNK];
  __shared__ float red[G + 1][ATT_THREADS / 32];
  __shared__ int ticket;
  const int kvh = blockIdx.x, s = blockIdx.y, d = threadIdx.x;
  const int sq = blockIdx.z;                       // sequence (batched decode)
  float* KC = p.kc + sq * p.caches;
  float* VC = p.vc + sq * p.caches;
  const float* QG = p.qg + sq * p.qgs;
  const float* KN = p.k + sq * p.kvs;
  const float* VN = p.v + sq * p.kvs;
  float* PO = p.part_o + (long long)sq * p.nh * p.nsplit * ATT_HD;
  float* PML = p.part_ml + (long long)sq * p.nh * p.nsplit * 2;
  int* CNT = p.counters + (long long)sq * p.nh;
  const int h0 = kvh * G;
  const int lane = d & 31, warp = d >> 5;
  if (d == 0) {
    KT_KIND(p.trace, KT_ATTN);
    KT_FIRST(p.trace, 1);
  }

  // ---------------- pre-wait: position, the first K/V chunk, constants ----------------
  const int pos = p.pos[sq];
  if (pos < 0 || pos >= p.ctx) {
    pdl_wait();
    pdl_trigger();
    if (d == 0 && s == 0 && kvh == 0) atomicExch(p.err, DERR_BAD_ARG);
    return;
  }
  const int L = pos + 1;
  const int nact = (L + p.split_len - 1) / p.split_len;
  const int j0 = s * p.split_len, j1 = min(j0 + p.split_len, L);
  float4 kreg[8];
  float vreg[ATT_CHUNK];
  if (s < nact) load_chunk(p, KC, VC, kvh, j0, min(j0 + ATT_CHUNK, j1), pos, kreg, vreg);
  const int half = p.rd / 2;
  const bool rot = d < 2 * half;
  const int pd = d < half ? d + half : d - half;
  const float wq_d = p.q_norm[d], wk_d = p.k_norm[d];
  const float wq_p = rot ? p.q_norm[pd] : 0.f, wk_p = rot ? p.k_norm[pd] : 0.f;
  const int ri = d < half ? d : pd;
  const float rc = rot ? p.rope_cos[(long long)pos * half + ri] : 1.f;
  const float rs = rot ? p.rope_sin[(long long)pos * half + ri] : 0.f;
  pdl_wait();
  pdl_trigger();
  if (d == 0) {
    KT_FIRST(p.trace, 2);
    KT_LAST(p.trace, 3);
  }
  if (s >= nact) return;

  // ---------------- the G query heads (and the new k): RMSNorm + RoPE ----------------
  const bool has_new = (pos >= j0 && pos < j1);
  float qv[G];
#pragma unroll
  for (int gi = 0; gi < G; ++gi) {
    qv[gi] = QG[(long long)(h0 + gi) * 2 * ATT_HD + d];
    qraw[gi][d] = qv[gi];
  }
  const float kv = has_new ? KN[kvh * ATT_HD + d] : 0.f;
  if (has_new) vnew[d] = VN[kvh * ATT_HD + d];
  kraw[d] = kv;
  {
    float a[G];
#pragma unroll
    for (int gi = 0; gi < G; ++gi) a[gi] = warp_sum(qv[gi] * qv[gi]);
    const float b = warp_sum(kv * kv);
    if (lane == 0) {
#pragma unroll
      for (int gi = 0; gi < G; ++gi) red[gi][warp] = a[gi];
      red[G][warp] = b;
    }
  }
  __syncthreads();
  float b = 0.f;
#pragma unroll
  for (int i = 0; i < ATT_THREADS / 32; ++i) b += red[G][i];
  const float ik = 1.0f / sqrtf(b / (float)ATT_HD + p.eps);
#pragma unroll
  for (int gi = 0; gi < G; ++gi) {
    float a = 0.f;
#pragma unroll
    for (int i = 0; i < ATT_THREADS / 32; ++i) a += red[gi][i];
    const float iq = 1.0f / sqrtf(a / (float)ATT_HD + p.eps);
    const float nq = qv[gi] * iq * wq_d;
    float qo = nq;
    if (rot) {
      const float pq = qraw[gi][pd] * iq * wq_p;
      qo = d < half ? nq * rc - pq * rs : pq * rs + nq * rc;
    }
    qs[gi][d] = qo;
  }
  if (has_new) {
    const float nk = kv * ik * wk_d;
    float ko = nk;
    if (rot) {
      const float pk = kraw[pd] * ik * wk_p;
      ko = d < half ? nk * rc - pk * rs : pk * rs + nk * rc;
    }
    knew[d] = ko;
  }
  __syncthreads();
  if (has_new) {
    const long long off = ((long long)pos * p.nkv + kvh) * ATT_HD + d;
    KC[off] = knew[d];
    VC[off] = vnew[d];
  }

  // ---------------- online softmax over 32-key chunks, G heads ----------------
  const float scale = 1.0f / sqrtf((float)ATT_HD);
  const int kk = d >> 3, part = d & 7;
  float m[G], l[G], o[G];
#pragma unroll
  for (int gi = 0; gi < G; ++gi) {
    m[gi] = -INFINITY;
    l[gi] = 0.f;
    o[gi] = 0.f;
  }
  float4 kreg2[8];
  float vreg2[ATT_CHUNK];
  for (int c0 = j0; c0 < j1; c0 += ATT_CHUNK) {
    const int cend = min(c0 + ATT_CHUNK, j1);
    if (c0 != j0) {
#pragma unroll
      for (int i = 0; i < 8; ++i) kreg[i] = kreg2[i];
#pragma unroll
      for (int q = 0; q < ATT_CHUNK; ++q) vreg[q] = vreg2[q];
    }
    // the next chunk's K/V rows are in flight while this chunk is computed
    if (c0 + ATT_CHUNK < j1) load_chunk(p, KC, VC, kvh, c0 + ATT_CHUNK, min(c0 + 2 * ATT_CHUNK, j1), pos, kreg2, vreg2);
    if (c0 + kk == pos) {
#pragma unroll
      for (int i = 0; i < 8; ++i) kreg[i] = *(const float4*)&knew[part * 32 + 4 * i];
    }
    float dots[G];
#pragma unroll
    for (int gi = 0; gi < G; ++gi) {
      float dot = 0.f;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float4 q4 = *(const float4*)&qs[gi][part * 32 + 4 * i];
        dot += q4.x * kreg[i].x + q4.y * kreg[i].y + q4.z * kreg[i].z + q4.w * kreg[i].w;
      }
      dot += __shfl_xor_sync(0xffffffffu, dot, 4);
      dot += __shfl_xor_sync(0xffffffffu, dot, 2);
      dot += __shfl_xor_sync(0xffffffffu, dot, 1);
      dots[gi] = dot;
    }
    __syncthreads();   // previous chunk's sc[] consumed
    if (part == 0)
#pragma unroll
      for (int gi = 0; gi < G; ++gi) sc[gi][kk] = (c0 + kk < cend) ? dots[gi] * scale : -INFINITY;
    __syncthreads();
#pragma unroll
    for (int gi = 0; gi < G; ++gi) {
      float cm = -INFINITY;
#pragma unroll
      for (int q = 0; q < ATT_CHUNK; ++q) cm = fmaxf(cm, sc[gi][q]);
      const float mn = fmaxf(m[gi], cm);
      const float corr = expf(m[gi] - mn);
      l[gi] *= corr;
      o[gi] *= corr;
#pragma unroll
      for (int q = 0; q < ATT_CHUNK; ++q) {
        const float e = expf(sc[gi][q] - mn);
        l[gi] += e;
        const float vv = (c0 + q == pos) ? vnew[d] : vreg[q];
        o[gi] = fmaf(e, vv, o[gi]);
      }
      m[gi] = mn;
    }
  }
  if (d == 0) KT_LAST(p.trace, 5);
#pragma unroll
  for (int gi = 0; gi < G; ++gi) {
    const int h = h0 + gi;
    PO[((long long)h * p.nsplit + s) * ATT_HD + d] = o[gi];
    if (d == 0) {
      PML[((long long)h * p.nsplit + s) * 2 + 0] = m[gi];
      PML[((long long)h * p.nsplit + s) * 2 + 1] = l[gi];
    }
  }

  // ---------------- last CTA of this KV head merges the splits ----------------
  __threadfence();
  __syncthreads();
  if (d == 0) ticket = atomicAdd(&CNT[kvh], 1);
  __syncthreads();
  if (ticket != nact - 1) return;
  __threadfence();
  if (d == 0) CNT[kvh] = 0;
#pragma unroll
  for (int gi = 0; gi < G; ++gi) {
    const int h = h0 + gi;
    const float* mlp = PML + (long long)h * p.nsplit * 2;
    float M = -INFINITY;
#pragma unroll 8
  #pragma unroll 8
  for (int t = 0; t < nact; ++t) M = fmaxf(M, __ldcg(mlp + 2 * t));
    float num = 0.f, den = 0.f;
#pragma unroll 8
    for (int t = 0; t < nact; ++t) {
      const float w = expf(__ldcg(mlp + 2 * t) - M);
      num = fmaf(w, __ldcg(PO + ((long long)h * p.nsplit + t) * ATT_HD + d), num);
      den = fmaf(w, __ldcg(mlp + 2 * t + 1), den);
    }
    const float g = QG[(long long)h * 2 * ATT_HD + ATT_HD + d];
    p.out[sq * p.outs + (long long)h * ATT_HD + d] = (num / den) * (1.0f / (1.0f + expf(-g)));
  }
  if (d == 0) KT_LAST(p.trace, 6);
}

template <int G>
cudaError_t launch_attn_group(const AttnParams& p, cudaStream_t st, bool pdl, int nseq) {
  static DeviceOnce once;
  cudaError_t ea = once.run([] {
    return cudaFuncSetAttribute(attn_decode_group_kernel<G>, cudaFuncAttributePreferredSharedMemoryCarveout,
                                cudaSharedmemCarveoutMaxShared);
  });
  if (ea != cudaSuccess) return ea;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(p.nkv, p.nsplit, nseq);
  cfg.blockDim = dim3(ATT_THREADS);
  cfg.stream = st;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, attn_decode_group_kernel<G>, p);
}

int launch_attn_decode(const AttnParams& p, cudaStream_t st, bool pdl, int nseq) {
  if (p.nh % p.nkv || p.split_len % ATT_CHUNK || p.split_len < ATT_CHUNK || p.rd > ATT_HD || p.rd % 2)
    return set_error(INFERNO_EINVAL, "attention: unsupported shape (nh=%d nkv=%d split=%d rd=%d)", p.nh, p.nkv,
                     p.split_len, p.rd);
  static DeviceOnce once;
  cudaError_t ea = once.run([] {
    return cudaFuncSetAttribute(attn_decode_kernel, cudaFuncAttributePreferredSharedMemoryCarveout,
                                cudaSharedmemCarveoutMaxShared);
  });
  if (ea != cudaSuccess) return set_error(INFERNO_ECUDA, "attention attribute: %s", cudaGetErrorString(ea));
  // GQA groups of 2, 4 or 8 query heads sharing one CTA per KV head
  // (INFERNO_ATT_GROUPED=1).  The choice is made when the graph is captured,
  // the position only on the device: grouping wins once a layer's KV has
  // outgrown L2 (config 4 at position 30000 of a 32K cache: 5.17 vs 5.59
  // ms/token) but loses while the rows still come from L2 (config 4 at
  // position ~2300 of the same cache: 297 vs 342 tokens/s; config 1 at a
  // 512-position cache: 1511 vs 1676), so one CTA per query head is the
  // default.
  const char* eg = getenv("INFERNO_ATT_GROUPED");      // read per launch (tests switch it)
  const int env_grouped = eg ? atoi(eg) : 0;
  const int G = p.nh / p.nkv;
  const bool grouped = env_grouped != 0;
  if (grouped && (G == 2 || G == 4 || G == 8)) {
    const cudaError_t e = G == 2 ? launch_attn_group<2>(p, st, pdl, nseq)
                          : G == 4 ? launch_attn_group<4>(p, st, pdl, nseq)
                                   : launch_attn_group<8>(p, st, pdl, nseq);
    return e == cudaSuccess ? 0 : set_error(INFERNO_ECUDA, "attention launch: %s", cudaGetErrorString(e));
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(p.nh, p.nsplit, nseq);
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

namespace inf {

void build_rope(int ctx, int rd, float theta, std::vector<float>& cs, std::vector<float>& sn) {
  // src/ModelCPU.jl:134-153: inv_freq in Float64 rounded to Float32, angle in
  // Float32, cos/sin of that Float32 angle (correctly rounded here).
  const int half = rd / 2;
  cs.assign((size_t)ctx * half, 0.f);
  sn.assign((size_t)ctx * half, 0.f);
  for (int i = 0; i < half; ++i) {
    float inv = (float)(1.0 / std::pow((double)theta, (2.0 * i) / (double)rd));
    for (int p = 0; p < ctx; ++p) {
      float f = inv * (float)p;
      cs[(size_t)p * half + i] = (float)std::cos((double)f);
      sn[(size_t)p * half + i] = (float)std::sin((double)f);
    }
  }
}

int attn_split_len(int max_ctx) {
  int sl = ATT_CHUNK;
  while ((max_ctx + sl - 1) / sl > 128) sl += ATT_CHUNK;
  return sl;
}

}  // namespace inf

using namespace inf;

extern "C" int inferno_attention_step(const float* qg, const float* k, const float* v, const float* q_norm,
                                      const float* k_norm, float eps, int n_heads, int n_kv_heads, int head_dim,
                                      int rope_dim, float rope_theta, float* k_cache, float* v_cache, int max_ctx,
                                      int pos, int split_len, float* out, void* stream) {
  if (!qg || !k || !v || !q_norm || !k_norm || !k_cache || !v_cache || !out)
    return set_error(INFERNO_EINVAL, "attention_step: null pointer");
  if (head_dim != ATT_HD) return set_error(INFERNO_EINVAL, "attention_step: head_dim must be %d", ATT_HD);
  if (n_heads < 1 || n_kv_heads < 1 || n_heads % n_kv_heads || rope_dim < 0 || rope_dim > head_dim || rope_dim % 2)
    return set_error(INFERNO_EINVAL, "attention_step: bad heads (%d / %d) or rope_dim %d", n_heads, n_kv_heads,
                     rope_dim);
  if (max_ctx < 1 || pos < 0 || pos >= max_ctx)
    return set_error(INFERNO_EINVAL, "attention_step: pos %d outside [0, %d)", pos, max_ctx);
  if (split_len == 0) split_len = attn_split_len(max_ctx);
  if (split_len < ATT_CHUNK || split_len % ATT_CHUNK)
    return set_error(INFERNO_EINVAL, "attention_step: split_len %d is not a positive multiple of %d", split_len,
                     ATT_CHUNK);
  cudaStream_t st = (cudaStream_t)stream;
  int dev = 0;
  INF_CUDA_TRY(cudaGetDevice(&dev));
  // RoPE rows 0..pos (the kernel reads row pos) and the split-K scratch
  std::vector<float> cs, sn;
  const int half = rope_dim / 2;
  build_rope(pos + 1, rope_dim, rope_theta, cs, sn);
  const int nsplit = (max_ctx + split_len - 1) / split_len;
  const size_t n_rope = (size_t)(pos + 1) * half, n_po = (size_t)n_heads * nsplit * ATT_HD,
               n_ml = (size_t)n_heads * nsplit * 2;
  const size_t bytes = (2 * n_rope + n_po + n_ml) * 4 + (size_t)(n_heads + 1) * 4 + 256;
  char* scratch = nullptr;
  INF_CUDA_TRY(cudaMallocAsync((void**)&scratch, bytes, st));
  float* rc = (float*)scratch;
  float* rs = rc + n_rope;
  float* po = rs + n_rope;
  float* ml = po + n_po;
  int* counters = (int*)(ml + n_ml);
  int* dpos = counters + n_heads;
  int rc_ = 0;
  cudaError_t e = cudaSuccess;
  if (n_rope) {
    e = cudaMemcpyAsync(rc, cs.data(), n_rope * 4, cudaMemcpyHostToDevice, st);
    if (e == cudaSuccess) e = cudaMemcpyAsync(rs, sn.data(), n_rope * 4, cudaMemcpyHostToDevice, st);
  }
  if (e == cudaSuccess) e = cudaMemsetAsync(counters, 0, (size_t)n_heads * 4, st);
  if (e == cudaSuccess) e = cudaMemcpyAsync(dpos, &pos, 4, cudaMemcpyHostToDevice, st);
  if (e != cudaSuccess) rc_ = set_error(INFERNO_ECUDA, "attention_step set-up: %s", cudaGetErrorString(e));
  if (!rc_) {
    AttnParams a{};
    a.qg = qg;
    a.k = k;
    a.v = v;
    a.q_norm = q_norm;
    a.k_norm = k_norm;
    a.eps = eps;
    a.rope_cos = rc;
    a.rope_sin = rs;
    a.rd = rope_dim;
    a.kc = k_cache;
    a.vc = v_cache;
    a.nh = n_heads;
    a.nkv = n_kv_heads;
    a.ctx = max_ctx;
    a.split_len = split_len;
    a.nsplit = nsplit;
    a.pos = dpos;
    a.part_o = po;
    a.part_ml = ml;
    a.counters = counters;
    a.out = out;
    a.err = device_error_word(dev);
    rc_ = launch_attn_decode(a, st, false);
  }
  // the host vectors must outlive the copies: wait before returning
  cudaError_t ef = cudaFreeAsync(scratch, st);
  cudaError_t es = cudaStreamSynchronize(st);
  if (rc_) return rc_;
  if (ef != cudaSuccess || es != cudaSuccess)
    return set_error(INFERNO_ECUDA, "attention_step: %s", cudaGetErrorString(ef != cudaSuccess ? ef : es));
  return 0;
}
