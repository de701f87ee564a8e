// Chunked prefill: the non-GEMV steps of up to PF_MAX_T prompt tokens per
// launch (the GEMVs of a chunk are the batched GEMV path, one weight read per
// chunk).  Replaces the token-by-token prompt loop of forward_cpu!
// (Inferno.jl src/ModelCPU.jl:945-989) with the same per-token arithmetic.
//
//  * gdn_chunk_kernel: GatedDeltaNetCPU's conv1d + gates + delta rule
//    (src/ModelCPU.jl:531-700) for T consecutive tokens.  A CTA owns 16 rows
//    of one head's state in registers across the T tokens; the conv inputs of
//    token t are the in_proj outputs of tokens t-K+1..t, taken from the chunk
//    buffer or, before the chunk, from the conv ring -- so no CTA waits for
//    another.  conv_ring_chunk_kernel then stores the chunk's last inputs in
//    the ring and advances the layer's step counter.
//  * attn_append_chunk_kernel: Q/K RMSNorm + partial RoPE of the chunk's keys
//    and their KV-cache rows (rmsnorm_rotary!, update_kv_cache!,
//    src/ModelCPU.jl:187-258); attn_chunk_kernel: every query of the chunk
//    against the cache up to its own position (causal), split-K online softmax
//    over 32-key tiles, merged by the last CTA of each (token, head), times
//    the sigmoid gate (src/FlashAttention.jl:16-74, src/ModelCPU.jl:846-851).
#include <algorithm>
#include "internal.h"
#include "common.cuh"
#include "params.h"
#include "../../include/inferno_b200.h"

namespace inf {

constexpr int PF_DK = 128;
constexpr int PF_ROWS = 16;
constexpr int PF_THREADS = 128;
constexpr int PF_MAXK = 4;
constexpr int PF_HD = 256;

__device__ __forceinline__ void pf_block_sum(float* v, int nv, float (*red)[4]) {
  for (int i = 0; i < nv; ++i) v[i] = warp_sum(v[i]);
  if ((threadIdx.x & 31) == 0)
    for (int i = 0; i < nv; ++i) red[i][threadIdx.x >> 5] = v[i];
  __syncthreads();
  for (int i = 0; i < nv; ++i) v[i] = (red[i][0] + red[i][1]) + (red[i][2] + red[i][3]);
  __syncthreads();
}

// p.x, p.qkv, p.y are [T][H], [T][C], [T][nv*dv]
__global__ void __launch_bounds__(PF_THREADS) gdn_chunk_kernel(const __grid_constant__ GdnParams p, int T) {
  extern __shared__ __align__(16) float pf_sm[];      // w_alpha row, w_beta row, in_norm
  __shared__ __align__(16) float qn[PF_DK], kn[PF_DK];
  __shared__ float vrow[PF_ROWS];
  __shared__ float red[5][4];
  const int h = blockIdx.x, r0 = blockIdx.y * PF_ROWS, tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31;
  const int g = h % p.nk, K = p.K, C = p.C, H = p.H;
  pdl_wait();
  pdl_trigger();
  float* wa_s = pf_sm;
  float* wb_s = pf_sm + H;
  float* wn_s = pf_sm + 2 * H;
  for (int i = tid * 4; i < H; i += PF_THREADS * 4) {
    *(float4*)&wa_s[i] = *(const float4*)&p.w_alpha[(long long)h * H + i];
    *(float4*)&wb_s[i] = *(const float4*)&p.w_beta[(long long)h * H + i];
    *(float4*)&wn_s[i] = *(const float4*)&p.in_norm[i];
  }
  const int t0 = *p.step;
  const int cq = g * PF_DK + tid, ck = p.nk * PF_DK + g * PF_DK + tid;
  const int cv = 2 * p.nk * PF_DK + h * p.dv + r0 + tid;     // valid for tid < PF_ROWS
  float wq[PF_MAXK], wk[PF_MAXK], wv[PF_MAXK], hq[PF_MAXK], hk[PF_MAXK], hv[PF_MAXK];
#pragma unroll
  for (int k = 0; k < PF_MAXK; ++k) {
    wq[k] = wk[k] = wv[k] = hq[k] = hk[k] = hv[k] = 0.f;
    if (k < K) {
      wq[k] = p.conv_w[(long long)cq * K + k];
      wk[k] = p.conv_w[(long long)ck * K + k];
      if (tid < PF_ROWS) wv[k] = p.conv_w[(long long)cv * K + k];
    }
    if (k < K - 1) {             // history: input of time t0-(K-1)+k
      int slot = (t0 - (K - 1) + k) % K;
      if (slot < 0) slot += K;
      hq[k] = p.ring[(long long)slot * C + cq];
      hk[k] = p.ring[(long long)slot * C + ck];
      if (tid < PF_ROWS) hv[k] = p.ring[(long long)slot * C + cv];
    }
  }
  constexpr int RPW = PF_ROWS / (PF_THREADS / 32);
  float4 srow[RPW];
#pragma unroll
  for (int j = 0; j < RPW; ++j)
    srow[j] = *((const float4*)(p.S + ((long long)h * p.dv + r0 + warp + 4 * j) * PF_DK) + lane);
  const float a_h = p.ssm_a[h], dt_h = p.dt_bias[h];
  __syncthreads();
  for (int t = 0; t < T; ++t) {
    const float* x = p.x + (long long)t * H;
    float acc[5] = {0.f, 0.f, 0.f, 0.f, 0.f};
    for (int i = tid; i < H; i += PF_THREADS) {
      const float xv = x[i], xw = xv * wn_s[i];
      acc[0] = fmaf(xv, xv, acc[0]);
      acc[1] = fmaf(wa_s[i], xw, acc[1]);
      acc[2] = fmaf(wb_s[i], xw, acc[2]);
    }
    // conv1d + SiLU: taps k < K-1 from earlier tokens of the chunk or the ring
    float vq = 0.f, vk = 0.f, vvv = 0.f;
#pragma unroll
    for (int k = 0; k < PF_MAXK; ++k) {
      if (k >= K) break;
      const int tau = t - (K - 1) + k;
      float iq, ik, iv = 0.f;
      if (tau >= 0) {
        const float* q = p.qkv + (long long)tau * C;
        iq = q[cq];
        ik = q[ck];
        if (tid < PF_ROWS) iv = q[cv];
      } else {
        iq = hq[K - 1 + tau];
        ik = hk[K - 1 + tau];
        iv = hv[K - 1 + tau];
      }
      vq += iq * wq[k];
      vk += ik * wk[k];
      vvv += iv * wv[k];
    }
    const float qv = vq / (1.0f + expf(-vq));
    const float kv = vk / (1.0f + expf(-vk));
    if (tid < PF_ROWS) vrow[tid] = vvv / (1.0f + expf(-vvv));
    acc[3] = qv * qv;
    acc[4] = kv * kv;
    pf_block_sum(acc, 5, red);
    const float scale = 1.0f / sqrtf(acc[0] / (float)H + p.eps);
    const float alpha = acc[1] * scale, beta_raw = acc[2] * scale;
    // gates in Float64 (src/ModelCPU.jl:618-636)
    double a = (double)alpha + (double)dt_h;
    a = fmin(20.0, fmax(-20.0, a));
    const double sp = log(1.0 + exp(a));
    const float dec = expf((float)((double)a_h * sp));
    const double bv = fmin(20.0, fmax(-20.0, (double)beta_raw));
    const float bg = (float)(1.0 / (1.0 + exp(-bv)));
    const float qnv = 1.0f / (sqrtf(acc[3]) + 1.0e-6f) * (1.0f / sqrtf((float)PF_DK));
    const float knv = 1.0f / (sqrtf(acc[4]) + 1.0e-6f);
    qn[tid] = qv * qnv;
    kn[tid] = kv * knv;
    __syncthreads();
    const float4 k4 = *(const float4*)&kn[lane * 4];
    const float4 q4 = *(const float4*)&qn[lane * 4];
#pragma unroll
    for (int j = 0; j < RPW; ++j) {
      const int rr = warp + 4 * j;
      float4 s = srow[j];
      s.x *= dec; s.y *= dec; s.z *= dec; s.w *= dec;
      const float sk = warp_sum(s.x * k4.x + s.y * k4.y + s.z * k4.z + s.w * k4.w);
      const float d = bg * (vrow[rr] - sk);
      s.x += d * k4.x; s.y += d * k4.y; s.z += d * k4.z; s.w += d * k4.w;
      const float yv = warp_sum(s.x * q4.x + s.y * q4.y + s.z * q4.z + s.w * q4.w);
      srow[j] = s;
      if (lane == 0) p.y[(long long)t * p.nv * p.dv + h * p.dv + r0 + rr] = yv;
    }
    __syncthreads();        // qn / kn / vrow reused by the next token
  }
#pragma unroll
  for (int j = 0; j < RPW; ++j)
    *((float4*)(p.S + ((long long)h * p.dv + r0 + warp + 4 * j) * PF_DK) + lane) = srow[j];
}

// the chunk's last inputs into the conv ring (time t0+tau in slot (t0+tau) % K)
// and the layer's step counter += T
__global__ void conv_ring_chunk_kernel(float* ring, const float* qkv, int* step, int C, int K, int T) {
  pdl_wait();
  pdl_trigger();
  const int t0 = *step;
  const int first = max(0, T - K);
  for (int idx = blockIdx.x * blockDim.x + threadIdx.x; idx < (T - first) * C; idx += gridDim.x * blockDim.x) {
    const int tau = first + idx / C, c = idx % C;
    ring[(long long)((t0 + tau) % K) * C + c] = qkv[(long long)tau * C + c];
  }
  // the counter itself is advanced by step_advance_kernel, launched after
  // this kernel, so every block of this one reads the same t0
}
__global__ void step_advance_kernel(int* step, int T) {
  pdl_wait();
  pdl_trigger();
  *step += T;
}

// ---------------------------------------------------------------------------
// attention
// ---------------------------------------------------------------------------
// p.qg / p.k / p.v hold T tokens (strides nh*2*hd, nkv*hd, nkv*hd); token t is
// at position pos0 + t.  Grid (T, nkv).
__global__ void __launch_bounds__(PF_HD) attn_append_chunk_kernel(const __grid_constant__ AttnParams p, int pos0) {
  __shared__ float kn[PF_HD];
  __shared__ float red[8];
  const int t = blockIdx.x, kvh = blockIdx.y, d = threadIdx.x;
  const int lane = d & 31, warp = d >> 5;
  pdl_wait();
  pdl_trigger();
  const int pos = pos0 + t;
  const float kv = p.k[((long long)t * p.nkv + kvh) * PF_HD + d];
  float b = warp_sum(kv * kv);
  if (lane == 0) red[warp] = b;
  __syncthreads();
  b = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) b += red[i];
  const float ik = 1.0f / sqrtf(b / (float)PF_HD + p.eps);
  kn[d] = kv * ik * p.k_norm[d];
  __syncthreads();
  const int half = p.rd / 2;
  if (d < half) {
    const float c = p.rope_cos[(long long)pos * half + d], sn = p.rope_sin[(long long)pos * half + d];
    const float x1 = kn[d], x2 = kn[d + half];
    kn[d] = x1 * c - x2 * sn;
    kn[d + half] = x1 * sn + x2 * c;
  }
  __syncthreads();
  const long long off = ((long long)pos * p.nkv + kvh) * PF_HD + d;
  p.kc[off] = kn[d];
  p.vc[off] = p.v[((long long)t * p.nkv + kvh) * PF_HD + d];
}

// Grid (nh, nsplit, T); counters [T][nh]; part_o [T][nh][nsplit][hd];
// part_ml [T][nh][nsplit][2]; out [T][nh*hd].
__global__ void __launch_bounds__(PF_HD) attn_chunk_kernel(const __grid_constant__ AttnParams p, int pos0) {
  __shared__ __align__(16) float qs[PF_HD];
  __shared__ float sc[32];
  __shared__ float red[8];
  __shared__ int ticket;
  const int h = blockIdx.x, s = blockIdx.y, t = blockIdx.z, d = threadIdx.x;
  const int kvh = h / (p.nh / p.nkv);
  const int lane = d & 31, warp = d >> 5;
  pdl_wait();
  pdl_trigger();
  const int pos = pos0 + t, L = pos + 1;
  const int nact = (L + p.split_len - 1) / p.split_len;
  if (s >= nact) return;
  const int j0 = s * p.split_len, j1 = min(j0 + p.split_len, L);
  const float* qg = p.qg + (long long)t * p.nh * 2 * PF_HD + (long long)h * 2 * PF_HD;
  const float qv = qg[d];
  float a = warp_sum(qv * qv);
  if (lane == 0) red[warp] = a;
  __syncthreads();
  a = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) a += red[i];
  const float iq = 1.0f / sqrtf(a / (float)PF_HD + p.eps);
  qs[d] = qv * iq * p.q_norm[d];
  __syncthreads();
  const int half = p.rd / 2;
  if (d < half) {
    const float c = p.rope_cos[(long long)pos * half + d], sn = p.rope_sin[(long long)pos * half + d];
    const float x1 = qs[d], x2 = qs[d + half];
    qs[d] = x1 * c - x2 * sn;
    qs[d + half] = x1 * sn + x2 * c;
  }
  __syncthreads();
  const float scale = 1.0f / sqrtf((float)PF_HD);
  const int kk = d >> 3, part = d & 7;
  float4 q8[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) q8[i] = *(const float4*)&qs[part * 32 + 4 * i];
  float m = -INFINITY, l = 0.f, o = 0.f;
  for (int c0 = j0; c0 < j1; c0 += 32) {
    const int cend = min(c0 + 32, j1);
    const int j = c0 + kk;
    float dot = 0.f;
    if (j < cend) {
      const float4* kr = (const float4*)(p.kc + ((long long)j * p.nkv + kvh) * PF_HD + part * 32);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float4 k4 = kr[i];
        dot += q8[i].x * k4.x + q8[i].y * k4.y + q8[i].z * k4.z + q8[i].w * k4.w;
      }
    }
    dot += __shfl_xor_sync(0xffffffffu, dot, 4);
    dot += __shfl_xor_sync(0xffffffffu, dot, 2);
    dot += __shfl_xor_sync(0xffffffffu, dot, 1);
    __syncthreads();
    if (part == 0) sc[kk] = (j < cend) ? dot * scale : -INFINITY;
    __syncthreads();
    float cm = -INFINITY;
#pragma unroll
    for (int q = 0; q < 32; ++q) cm = fmaxf(cm, sc[q]);
    const float mn = fmaxf(m, cm);
    const float corr = expf(m - mn);
    l *= corr;
    o *= corr;
    for (int q = 0; q < 32; ++q) {
      if (c0 + q >= cend) break;
      const float e = expf(sc[q] - mn);
      l += e;
      o = fmaf(e, p.vc[((long long)(c0 + q) * p.nkv + kvh) * PF_HD + d], o);
    }
    m = mn;
  }
  const long long pi = ((long long)t * p.nh + h) * p.nsplit + s;
  p.part_o[pi * PF_HD + d] = o;
  if (d == 0) {
    p.part_ml[pi * 2 + 0] = m;
    p.part_ml[pi * 2 + 1] = l;
  }
  __threadfence();
  __syncthreads();
  int* ctr = p.counters + (long long)t * p.nh + h;
  if (d == 0) ticket = atomicAdd(ctr, 1);
  __syncthreads();
  if (ticket != nact - 1) return;
  __threadfence();
  if (d == 0) *ctr = 0;
  const float* mlp = p.part_ml + ((long long)t * p.nh + h) * p.nsplit * 2;
  float M = -INFINITY;
  for (int u = 0; u < nact; ++u) M = fmaxf(M, __ldcg(mlp + 2 * u));
  float num = 0.f, den = 0.f;
  for (int u = 0; u < nact; ++u) {
    const float w = expf(__ldcg(mlp + 2 * u) - M);
    num = fmaf(w, __ldcg(p.part_o + (((long long)t * p.nh + h) * p.nsplit + u) * PF_HD + d), num);
    den = fmaf(w, __ldcg(mlp + 2 * u + 1), den);
  }
  const float gte = qg[PF_HD + d];
  p.out[(long long)t * p.nh * PF_HD + (long long)h * PF_HD + d] = (num / den) * (1.0f / (1.0f + expf(-gte)));
}

// ---------------------------------------------------------------------------
// GDN prefill, token-parallel part: for token t of the chunk and value head h
// the conv1d + SiLU of its q / k / v channels (inputs of tokens t-K+1..t from
// the chunk or, before it, from the conv ring), the L2-normalised q (times
// 1/sqrt(dk)) and k, and the Float64 gates of GatedDeltaNetCPU
// (src/ModelCPU.jl:555-636): decay g = a_h * softplus(alpha + dt_h) and
// beta = sigmoid(beta_raw), alpha / beta_raw = w . RMSNorm(x_t).  Grid (T, nv),
// 128 threads (one q / k / v channel each).  The recurrence then runs in
// gdn_seq_kernel.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(PF_DK) gdn_prep_kernel(const __grid_constant__ GdnParams p, int T, GdnScratch o) {
  __shared__ float red[5][4];
  const int t = blockIdx.x, h = blockIdx.y, tid = threadIdx.x;
  const int g = h % p.nk, K = p.K, C = p.C, H = p.H;
  pdl_wait();
  pdl_trigger();
  const int t0 = *p.step;
  const float* x = p.x + (long long)t * H;
  float acc[5] = {0.f, 0.f, 0.f, 0.f, 0.f};
  for (int i = tid; i < H; i += PF_DK) {
    const float xv = x[i], xw = xv * p.in_norm[i];
    acc[0] = fmaf(xv, xv, acc[0]);
    acc[1] = fmaf(p.w_alpha[(long long)h * H + i], xw, acc[1]);
    acc[2] = fmaf(p.w_beta[(long long)h * H + i], xw, acc[2]);
  }
  const int cq = g * PF_DK + tid, ck = p.nk * PF_DK + g * PF_DK + tid;
  const int cv = 2 * p.nk * PF_DK + h * p.dv + tid;       // valid for tid < dv
  float vq = 0.f, vk = 0.f, vvv = 0.f;
  for (int k = 0; k < K; ++k) {
    const int tau = t - (K - 1) + k;
    float iq, ik, iv = 0.f;
    if (tau >= 0) {
      const float* q = p.qkv + (long long)tau * C;
      iq = q[cq];
      ik = q[ck];
      if (tid < p.dv) iv = q[cv];
    } else {      // history: input of time t0 + tau, kept in ring slot (t0 + tau) mod K
      int slot = (t0 + tau) % K;
      if (slot < 0) slot += K;
      const float* r = p.ring + (long long)slot * C;
      iq = r[cq];
      ik = r[ck];
      if (tid < p.dv) iv = r[cv];
    }
    vq += iq * p.conv_w[(long long)cq * K + k];
    vk += ik * p.conv_w[(long long)ck * K + k];
    if (tid < p.dv) vvv += iv * p.conv_w[(long long)cv * K + k];
  }
  const float qv = vq / (1.0f + expf(-vq));
  const float kv = vk / (1.0f + expf(-vk));
  acc[3] = qv * qv;
  acc[4] = kv * kv;
  pf_block_sum(acc, 5, red);
  const long long row = (long long)t * p.nv + h;
  o.qn[row * PF_DK + tid] = qv * (1.0f / (sqrtf(acc[3]) + 1.0e-6f) * (1.0f / sqrtf((float)PF_DK)));
  o.kn[row * PF_DK + tid] = kv * (1.0f / (sqrtf(acc[4]) + 1.0e-6f));
  if (tid < p.dv) o.vv[row * p.dv + tid] = vvv / (1.0f + expf(-vvv));
  if (tid == 0) {
    const float scale = 1.0f / sqrtf(acc[0] / (float)H + p.eps);
    const float alpha = acc[1] * scale, beta_raw = acc[2] * scale;
    double a = (double)alpha + (double)p.dt_bias[h];
    a = fmin(20.0, fmax(-20.0, a));
    const double sp = log(1.0 + exp(a));
    o.g[row] = (float)((double)p.ssm_a[h] * sp);
    const double bv = fmin(20.0, fmax(-20.0, (double)beta_raw));
    o.beta[row] = (float)(1.0 / (1.0 + exp(-bv)));
  }
}

namespace {
template <class F, class... A>
int pf_launch(F kern, dim3 grid, dim3 block, size_t smem, cudaStream_t st, A... args) {
  kern<<<grid, block, smem, st>>>(args...);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? 0 : set_error(INFERNO_ECUDA, "prefill launch: %s", cudaGetErrorString(e));
}
}  // namespace

int launch_gdn_chunk(const GdnParams& p, int T, cudaStream_t st) {
  if (T < 1 || T > PF_MAX_T || p.dv % PF_ROWS || p.K < 1 || p.K > PF_MAXK || p.H % 4)
    return set_error(INFERNO_EINVAL, "gdn chunk: unsupported dims");
  static DeviceOnce once;
  cudaError_t ea = once.run(
      [] { return cudaFuncSetAttribute(gdn_chunk_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 3 * 8192 * 4); });
  if (ea != cudaSuccess) return set_error(INFERNO_ECUDA, "GDN chunk attribute: %s", cudaGetErrorString(ea));
  int rc;
  if ((rc = pf_launch(gdn_chunk_kernel, dim3(p.nv, p.dv / PF_ROWS), dim3(PF_THREADS), (size_t)3 * p.H * 4, st, p, T)))
    return rc;
  if ((rc = pf_launch(conv_ring_chunk_kernel, dim3(std::max(1, (T * p.C + 255) / 256)), dim3(256), 0, st, p.ring,
                      p.qkv, p.step, p.C, p.K, T)))
    return rc;
  return pf_launch(step_advance_kernel, dim3(1), dim3(1), 0, st, p.step, T);
}

int launch_gdn_prefill(const GdnParams& p, int T, const GdnScratch& o, cudaStream_t st) {
  if (T < 1 || p.dv % PF_ROWS || p.dv > PF_DK || p.K < 1 || p.K > PF_MAXK || p.H % 4)
    return set_error(INFERNO_EINVAL, "gdn prefill: unsupported dims");
  int rc;
  if ((rc = pf_launch(gdn_prep_kernel, dim3(T, p.nv), dim3(PF_DK), 0, st, p, T, o))) return rc;
  if ((rc = pf_launch(conv_ring_chunk_kernel, dim3(std::max(1, (std::min(T, p.K) * p.C + 255) / 256)), dim3(256), 0,
                      st, p.ring, p.qkv, p.step, p.C, p.K, T)))
    return rc;
  if ((rc = pf_launch(step_advance_kernel, dim3(1), dim3(1), 0, st, p.step, T))) return rc;
  return launch_gdn_seq(T, p.nv, p.dv, o.qn, o.kn, o.vv, o.beta, o.g, p.S, p.y, st);
}

int launch_attn_chunk(const AttnParams& p, int pos0, int T, cudaStream_t st) {
  if (T < 1 || T > PF_MAX_T) return set_error(INFERNO_EINVAL, "attention chunk: bad T");
  int rc;
  if ((rc = pf_launch(attn_append_chunk_kernel, dim3(T, p.nkv), dim3(PF_HD), 0, st, p, pos0))) return rc;
  return pf_launch(attn_chunk_kernel, dim3(p.nh, p.nsplit, T), dim3(PF_HD), 0, st, p, pos0);
}

}  // namespace inf
