// On-device token sampling: the sampler of the CPU decode path
// (generate_cpu / softmax_sample, Inferno.jl src/ModelCPU.jl:1123-1225),
// restated for one CTA of 1024 threads over the vocabulary:
//   1. presence penalty (l -= p) then repetition penalty (l > 0 ? l / r : l * r)
//      for tokens already seen (:1202-1225), then l / temperature;
//   2. top-k (top_k > 0): the k largest logits, ties to the lower index (stable
//      sortperm(rev=true)); softmax over the kept logits (all of them when
//      top_k == 0);
//   3. top-p: cumulative probability in descending order until >= top_p, the
//      rest zeroed, renormalised;
//   4. min-p: probabilities below max_prob * min_p zeroed, renormalised;
//   5. one uniform draw u: the first index (natural order) whose cumulative
//      probability reaches u.
// Candidates: an exact radix select finds the K-th largest scaled logit
// (K = top_k, or 1024 when top_k == 0: the nucleus is then searched within
// the 1024 most probable tokens, as src/Engine.jl:74-78 does); the softmax
// normaliser covers every token when top_k == 0.  Everything after the select
// runs on <= 1024 candidates in shared memory.
#include <cstdint>
#include "internal.h"
#include "common.cuh"
#include "../../include/inferno_b200.h"

namespace inf {

constexpr int SMP_THREADS = 1024;
constexpr int SMP_MAXK = 1024;

__device__ __forceinline__ float smp_scaled(const float* logits, const uint8_t* seen, const SampleArgs& a, int i) {
  float l = logits[i];
  if (seen && seen[i]) {
    l -= a.presence;                                   // apply_presence_penalty!
    if (a.repetition != 1.0f) l = l > 0.f ? l / a.repetition : l * a.repetition;   // apply_repetition_penalty!
  }
  return (a.temperature != 1.0f && a.temperature != 0.0f) ? l / a.temperature : l;   // 0: greedy
}
__device__ __forceinline__ uint32_t smp_key(float f) { return float_ordered(f); }

// Philox-4x32-10 (Salmon et al., SC'11): one 32-bit output from (key, counter)
__device__ __forceinline__ uint32_t philox(unsigned long long key, unsigned long long ctr) {
  uint32_t c0 = (uint32_t)ctr, c1 = (uint32_t)(ctr >> 32), c2 = 0, c3 = 0;
  uint32_t k0 = (uint32_t)key, k1 = (uint32_t)(key >> 32);
#pragma unroll
  for (int r = 0; r < 10; ++r) {
    const uint32_t h0 = __umulhi(0xD2511F53u, c0), l0 = 0xD2511F53u * c0;
    const uint32_t h1 = __umulhi(0xCD9E8D57u, c2), l1 = 0xCD9E8D57u * c2;
    c0 = h1 ^ c1 ^ k0;
    c1 = l1;
    c2 = h0 ^ c3 ^ k1;
    c3 = l0;
    k0 += 0x9E3779B9u;
    k1 += 0xBB67AE85u;
  }
  return c0;
}

template <class T>
__device__ __forceinline__ T block_reduce_sum(T v, T* red) {
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  __syncthreads();
  if (lane == 0) red[w] = v;
  __syncthreads();
  T s = 0;
  for (int i = 0; i < SMP_THREADS / 32; ++i) s += red[i];
  return s;
}

// u >= 0: the draw; u < 0: Philox(seed, *step) (the engine's token counter)
__global__ void __launch_bounds__(SMP_THREADS) sample_kernel(const float* __restrict__ logits, int V, SampleArgs a,
                                                             const uint8_t* seen, float u, const int* step,
                                                             int* out_tok, unsigned long long* out_key,
                                                             uint8_t* mark_seen) {
  __shared__ unsigned hist[256];
  __shared__ float redf[32];
  __shared__ unsigned redu[32];
  __shared__ float cs[SMP_MAXK];
  __shared__ int ci[SMP_MAXK];
  __shared__ unsigned sh_prefix, sh_remaining, sh_count;
  __shared__ int sh_pick;
  const int tid = threadIdx.x;
  pdl_wait();
  pdl_trigger();
  const bool greedy = a.temperature == 0.0f;
  const int K = greedy ? 1 : (a.top_k > 0 ? min(a.top_k, min(V, SMP_MAXK)) : min(V, SMP_MAXK));

  // ---- max of the scaled logits ----
  float mx = -INFINITY;
  for (int i = tid; i < V; i += SMP_THREADS) mx = fmaxf(mx, smp_scaled(logits, seen, a, i));
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  if ((tid & 31) == 0) redf[tid >> 5] = mx;
  __syncthreads();
  mx = -INFINITY;
  for (int i = 0; i < SMP_THREADS / 32; ++i) mx = fmaxf(mx, redf[i]);

  // ---- radix select of the K-th largest key (8-bit digits, high first) ----
  if (tid == 0) { sh_prefix = 0; sh_remaining = (unsigned)K; }
  for (int pass = 0; pass < 4; ++pass) {
    const int shift = 24 - 8 * pass;
    const uint32_t hmask = pass == 0 ? 0u : (0xffffffffu << (shift + 8));
    for (int i = tid; i < 256; i += SMP_THREADS) hist[i] = 0;
    __syncthreads();
    const uint32_t prefix = sh_prefix;
    for (int i = tid; i < V; i += SMP_THREADS) {
      const uint32_t k = smp_key(smp_scaled(logits, seen, a, i));
      if ((k & hmask) == (prefix & hmask)) atomicAdd(&hist[(k >> shift) & 255u], 1u);
    }
    __syncthreads();
    if (tid == 0) {
      unsigned rem = sh_remaining, acc = 0;
      int d = 255;
      for (; d > 0; --d) {
        if (acc + hist[d] >= rem) break;
        acc += hist[d];
      }
      sh_prefix = prefix | ((uint32_t)d << shift);
      sh_remaining = rem - acc;      // how many with this exact prefix we still need
    }
    __syncthreads();
  }
  const uint32_t thr = sh_prefix;    // key of the K-th largest value
  const unsigned need_eq = sh_remaining;
  // ---- gather: keys above thr, plus the first need_eq keys equal to thr in
  // index order (contiguous chunk per thread + scan), and the normaliser ----
  const int chunk = (V + SMP_THREADS - 1) / SMP_THREADS;
  const int i0 = tid * chunk, i1 = min(V, i0 + chunk);
  unsigned my_eq = 0;
  float my_sum = 0.f;
  for (int i = i0; i < i1; ++i) {
    const float s = smp_scaled(logits, seen, a, i);
    if (smp_key(s) == thr) ++my_eq;
    if (a.top_k <= 0) my_sum += expf(s - mx);
  }
  // exclusive scan of my_eq over threads (index order)
  unsigned incl = my_eq;
  for (int o = 1; o < 32; o <<= 1) {
    const unsigned t = __shfl_up_sync(0xffffffffu, incl, o);
    if ((tid & 31) >= o) incl += t;
  }
  if ((tid & 31) == 31) redu[tid >> 5] = incl;
  if (tid == 0) sh_count = 0;
  __syncthreads();
  unsigned wbase = 0;
  for (int i = 0; i < (tid >> 5); ++i) wbase += redu[i];
  unsigned eq_before = wbase + incl - my_eq;
  const float zsum_all = a.top_k <= 0 ? block_reduce_sum(my_sum, redf) : 0.f;
  for (int i = i0; i < i1; ++i) {
    const float s = smp_scaled(logits, seen, a, i);
    const uint32_t k = smp_key(s);
    bool keep = k > thr;
    if (k == thr) {
      keep = eq_before < need_eq;
      ++eq_before;
    }
    if (keep) {
      const unsigned slot = atomicAdd(&sh_count, 1u);
      if (slot < SMP_MAXK) { cs[slot] = s; ci[slot] = i; }
    }
  }
  __syncthreads();
  const int n = min((int)sh_count, SMP_MAXK);
  for (int j = n + tid; j < SMP_MAXK; j += SMP_THREADS) { cs[j] = -INFINITY; ci[j] = 0x7fffffff; }
  __syncthreads();
  // ---- bitonic sort: value descending, index ascending ----
  for (int size = 2; size <= SMP_MAXK; size <<= 1)
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      const int j = tid, p = j ^ stride;
      if (p > j) {
        const bool desc = (j & size) == 0;
        const bool before = cs[j] > cs[p] || (cs[j] == cs[p] && ci[j] < ci[p]);   // j ahead of p
        if (desc != before) {
          const float tv = cs[j]; cs[j] = cs[p]; cs[p] = tv;
          const int ti = ci[j]; ci[j] = ci[p]; ci[p] = ti;
        }
      }
      __syncthreads();
    }
  if (greedy) {
    if (tid == 0) sh_pick = ci[0];
  } else {
    // probabilities (rank order) in cs[]
    const float e = tid < n ? expf(cs[tid] - mx) : 0.f;
    const float z = a.top_k > 0 ? block_reduce_sum(e, redf) : zsum_all;
    __syncthreads();
    cs[tid] = e / z;
    __syncthreads();
    if (tid == 0) {
      int keep = n;
      if (a.top_p < 1.0f) {                          // nucleus (sorted order)
        float c = 0.f;
        for (int j = 0; j < n; ++j) {
          c += cs[j];
          if (c >= a.top_p) { keep = j + 1; break; }
        }
      }
      float tot = 0.f;
      for (int j = 0; j < keep; ++j) tot += cs[j];
      for (int j = keep; j < SMP_MAXK; ++j) cs[j] = 0.f;
      if (a.top_p < 1.0f && tot > 0.f)
        for (int j = 0; j < keep; ++j) cs[j] /= tot;
      if (a.min_p > 0.0f) {                          // relative to the largest probability
        const float th = cs[0] * a.min_p;
        float t2 = 0.f;
        for (int j = 0; j < keep; ++j) {
          if (cs[j] < th) cs[j] = 0.f;
          t2 += cs[j];
        }
        if (t2 > 0.f)
          for (int j = 0; j < keep; ++j) cs[j] /= t2;
      }
    }
    __syncthreads();
    // draw over the candidates in index order: sort by index ascending
    for (int size = 2; size <= SMP_MAXK; size <<= 1)
      for (int stride = size >> 1; stride > 0; stride >>= 1) {
        const int j = tid, p = j ^ stride;
        if (p > j) {
          const bool asc = (j & size) == 0;
          if ((ci[j] > ci[p]) == asc) {
            const float tv = cs[j]; cs[j] = cs[p]; cs[p] = tv;
            const int ti = ci[j]; ci[j] = ci[p]; ci[p] = ti;
          }
        }
        __syncthreads();
      }
    if (tid == 0) {
      float r = u;
      if (r < 0.f) r = (float)(philox(a.seed, step ? (unsigned long long)*step : 0ull) >> 8) * (1.0f / 16777216.0f);
      float c = 0.f;
      int pick = V - 1;                               // reference: length(probs) when nothing reaches r
      for (int j = 0; j < n; ++j) {
        c += cs[j];
        if (cs[j] > 0.f && r <= c) { pick = ci[j]; break; }
      }
      sh_pick = pick;
    }
  }
  __syncthreads();
  if (tid == 0) {
    const int pick = sh_pick;
    if (out_tok) *out_tok = pick;
    if (out_key) *out_key = (unsigned long long)(0xffffffffu - (uint32_t)pick);   // as a packed argmax key
    if (mark_seen) mark_seen[pick] = 1;
  }
}

int launch_sample(const float* logits, int V, const SampleArgs& a, const uint8_t* seen, float u, const int* step,
                  int* out_tok, unsigned long long* out_key, uint8_t* mark_seen, cudaStream_t st, bool pdl) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(1);
  cfg.blockDim = dim3(SMP_THREADS);
  cfg.stream = st;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = pdl ? 1 : 0;
  cudaError_t e = cudaLaunchKernelEx(&cfg, sample_kernel, logits, V, a, seen, u, step, out_tok, out_key, mark_seen);
  return e == cudaSuccess ? 0 : set_error(INFERNO_ECUDA, "sample launch: %s", cudaGetErrorString(e));
}

}  // namespace inf

using namespace inf;

extern "C" int inferno_sample_logits(const float* logits, int vocab, const InfernoSampling* s, const uint8_t* seen,
                                     float u, int32_t* out_token, void* stream) {
  if (!logits || vocab <= 0 || !s || !out_token) return set_error(INFERNO_EINVAL, "sample_logits: bad arguments");
  if (s->temperature < 0.f || s->top_p <= 0.f || s->top_p > 1.f || s->min_p < 0.f || s->min_p >= 1.f ||
      s->repetition_penalty <= 0.f)
    return set_error(INFERNO_EINVAL, "sample_logits: parameter out of range");
  SampleArgs a{s->temperature, s->top_p, s->min_p, s->presence_penalty, s->repetition_penalty, s->top_k, s->seed};
  return launch_sample(logits, vocab, a, seen, u, nullptr, out_token, nullptr, nullptr, (cudaStream_t)stream, false);
}
