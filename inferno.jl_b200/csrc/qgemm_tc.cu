// Quantized GEMM on the 5th-generation tensor cores (tcgen05), for the
// batched / prefill products Y[t][r] = sum_k W[r][k] * X[t][k] with T >= 16
// token columns: the prompt loop of forward_cpu! (Inferno.jl
// src/ModelCPU.jl:970-986, every mul! of src/ModelCPU.jl:435-444 run for many
// tokens at once) and the config-2 batched GEMM.
//
// Per CTA: a 128-row tile of W (one matrix segment; for the SwiGLU pair 64
// gate + 64 up rows) against a BN-token tile of X, K walked in steps of 64.
//   warp 0      raw producer: the GGUF super-blocks of the 128 rows by
//               16-byte cp.async (aligned supersets for rows that do not
//               start on 16 bytes), lane = row, completion on an mbarrier;
//   warp 1      allocates the TMEM accumulator (BN fp32 columns x 128 lanes)
//               and issues tcgen05.mma from one thread;
//   warp 2      activation producer: fp16 tiles by 2-D TMA
//               (cp.async.bulk.tensor, SWIZZLE_128B, zero fill past T);
//   warps 3-18  dequantize: four threads per weight row, 16 weights each per
//               K step with the fp32 arithmetic of Dequant.jl, written as
//               fp16 into the canonical K-major SWIZZLE_128B operand tile;
//               warps 3-6 then drain the accumulator with tcgen05.ld and
//               apply the epilogue.
// Rings: raw super-blocks (NR), dequantized A tiles (NA), activation tiles
// (NB); every hand-off is an mbarrier, MMA completion is signalled with
// tcgen05.commit.  All waits are bounded and report DERR_MBAR_TIMEOUT.
// Split K (grid.z slices of the super-blocks) fills the SMs when the output
// has few tiles: each slice parks its fp32 tile in a workspace and the last
// slice to arrive (atomic ticket) sums them in slice order and applies the
// epilogue, so results do not depend on arrival order.
//
// Precision: with `split` the fp32 weight w and activation x are carried as
// fp16 pairs (hi = fp16(w), lo = fp16(w - hi)) and the product is
// hi*hi + hi*lo + lo*hi (three MMAs, about 22 significant bits: the fp32
// GEMV's results to ~1e-6 relative); without it one fp16 MMA (11 bits).
// Weights are scaled by a power of two per matrix and activations per token
// (both undone in the epilogue) so that hi and lo stay normal fp16 numbers.
#include <algorithm>
#include <climits>
#include <cstring>
#include <mutex>
#include "internal.h"
#include "common.cuh"
#include "gemv.cuh"
#include "tc.cuh"
#include "../../include/inferno_b200.h"

namespace inf {

constexpr int QG_M = 128;             // weight rows per tile (TMEM lanes)
constexpr int QG_BK = 64;             // K per step (one 128-byte fp16 row)
constexpr int QG_DQ_WARPS = 16;       // dequantizing warps: four threads per weight row
constexpr int QG_THREADS = 64 + 32 * QG_DQ_WARPS;
constexpr int QG_WS_CTAS = 160;       // split-K is used while tiles x slices <= this (workspace bound)
constexpr int QG_ATILE = QG_M * 128;  // bytes of one fp16 A tile (16 KB)

struct QgSeg {
  const uint8_t* W;
  float* y;
  int rows;
  int mtile0;       // first M tile of this segment
};

struct QgParams {
  QgSeg seg[4];
  int nseg, n_mtiles;
  int K, nsb;
  long long row_bytes;
  int slot;              // bytes per row of one raw stage
  int T;
  long long y_stride;    // floats between token rows of y
  int epi;               // QG_STORE / QG_ADD / QG_SWIGLU
  int nbs, nas, nrs;     // ring stages: activation tiles, dequantized A tiles, raw super-blocks
  int kps;               // K steps per dequantized A stage (1 or 2): one hand-off per stage
  int split;
  int trace;             // debug (-DINFERNO_KTRACE=1 builds): %globaltimer stamps into qg_trace
  int dbgmode;           // debug timing only (-DINFERNO_KTRACE=1 builds; wrong results), bits: 1 no MMAs, 2 no dequantization,
                         // 4 no proxy fence, 8 no weight staging after the first stages,
                         // 16 no activation loads, 32 one MMA per K slice instead of three, 64 polling waits,
                         // 128 plain arrivals instead of MMA commits
  float* ws;             // split K: [tile][slice][BN][128] fp32 partial tiles
  int* tickets;          // split K: arrivals per output tile (zero between launches)
  const float* xexp;     // [T] power-of-two exponent applied to each token's fp16 activations
  const float* wbound;   // bound of |w| over the matrix (weight scale)
  int* err;
};
enum { QG_STORE = 0, QG_ADD = 1, QG_SWIGLU = 2 };

struct alignas(64) QgMaps {
  CUtensorMap hi, lo;
};

template <int TYPE>
struct QgBlk;
template <>
struct QgBlk<T_Q4_K> { static constexpr int BB = 144; };
template <>
struct QgBlk<T_Q5_K> { static constexpr int BB = 176; };
template <>
struct QgBlk<T_Q6_K> { static constexpr int BB = 210; };
template <>
struct QgBlk<T_Q8_0> { static constexpr int BB = 272; };   // 8 blocks of 34 bytes per 256 inputs

__device__ __forceinline__ uint32_t ld_u32(const uint8_t* p) { return lds_u32_any(p); }

// 6-bit scale / min j of a K-quant super-block (src/Dequant.jl:345-362)
__device__ __forceinline__ void qg_kscale(const uint8_t* sc, int j, float& s, float& m) {
  const uint32_t w0 = ld_u32(sc), w1 = ld_u32(sc + 4), w2 = ld_u32(sc + 8);
  uint32_t sj, mj;
  if (j < 4) {
    sj = (w0 >> (8 * j)) & 63;
    mj = (w1 >> (8 * j)) & 63;
  } else {
    const int q = j - 4;
    const uint32_t hi = (w2 >> (8 * q)) & 0xff;        // sc[j + 4]
    sj = (hi & 0x0f) | (((w0 >> (8 * q + 6)) & 3) << 4);
    mj = (hi >> 4) | (((w1 >> (8 * q + 6)) & 3) << 4);
  }
  s = (float)sj;
  m = (float)mj;
}

// 64 fp32 weights of K step ks (0..3) of one super-block, with the
// oracle's / Dequant.jl's rounding order.
template <int TYPE>
__device__ __forceinline__ void qg_dequant(const uint8_t* rp, int ks, float (&w)[64]) {
  if constexpr (TYPE == T_Q4_K || TYPE == T_Q5_K) {
    const float d = h2f_bits((uint16_t)(ld_u32(rp) & 0xffff)), dmin = h2f_bits((uint16_t)(ld_u32(rp) >> 16));
    float s1, m1, s2, m2;
    qg_kscale(rp + 4, 2 * ks, s1, m1);
    qg_kscale(rp + 4, 2 * ks + 1, s2, m2);
    const float d1 = d * s1, mn1 = dmin * m1, d2 = d * s2, mn2 = dmin * m2;
    const uint8_t* qs = rp + (TYPE == T_Q4_K ? 16 : 48) + 32 * ks;
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      const uint32_t v = ld_u32(qs + 4 * q);
      uint32_t h = 0;
      if constexpr (TYPE == T_Q5_K) h = ld_u32(rp + 16 + 4 * q);
#pragma unroll
      for (int b = 0; b < 4; ++b) {
        uint32_t lo = (v >> (8 * b)) & 15, hi = (v >> (8 * b + 4)) & 15;
        if constexpr (TYPE == T_Q5_K) {
          const uint32_t hb = (h >> (8 * b)) & 0xff;
          lo += ((hb >> (2 * ks)) & 1) << 4;
          hi += ((hb >> (2 * ks + 1)) & 1) << 4;
        }
        w[4 * q + b] = d1 * (float)lo - mn1;
        w[32 + 4 * q + b] = d2 * (float)hi - mn2;
      }
    }
  } else if constexpr (TYPE == T_Q6_K) {
    const int ns = ks >> 1, hi = ks & 1;
    const uint8_t* L = rp + 64 * ns;
    const uint8_t* Hh = rp + 128 + 32 * ns;
    const int8_t* S = (const int8_t*)(rp + 192 + 8 * ns);
    const float d = h2f_bits((uint16_t)(rp[208] | (rp[209] << 8)));
    const float sa0 = d * (float)S[4 * hi + 0], sa1 = d * (float)S[4 * hi + 1];
    const float sb0 = d * (float)S[4 * hi + 2], sb1 = d * (float)S[4 * hi + 3];
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      const uint32_t la = ld_u32(L + 4 * q), lb = ld_u32(L + 32 + 4 * q), hh = ld_u32(Hh + 4 * q);
#pragma unroll
      for (int b = 0; b < 4; ++b) {
        const int l = 4 * q + b;
        const uint32_t hv = (hh >> (8 * b)) & 0xff;
        const uint32_t a = (la >> (8 * b)) & 0xff, bb = (lb >> (8 * b)) & 0xff;
        int q1, q2;
        if (hi == 0) {
          q1 = (int)((a & 15) | ((hv & 3) << 4)) - 32;
          q2 = (int)((bb & 15) | (((hv >> 2) & 3) << 4)) - 32;
        } else {
          q1 = (int)((a >> 4) | (((hv >> 4) & 3) << 4)) - 32;
          q2 = (int)((bb >> 4) | (((hv >> 6) & 3) << 4)) - 32;
        }
        w[l] = (l < 16 ? sa0 : sa1) * (float)q1;
        w[32 + l] = (l < 16 ? sb0 : sb1) * (float)q2;
      }
    }
  } else {   // Q8_0: blocks 2ks, 2ks+1 of the eight 34-byte blocks
#pragma unroll
    for (int hb = 0; hb < 2; ++hb) {
      const uint8_t* b = rp + 34 * (2 * ks + hb);
      const float d = h2f_bits((uint16_t)(b[0] | (b[1] << 8)));
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        const uint32_t v = ld_u32(b + 2 + 4 * q);
#pragma unroll
        for (int e = 0; e < 4; ++e) w[32 * hb + 4 * q + e] = d * (float)(int8_t)((v >> (8 * e)) & 0xff);
      }
    }
  }
}

// 16 fp32 weights of K step ks (0..3) of one super-block, segment seg (0..3)
// of the step's 64: values 16*seg..16*seg+15, Dequant.jl's rounding order.
template <int TYPE>
__device__ __forceinline__ void qg_dequant16(const uint8_t* rp, int ks, int seg, float (&w)[16]) {
  const int off = 16 * (seg & 1), half = seg >> 1;
  if constexpr (TYPE == T_Q4_K || TYPE == T_Q5_K) {
    const uint32_t dd = ld_u32(rp);
    const float d = h2f_bits((uint16_t)(dd & 0xffff)), dmin = h2f_bits((uint16_t)(dd >> 16));
    float sc, mn;
    qg_kscale(rp + 4, 2 * ks + half, sc, mn);
    const float d1 = d * sc, m1 = dmin * mn;
    const uint8_t* qs = rp + (TYPE == T_Q4_K ? 16 : 48) + 32 * ks + off;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const uint32_t v = ld_u32(qs + 4 * q);
      uint32_t h = 0;
      if constexpr (TYPE == T_Q5_K) h = ld_u32(rp + 16 + off + 4 * q);
#pragma unroll
      for (int b = 0; b < 4; ++b) {
        uint32_t c = (v >> (8 * b + 4 * half)) & 15;
        if constexpr (TYPE == T_Q5_K) c += ((h >> (8 * b + 2 * ks + half)) & 1) << 4;
        w[4 * q + b] = d1 * (float)c - m1;
      }
    }
  } else if constexpr (TYPE == T_Q6_K) {
    const int ns = ks >> 1, hi = ks & 1;
    const uint8_t* L = rp + 64 * ns + 32 * half + off;
    const uint8_t* Hh = rp + 128 + 32 * ns + off;
    const int8_t sci = (int8_t)rp[192 + 8 * ns + 4 * hi + 2 * half + (seg & 1)];
    const float d = h2f_bits((uint16_t)(rp[208] | (rp[209] << 8)));
    const float sd = d * (float)sci;
    const int qsh = 4 * hi, hsh = 2 * half + 4 * hi;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const uint32_t la = ld_u32(L + 4 * q), hh = ld_u32(Hh + 4 * q);
#pragma unroll
      for (int b = 0; b < 4; ++b) {
        const uint32_t a = (la >> (8 * b)) & 0xff, hv = (hh >> (8 * b)) & 0xff;
        const int qv = (int)(((a >> qsh) & 15) | (((hv >> hsh) & 3) << 4)) - 32;
        w[4 * q + b] = sd * (float)qv;
      }
    }
  } else {   // Q8_0: block 2ks + half of the eight 34-byte blocks
    const uint8_t* b = rp + 34 * (2 * ks + half);
    const float d = h2f_bits((uint16_t)(b[0] | (b[1] << 8)));
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const uint32_t v = ld_u32(b + 2 + off + 4 * q);
#pragma unroll
      for (int e = 0; e < 4; ++e) w[4 * q + e] = d * (float)(int8_t)((v >> (8 * e)) & 0xff);
    }
  }
}

// fp32 weight pair -> fp16 hi pair and fp16 lo pair (lo = w - hi, rounded)
__device__ __forceinline__ void qg_split2(f2_t w2, uint32_t& h, uint32_t& l) {
  const float2 w = upk2(w2);
  const __half2 hh = __floats2half2_rn(w.x, w.y);
  const float2 hf = __half22float2(hh);
  const float2 d = upk2(fsub2(w2, pk2f(hf.x, hf.y)));
  const __half2 ll = __floats2half2_rn(d.x, d.y);
  h = *(const uint32_t*)&hh;
  l = *(const uint32_t*)&ll;
}

// explicit shared-memory accesses (32-bit shared-window addresses)
__device__ __forceinline__ uint4 lds128(uint32_t a) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(a));
  return v;
}
__device__ __forceinline__ uint32_t lds32(uint32_t a) {
  uint32_t v;
  asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(a));
  return v;
}
__device__ __forceinline__ void sts128(uint32_t a, uint32_t x, uint32_t y, uint32_t z, uint32_t w) {
  asm volatile("st.shared.v4.u32 [%0], {%1, %2, %3, %4};" ::"r"(a), "r"(x), "r"(y), "r"(z), "r"(w) : "memory");
}

// the 16 bytes at a 2-byte aligned shared address, as 4 words
__device__ __forceinline__ void lds_16_any(uint32_t a, uint32_t (&o)[4]) {
  const uint32_t q = a & ~3u, sh = (a & 3u) * 8u;
  uint32_t w[5];
#pragma unroll
  for (int i = 0; i < 5; ++i) w[i] = lds32(q + 4 * i);
#pragma unroll
  for (int i = 0; i < 4; ++i) o[i] = __funnelshift_r(w[i], w[i + 1], sh);
}

// 16 weights of K step ks, segment seg, times the matrix's power-of-two
// scale, as fp16 hi / lo pairs (h[e], l[e] hold weights 2e, 2e+1).  Same
// fp32 values as qg_dequant16 (Dequant.jl's rounding order; the products
// are exact, scaling by a power of two commutes with the rounding); the
// codes become floats through the 2^23 magic-number trick and the
// arithmetic runs on fp32 pairs.
template <int TYPE>
__device__ __forceinline__ void qg_dq16_split(const uint8_t* rp, uint32_t ra, int ks, int seg, float wscale,
                                              uint32_t (&h)[8], uint32_t (&l)[8]) {
  const int off = 16 * (seg & 1), half = seg >> 1;
  if constexpr (TYPE == T_Q4_K) {
    // rows of Q4_K super-blocks (144 bytes) start on 16 bytes
    const uint4 hd = lds128(ra);
    const float d = h2f_bits((uint16_t)(hd.x & 0xffff)), dmin = h2f_bits((uint16_t)(hd.x >> 16));
    const int j = 2 * ks + half;
    uint32_t sj, mj;
    if (j < 4) {
      sj = (hd.y >> (8 * j)) & 63;
      mj = (hd.z >> (8 * j)) & 63;
    } else {
      const int q = j - 4;
      const uint32_t hi = (hd.w >> (8 * q)) & 0xff;
      sj = (hi & 0x0f) | (((hd.y >> (8 * q + 6)) & 3) << 4);
      mj = (hi >> 4) | (((hd.z >> (8 * q + 6)) & 3) << 4);
    }
    const float D = d * (float)sj * wscale, M = dmin * (float)mj * wscale;
    const f2_t D2 = pk2f(D, D), nM2 = pk2f(-M, -M), mg = pk2f(MAGIC, MAGIC);
    const uint4 q4 = lds128(ra + 16 + 32 * ks + off);
    const uint32_t qw[4] = {q4.x, q4.y, q4.z, q4.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint32_t nib = (qw[i] >> (4 * half)) & 0x0f0f0f0fu;
      qg_split2(ffma2(D2, bytes2<0>(nib, mg), nM2), h[2 * i], l[2 * i]);
      qg_split2(ffma2(D2, bytes2<2>(nib, mg), nM2), h[2 * i + 1], l[2 * i + 1]);
    }
  } else if constexpr (TYPE == T_Q6_K) {
    const int ns = ks >> 1, hi = ks & 1;
    const uint32_t sa = ra + 192 + 8 * ns + 4 * hi + 2 * half + (seg & 1);
    const int8_t sci = (int8_t)((lds32(sa & ~3u) >> (8 * (sa & 3u))) & 0xff);
    const uint32_t da = ra + 208;      // 2-byte aligned
    const float d = h2f_bits((uint16_t)((lds32(da & ~3u) >> (8 * (da & 3u))) & 0xffff));
    const float sd = d * (float)sci * wscale;
    const f2_t S2 = pk2f(sd, sd), mg = pk2f(MAGIC + 32.0f, MAGIC + 32.0f);
    uint32_t la[4], hh[4];
    lds_16_any(ra + 64 * ns + 32 * half + off, la);
    lds_16_any(ra + 128 + 32 * ns + off, hh);
    const int qsh = 4 * hi, hsh = 2 * half + 4 * hi;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint32_t q6 = ((la[i] >> qsh) & 0x0f0f0f0fu) | (((hh[i] >> hsh) & 0x03030303u) << 4);
      const f2_t lo2 = bytes2<0>(q6, mg), hi2 = bytes2<2>(q6, mg);   // q - 32, exact
      const float2 a = upk2(lo2), b = upk2(hi2);
      qg_split2(pk2f(a.x * sd, a.y * sd), h[2 * i], l[2 * i]);
      qg_split2(pk2f(b.x * sd, b.y * sd), h[2 * i + 1], l[2 * i + 1]);
      (void)S2;
    }
  } else {
    float w[16];
    qg_dequant16<TYPE>(rp, ks, seg, w);
#pragma unroll
    for (int e = 0; e < 8; ++e) qg_split2(pk2f(w[2 * e] * wscale, w[2 * e + 1] * wscale), h[e], l[e]);
  }
}

__device__ __forceinline__ int qg_exp_for(float bound) {
  // power of two that brings `bound` just under 2^14 (fp16 max is 65504)
  if (!(bound > 0.f) || !(bound <= 3.0e38f)) return 0;
  int e = 0;
  frexpf(bound, &e);             // bound < 2^e
  return max(-120, min(120, 14 - e));
}

__device__ __forceinline__ uint32_t pack_h2(float a, float b) {
  const __half2 h = __floats2half2_rn(a, b);
  return *(const uint32_t*)&h;
}

// bounded wait that polls with mbarrier.test_wait (no suspend hint)
__device__ __forceinline__ bool qg_wait(uint64_t* bar, uint32_t parity, int* err, bool spin) {
  if (!spin) return mbar_wait(bar, parity, err);
  for (uint32_t i = 0; i < (1u << 28); ++i) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    if (ok) return true;
  }
  if (err) atomicExch(err, DERR_MBAR_TIMEOUT);
  return false;
}

// debug timeline of one CTA (QgParams::trace): 16 %globaltimer stamps
__device__ unsigned long long qg_trace[16];
#define QG_STAMP(i)                                                                          \
  do {                                                                                       \
    if (INFERNO_KTRACE && p.trace && blockIdx.x == 0 && blockIdx.y == 0 && blockIdx.z == 0) qg_trace[i] = gtimer(); \
  } while (0)

template <int TYPE, int BN>
__global__ void __launch_bounds__(QG_THREADS, 1)
    qgemm_tc_kernel(const __grid_constant__ QgParams p, const __grid_constant__ QgMaps maps) {
  extern __shared__ uint8_t qg_smem_raw[];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int split = p.split;
  const int nsplit = split ? 2 : 1;
  const int NA = p.nas, NR = p.nrs, NB = p.nbs, KPS = p.kps;
  const bool spin = INFERNO_KTRACE && (p.dbgmode & 64);
  // ---- shared memory carve-up (1024-byte aligned operand tiles) ----
  uint8_t* base = (uint8_t*)(((uintptr_t)qg_smem_raw + 1023) & ~(uintptr_t)1023);
  uint8_t* sA = base;                                        // [NA][KPS][nsplit][16 KB]
  uint8_t* sB = sA + (size_t)NA * KPS * nsplit * QG_ATILE;   // [NB][nsplit][BN * 128]
  const int btile = BN * 128;
  uint8_t* sRaw = sB + (size_t)NB * nsplit * btile;          // [NR][128][slot]
  uint64_t* bars = (uint64_t*)(sRaw + (size_t)NR * QG_M * p.slot);
  uint64_t* a_full = bars;               // NA
  uint64_t* a_empty = a_full + NA;       // NA
  uint64_t* b_full = a_empty + NA;       // NB
  uint64_t* b_empty = b_full + NB;       // NB
  uint64_t* acc_full = b_empty + NB;     // 1
  uint32_t* s_tmem = (uint32_t*)(acc_full + 1);
  int* s_last = (int*)(s_tmem + 1);

  // ---- tile coordinates; blockIdx.z = slice of the K super-blocks ----
  const int mt = blockIdx.x, t0 = blockIdx.y * BN, kz = blockIdx.z, nz = gridDim.z;
  int sg = 0;
  while (sg + 1 < p.nseg && mt >= p.seg[sg + 1].mtile0) ++sg;
  const bool swiglu = p.epi == QG_SWIGLU;
  const int rows_per_tile = swiglu ? QG_M / 2 : QG_M;
  const int r0 = (mt - p.seg[sg].mtile0) * rows_per_tile;
  if (tid == 0) QG_STAMP(0);
  if (INFERNO_KTRACE && p.trace && tid == 0) atomicMax(&qg_trace[12], gtimer());       // latest CTA start
  const int sb0 = (int)((long long)kz * p.nsb / nz), sb1 = (int)((long long)(kz + 1) * p.nsb / nz);
  const int nsbz = sb1 - sb0, nk = 4 * nsbz;

  if (tid == 0) {
    for (int i = 0; i < NA; ++i) {
      mbar_init(&a_full[i], QG_DQ_WARPS);
      mbar_init(&a_empty[i], 1);
    }
    for (int i = 0; i < NB; ++i) {
      mbar_init(&b_full[i], 1);
      mbar_init(&b_empty[i], 1);
    }
    mbar_init(acc_full, 1);
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(s_tmem, BN < 32 ? 32 : BN);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *s_tmem;

  if (warp == 0) {
    // ================= activation producer =================
    // activations and token exponents come from the preceding kernels
    pdl_wait();
    if (lane == 0) QG_STAMP(8);
    if (lane == 0) {
      const uint32_t bx = (uint32_t)btile;
      for (int i = 0; i < nk; ++i) {
        const int bs = i % NB;
        if (i >= NB && !qg_wait(&b_empty[bs], ((i / NB) - 1) & 1, p.err, spin)) break;
        if (INFERNO_KTRACE && (p.dbgmode & 16)) {          // debug timing: no activation loads
          mbar_arrive(&b_full[bs]);
          continue;
        }
        mbar_arrive_expect_tx(&b_full[bs], bx * nsplit);
        uint8_t* bd = sB + (size_t)bs * nsplit * btile;
        const int kx = (4 * sb0 + i) * QG_BK;
        tma_load_2d(bd, &maps.hi, kx, t0, &b_full[bs]);
        if (split) tma_load_2d(bd + btile, &maps.lo, kx, t0, &b_full[bs]);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ================= MMA issuer =================
    if (lane == 0) {
      const uint32_t idesc = umma_idesc_f16(QG_M, BN);
      bool ok = true;
      for (int i = 0; i < nk && ok; ++i) {
        const int m = i / KPS, s2 = i - m * KPS, as = m % NA, bs = i % NB;
        if (s2 == 0) ok = qg_wait(&a_full[as], (m / NA) & 1, p.err, spin);
        ok = ok && qg_wait(&b_full[bs], (i / NB) & 1, p.err, spin);
        if (!ok) break;
        tc_fence_after();
        if (i == 0) QG_STAMP(3);
        const uint32_t a_hi = smem_u32(sA + (size_t)(as * KPS + s2) * nsplit * QG_ATILE);
        const uint32_t b_hi = smem_u32(sB + (size_t)bs * nsplit * btile);
        const uint64_t dah = umma_desc_sw128(a_hi), dbh = umma_desc_sw128(b_hi);
        const uint64_t dal = umma_desc_sw128(a_hi + QG_ATILE), dbl = umma_desc_sw128(b_hi + btile);
#pragma unroll
        for (int kk = 0; kk < QG_BK / 16; ++kk) {
          if (INFERNO_KTRACE && (p.dbgmode & 1)) break;
          const uint64_t o = (uint64_t)(2 * kk);     // +32 bytes along K
          umma_f16(tbase, dah + o, dbh + o, idesc, (i | kk) != 0);
          if (split && !(INFERNO_KTRACE && (p.dbgmode & 32))) {
            umma_f16(tbase, dah + o, dbl + o, idesc, 1);
            umma_f16(tbase, dal + o, dbh + o, idesc, 1);
          }
        }
        if (INFERNO_KTRACE && (p.dbgmode & 128)) {        // debug timing: plain arrivals instead of MMA commits
          if (s2 == KPS - 1) mbar_arrive(&a_empty[as]);
          mbar_arrive(&b_empty[bs]);
          continue;
        }
        if (s2 == KPS - 1) umma_commit(&a_empty[as]);
        umma_commit(&b_empty[bs]);
      }
      umma_commit(acc_full);
      QG_STAMP(5);
    }
    __syncwarp();
  } else {
    // ================= dequantize, then epilogue =================
    // thread (row dr, segment dseg) of warps 2..17.  The four threads of a
    // row stage its super-blocks themselves (16-byte cp.async of the aligned
    // superset, chunks dseg, dseg + 4, ...) into an NR-stage ring, and wait
    // for them with cp.async.wait_group: no producer warp, no mbarrier, and
    // the weights (constants) stream in before griddepcontrol.wait.
    const int du = tid - 64, dr = du >> 2, dseg = du & 3;
    int ds = sg, drow = r0 + dr;
    if (swiglu) {
      ds = dr < 64 ? 0 : 1;
      drow = r0 + (dr & 63);
    }
    const bool dvalid = drow < p.seg[ds].rows;
    const uintptr_t rowsrc = dvalid ? (uintptr_t)(p.seg[ds].W + (long long)drow * p.row_bytes) : 0;
    uint8_t* myraw = sRaw + (size_t)dr * p.slot;
    auto stage_raw = [&](int j) {
      if (dvalid && j < nsbz) {
        const uintptr_t a = rowsrc + (uintptr_t)(sb0 + j) * QgBlk<TYPE>::BB;
        const uintptr_t a0 = a & ~(uintptr_t)15, a1 = (a + QgBlk<TYPE>::BB + 15) & ~(uintptr_t)15;
        uint8_t* d = myraw + (size_t)(j % NR) * QG_M * p.slot;
        for (uintptr_t o = 16 * dseg; o < a1 - a0; o += 64)
          asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(d + o)), "l"(a0 + o) : "memory");
      }
      asm volatile("cp.async.commit_group;" ::: "memory");
    };
    for (int j = 0; j < NR - 1; ++j) stage_raw(j);
    const int sw = qg_exp_for(*p.wbound);     // set at finalize (constant weights)
    const float wscale = ldexpf(1.0f, sw);
    bool ok = true;
    for (int i = 0; i < nk && ok; ++i) {
      const int j = i >> 2, ks = i & 3, rs = j % NR, m = i / KPS, s2 = i - m * KPS, as = m % NA;
      if (ks == 0 && !(INFERNO_KTRACE && (p.dbgmode & 8))) {
        __syncwarp();                 // the row's threads are done with stage (j - 1) % NR
        stage_raw(j + NR - 1);
        if (NR == 3) asm volatile("cp.async.wait_group 2;" ::: "memory");
        else asm volatile("cp.async.wait_group 1;" ::: "memory");
        __syncwarp();                 // the row's four threads' copies are visible
      }
      if (s2 == 0 && m >= NA) ok = qg_wait(&a_empty[as], ((m / NA) - 1) & 1, p.err, spin);
      if (!ok) break;
      if (tid == 64 && i == 0) QG_STAMP(2);
      uint8_t* ah = sA + (size_t)(as * KPS + s2) * nsplit * QG_ATILE;
      uint32_t h[8], l[8];
      if (dvalid && !(INFERNO_KTRACE && (p.dbgmode & 2))) {
        const uintptr_t a = rowsrc + (uintptr_t)(sb0 + j) * QgBlk<TYPE>::BB;
        const uint8_t* rp = myraw + (size_t)rs * QG_M * p.slot + (a & 15);
        qg_dq16_split<TYPE>(rp, smem_u32(rp), ks, dseg, wscale, h, l);
      } else {
#pragma unroll
        for (int e = 0; e < 8; ++e) h[e] = l[e] = 0u;
      }
#pragma unroll
      for (int cc = 0; cc < 2; ++cc) {
        const int c = 2 * dseg + cc;
        const uint32_t sa = smem_u32(ah) + sw128_off(dr, c);
        sts128(sa, h[4 * cc], h[4 * cc + 1], h[4 * cc + 2], h[4 * cc + 3]);
        if (split) sts128(sa + QG_ATILE, l[4 * cc], l[4 * cc + 1], l[4 * cc + 2], l[4 * cc + 3]);
      }
      if (s2 == KPS - 1) {
        if (!(INFERNO_KTRACE && (p.dbgmode & 4))) fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&a_full[as]);
      }
    }
    asm volatile("cp.async.wait_all;" ::: "memory");
    if (tid == 64) QG_STAMP(4);
    {
      // ---- epilogue: all 16 dequantizing warps.  Warp w reads TMEM lane
      // quarter w & 3 (thread = tile row) and column group (w - 2) >> 2 ----
      pdl_wait();      // residual rows (QG_ADD) and the token exponents
      const int q = warp & 3, cg = (warp - 2) >> 2;
      constexpr int CW = BN / 4;                 // columns per warp
      const int c_lo = cg * CW;
      const int r = 32 * q + lane;
      int s = sg, row = r0 + r;
      if (swiglu) {
        s = r < 64 ? 0 : 1;
        row = r0 + (r & 63);
      }
      const bool valid = row < p.seg[s].rows;
      float* cs = (float*)(s_last + 4);          // [BN] per-column descale
      if (du < BN) {
        const int t = t0 + du;
        cs[du] = t < p.T ? ldexpf(1.0f, -sw - (int)p.xexp[t]) : 0.f;
      }
      if (ok) ok = mbar_wait(acc_full, 0, p.err);
      tc_fence_after();
      if (tid == 64) QG_STAMP(6);
      const uint32_t taddr = tbase + ((uint32_t)(32 * q) << 16) + (uint32_t)c_lo;
      // split K: every slice parks its raw accumulator tile in the workspace;
      // the slice that arrives last sums them in slice order (deterministic)
      // and applies the epilogue
      const long long tile = (long long)blockIdx.y * gridDim.x + mt;
      float* wsl = nz > 1 ? p.ws + (tile * nz) * (long long)(BN * QG_M) : nullptr;
      bool last = true;
      if (nz > 1) {
#pragma unroll
        for (int c0 = 0; c0 < CW; c0 += 8) {
          uint32_t v[8];
          tmem_ld_x8(taddr + (uint32_t)c0, v);
          tmem_wait_ld();
#pragma unroll
          for (int j = 0; j < 8; ++j)
            __stcg(wsl + (long long)kz * BN * QG_M + (c_lo + c0 + j) * QG_M + r, __uint_as_float(v[j]));
        }
        __threadfence();
        named_bar_sync(1, 32 * QG_DQ_WARPS);
        if (tid == 64) {
          const int prev = atomicAdd(&p.tickets[tile], 1);
          *s_last = prev == nz - 1;
          if (prev == nz - 1) p.tickets[tile] = 0;      // ready for the next launch
        }
        named_bar_sync(1, 32 * QG_DQ_WARPS);
        last = *s_last != 0;
        if (last) __threadfence();
        if (tid == 64) QG_STAMP(9);
      } else {
        named_bar_sync(1, 32 * QG_DQ_WARPS);     // cs[] written
      }
      if (last) {
        float* xch = (float*)sA;                 // SwiGLU: [128][BN] (the A ring is free now)
#pragma unroll
        for (int c0 = 0; c0 < CW; c0 += 8) {
          float v[8];
          if (nz > 1) {
#pragma unroll
            for (int j = 0; j < 8; ++j) v[j] = 0.f;
            for (int z = 0; z < nz; ++z)
#pragma unroll
              for (int j = 0; j < 8; ++j) v[j] += __ldcg(wsl + (long long)z * BN * QG_M + (c_lo + c0 + j) * QG_M + r);
          } else {
            uint32_t u[8];
            tmem_ld_x8(taddr + (uint32_t)c0, u);
            tmem_wait_ld();
#pragma unroll
            for (int j = 0; j < 8; ++j) v[j] = __uint_as_float(u[j]);
          }
          if (!ok) continue;
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const int c = c_lo + c0 + j, t = t0 + c;
            const float val = v[j] * cs[c];
            if (swiglu) {
              xch[(r < 64 ? 64 + r : r - 64) * BN + c] = val;   // gate rows beside the up rows
            } else if (valid && t < p.T) {
              float* y = p.seg[s].y + (long long)t * p.y_stride + row;
              if (p.epi == QG_ADD) *y += val;
              else *y = val;
            }
          }
        }
        if (swiglu) {
          named_bar_sync(1, 32 * QG_DQ_WARPS);
          // thread (gate row rr, column group): 64 rows x 8 groups over 512 threads
          const int rr = du & 63, g8 = du >> 6;
          const int grow = r0 + rr;
          if (grow < p.seg[0].rows && ok) {
            for (int c = g8; c < BN; c += 8) {
              const int t = t0 + c;
              if (t >= p.T) break;
              const float g = xch[(64 + rr) * BN + c], u = xch[rr * BN + c];
              p.seg[0].y[(long long)t * p.y_stride + grow] = g / (1.0f + expf(-g)) * u;   // src/ModelCPU.jl:455-468
            }
          }
        }
      }
    }
  }
  if (tid == 64) QG_STAMP(7);
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tbase, BN < 32 ? 32 : BN);
  }
  if (tid == 32) QG_STAMP(10);
  if (INFERNO_KTRACE && p.trace && tid == 32) atomicMax(&qg_trace[11], gtimer());      // latest CTA end
  if (INFERNO_KTRACE && p.trace && tid == 64 && p.seg[0].rows > 0) atomicMax(&qg_trace[13], (unsigned long long)(nk));
}

// ---------------------------------------------------------------------------
// activations -> fp16 hi / lo rows with a per-token power-of-two scale
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) qg_act_kernel(const float* x, long long x_stride, int K, int pro,
                                                     const float* pro_w, const float* pro_z, int group, float eps,
                                                     __half* xhi, __half* xlo, float* xexp, int T) {
  __shared__ float red[2][8];
  const int t = blockIdx.x, tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
  if (t >= T) {    // padding rows of the last token tile
    pdl_wait();
    pdl_trigger();
    for (int i = 2 * tid; i < K; i += 512) {
      *(__half2*)&xhi[(long long)t * K + i] = __floats2half2_rn(0.f, 0.f);
      *(__half2*)&xlo[(long long)t * K + i] = __floats2half2_rn(0.f, 0.f);
    }
    if (tid == 0) xexp[t] = 0.f;
    return;
  }
  const float* xr = x + (long long)t * x_stride;
  const float* zr = pro_z ? pro_z + (long long)t * x_stride : nullptr;
  // shared: the row [K], then the norm weights (K for RMSNorm, `group` for
  // the head norm) -- constants, staged before griddepcontrol.wait
  extern __shared__ float qa_v[];
  float* wsm = qa_v + K;
  const int nw = pro == PRO_RMSNORM ? K : pro == PRO_HEADNORM_GATE ? group : 0;
  for (int i = tid; i < nw; i += 256) wsm[i] = pro_w[i];
  pdl_wait();
  pdl_trigger();
  // one global pass over the row (and z), with the RMSNorm statistics
  float ss = 0.f;
  for (int i = tid; i < K; i += 256) {
    const float v = xr[i];
    qa_v[i] = v;
    ss = fmaf(v, v, ss);
  }
  ss = warp_sum(ss);
  if (lane == 0) red[0][w] = ss;
  __syncthreads();
  float tot = 0.f;
  for (int i = 0; i < 8; ++i) tot += red[0][i];
  const float inv = pro == PRO_RMSNORM ? 1.0f / sqrtf(tot / (float)K + eps) : 1.0f;
  float amax = 0.f;
  if (pro == PRO_HEADNORM_GATE) {
    // head-norm x SiLU(z) (the ssm_out input): one warp per head group
    for (int h = w; h < K / group; h += 8) {
      float hs = 0.f;
      for (int e = lane; e < group; e += 32) hs = fmaf(qa_v[h * group + e], qa_v[h * group + e], hs);
      hs = warp_sum(hs);
      const float sc = 1.0f / sqrtf(hs / (float)group + eps);
      for (int e = lane; e < group; e += 32) {
        const int i = h * group + e;
        const float z = zr[i];
        const float v = qa_v[i] * sc * wsm[e] * (z / (1.0f + expf(-z)));
        qa_v[i] = v;
        amax = fmaxf(amax, fabsf(v));
      }
    }
  } else {
    for (int i = tid; i < K; i += 256) {
      const float v = pro == PRO_RMSNORM ? qa_v[i] * inv * wsm[i] : qa_v[i];
      qa_v[i] = v;
      amax = fmaxf(amax, fabsf(v));
    }
  }
  amax = warp_max(amax);
  __syncthreads();
  if (lane == 0) red[1][w] = amax;
  __syncthreads();
  float m = 0.f;
  for (int i = 0; i < 8; ++i) m = fmaxf(m, red[1][i]);
  const int e = qg_exp_for(m);
  const float sc = ldexpf(1.0f, e);
  for (int i = 2 * tid; i < K; i += 512) {
    const float a = qa_v[i] * sc, b = qa_v[i + 1] * sc;
    const __half2 h = __floats2half2_rn(a, b);
    const float2 hf = __half22float2(h);
    *(__half2*)&xhi[(long long)t * K + i] = h;
    *(__half2*)&xlo[(long long)t * K + i] = __floats2half2_rn(a - hf.x, b - hf.y);
  }
  if (tid == 0) xexp[t] = (float)e;
}

// bound of |w| over the weight blocks of a matrix: |d| * 63 * 63 + |dmin| * 63
// for the K-quants (covers Q4_K / Q5_K / Q6_K codes), |d| * 128 for Q8_0
__global__ void qg_wbound_kernel(const uint8_t* W, long long nblocks, int type, float* out) {
  float m = 0.f;
  for (long long b = (long long)blockIdx.x * blockDim.x + threadIdx.x; b < nblocks;
       b += (long long)gridDim.x * blockDim.x) {
    float v;
    if (type == T_Q6_K) {
      const uint8_t* p = W + b * 210 + 208;
      v = fabsf(h2f_bits((uint16_t)(p[0] | (p[1] << 8)))) * 128.f * 32.f;
    } else if (type == T_Q8_0) {
      const uint8_t* p = W + b * 34;
      v = fabsf(h2f_bits((uint16_t)(p[0] | (p[1] << 8)))) * 128.f;
    } else {
      const uint8_t* p = W + b * (type == T_Q4_K ? 144 : 176);
      v = fabsf(h2f_bits((uint16_t)(p[0] | (p[1] << 8)))) * 63.f * 31.f +
          fabsf(h2f_bits((uint16_t)(p[2] | (p[3] << 8)))) * 63.f;
    }
    if (v == v) m = fmaxf(m, v);
  }
  m = warp_max(m);
  if ((threadIdx.x & 31) == 0) atomicMax((int*)out, __float_as_int(m));
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
namespace {

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = (EncodeTiledFn)p;
  });
  return fn;
}

// [T][K] fp16 rows, box = 64 x BN, SWIZZLE_128B, zero fill past T
int make_act_map(CUtensorMap* m, const __half* base, int K, int T, int BN) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return set_error(INFERNO_ECUDA, "qgemm: cuTensorMapEncodeTiled is not available");
  if (((uintptr_t)base & 15) || K % QG_BK)
    return set_error(INFERNO_EINVAL, "qgemm: activation rows must be 16-byte aligned with K %% 64 == 0");
  const cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)T};
  const cuuint64_t strides[1] = {(cuuint64_t)K * 2};
  const cuuint32_t box[2] = {(cuuint32_t)QG_BK, (cuuint32_t)BN};
  const cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, (void*)base, dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(INFERNO_ECUDA, "qgemm: cuTensorMapEncodeTiled failed (%d)", (int)r);
  return 0;
}

template <int TYPE, int BN>
cudaError_t qg_launch_bn(const QgParams& p, const QgMaps& maps, dim3 grid, size_t smem, cudaStream_t st, bool pdl) {
  static DeviceOnce once;
  cudaError_t ea = once.run([] {
    return cudaFuncSetAttribute(qgemm_tc_kernel<TYPE, BN>, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
  });
  if (ea != cudaSuccess) return ea;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(QG_THREADS);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, qgemm_tc_kernel<TYPE, BN>, p, maps);
}

template <int TYPE>
cudaError_t qg_launch(const QgParams& p, const QgMaps& maps, int BN, dim3 grid, size_t smem, cudaStream_t st,
                      bool pdl) {
  switch (BN) {
    case 32: return qg_launch_bn<TYPE, 32>(p, maps, grid, smem, st, pdl);
    case 64: return qg_launch_bn<TYPE, 64>(p, maps, grid, smem, st, pdl);
    default: return qg_launch_bn<TYPE, 128>(p, maps, grid, smem, st, pdl);
  }
}

}  // namespace

bool qgemm_supported(int type) { return type == T_Q4_K || type == T_Q5_K || type == T_Q6_K || type == T_Q8_0; }

int qgemm_bn(int T) { return T <= 32 ? 32 : T <= 64 ? 64 : 128; }
// debug: the last traced launch's stamps (ns, relative to stamp 0)
int qgemm_trace_read(long long* out16) {
  unsigned long long h[16];
  if (cudaMemcpyFromSymbol(h, qg_trace, sizeof h) != cudaSuccess) return -1;
  for (int i = 0; i < 16; ++i) out16[i] = h[i] ? (long long)(h[i] - h[0]) : -1;
  return 0;
}

size_t qgemm_ws_bytes() { return (size_t)QG_WS_CTAS * 128 * QG_M * 4; }

int qgemm_rows_padded(int T) {
  const int bn = qgemm_bn(T);
  return (T + bn - 1) / bn * bn;
}

int launch_qgemm_act(const float* x, long long x_stride, int K, int T, int pro, const float* pro_w,
                     const float* pro_z, int group, float eps, __half* xhi, __half* xlo, float* xexp,
                     cudaStream_t st, bool pdl) {
  if (T <= 0) return 0;
  if (K % 2 || K > 16384) return set_error(INFERNO_EINVAL, "qgemm activations: K %d", K);
  static DeviceOnce once;
  cudaError_t ea = once.run(
      [] { return cudaFuncSetAttribute(qg_act_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 128 * 1024); });
  if (ea != cudaSuccess) return set_error(INFERNO_ECUDA, "qgemm activations attribute: %s", cudaGetErrorString(ea));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(qgemm_rows_padded(T));
  cfg.blockDim = dim3(256);
  cfg.dynamicSmemBytes = (size_t)K * 8;
  cfg.stream = st;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = pdl ? 1 : 0;
  cudaError_t e = cudaLaunchKernelEx(&cfg, qg_act_kernel, x, x_stride, K, pro, pro_w, pro_z, group, eps, xhi, xlo,
                                     xexp, T);
  return e == cudaSuccess ? 0 : set_error(INFERNO_ECUDA, "qgemm activations launch: %s", cudaGetErrorString(e));
}

int launch_qgemm_wbound(int type, const void* W, long long rows, int K, float* out, cudaStream_t st, bool reset) {
  const long long nblocks = rows * (K / (type == T_Q8_0 ? 32 : 256));
  cudaError_t e = reset ? cudaMemsetAsync(out, 0, 4, st) : cudaSuccess;
  if (e != cudaSuccess) return set_error(INFERNO_ECUDA, "qgemm weight bound: %s", cudaGetErrorString(e));
  const int grid = (int)std::min<long long>(1184, (nblocks + 255) / 256);
  if (grid > 0) qg_wbound_kernel<<<grid, 256, 0, st>>>((const uint8_t*)W, nblocks, type, out);
  e = cudaGetLastError();
  return e == cudaSuccess ? 0 : set_error(INFERNO_ECUDA, "qgemm weight bound: %s", cudaGetErrorString(e));
}

int launch_qgemm(const QgemmCall& c, cudaStream_t st, bool pdl) {
  if (!qgemm_supported(c.type)) return set_error(INFERNO_EINVAL, "qgemm: type %d has no tensor-core path", c.type);
  if (c.K % 256 || c.K <= 0) return set_error(INFERNO_EINVAL, "qgemm: K %d not a multiple of 256", c.K);
  if (c.T <= 0) return 0;
  if (c.nmats < 1 || c.nmats > 4 || (c.epi == QG_SWIGLU && c.nmats != 2))
    return set_error(INFERNO_EINVAL, "qgemm: bad matrix count %d", c.nmats);
  const int BN = qgemm_bn(c.T);
  QgParams p = {};
  const int rows_per_tile = c.epi == QG_SWIGLU ? QG_M / 2 : QG_M;
  int mt = 0;
  for (int i = 0; i < c.nmats; ++i) {
    p.seg[i].W = (const uint8_t*)c.mats[i].W;
    p.seg[i].y = c.mats[i].y;
    p.seg[i].rows = c.mats[i].rows;
    p.seg[i].mtile0 = mt;
    if (!(c.epi == QG_SWIGLU && i == 1)) mt += (c.mats[i].rows + rows_per_tile - 1) / rows_per_tile;
    else p.seg[i].mtile0 = INT_MAX;
  }
  if (c.epi == QG_SWIGLU && c.mats[0].rows != c.mats[1].rows)
    return set_error(INFERNO_EINVAL, "qgemm: SwiGLU matrices differ in rows");
  p.nseg = c.nmats;
  p.n_mtiles = mt;
  p.K = c.K;
  p.nsb = c.K / 256;
  const int bb = c.type == T_Q4_K ? 144 : c.type == T_Q5_K ? 176 : c.type == T_Q6_K ? 210 : 272;
  p.row_bytes = (long long)p.nsb * bb;
  p.slot = (bb + 15) / 16 * 16 + 16;           // aligned superset of one super-block
  p.T = c.T;
  p.y_stride = c.y_stride;
  p.epi = c.epi;
  p.split = c.split ? 1 : 0;
  p.xexp = c.xexp;
  p.wbound = c.wbound;
  p.err = c.err;
  const int nsplit = p.split ? 2 : 1;
  const size_t rstage = (size_t)QG_M * p.slot;
  const size_t bstage = (size_t)nsplit * BN * 128;
  const size_t cap = 227 * 1024 - 1024 - 1024;
  // Ring depths.  The activation (B) tiles come from L2 by TMA with a
  // latency of about a microsecond, and a B stage can only be refilled once
  // the MMAs of its step completed: steps run at ~latency / NB, so B gets
  // the depth (up to 8 stages); dequantized A tiles need only two stages (the
  // dequantizing warps work one step ahead of the MMA), the raw super-block
  // ring three (two super-blocks of HBM prefetch).
  // K steps per A stage: INFERNO_QG_KPS=2 hands two K steps from the
  // dequantizing warps to the MMA issuer at once (measured: no faster than
  // one -- the step time is set by the dequantization chain itself).
  static const int env_kps = getenv("INFERNO_QG_KPS") ? atoi(getenv("INFERNO_QG_KPS")) : 1;
  int kps = env_kps == 1 ? 1 : 2, nas = 2, nrs = 3, nbs = 8;
  auto need = [&] { return (size_t)nas * kps * nsplit * QG_ATILE + nrs * rstage + nbs * bstage; };
  auto shrink = [&] {
    while (need() > cap && nbs > 3) --nbs;
    while (need() > cap && nrs > 2) --nrs;
  };
  shrink();
  if (need() > cap && kps == 2) {
    kps = 1;
    nrs = 3;
    nbs = 8;
    shrink();
  }
  while (need() > cap && nbs > 2) --nbs;
  if (need() > cap) return set_error(INFERNO_EINVAL, "qgemm: tiles do not fit shared memory");
  p.nbs = nbs;
  p.nas = nas;
  p.nrs = nrs;
  p.kps = kps;
  const size_t smem = 1024 + need() + 1024;     // alignment slack, barriers, column scales
  // split K while the output tiles leave SMs idle (one CTA per SM)
  const int ntt = (c.T + BN - 1) / BN, tiles = mt * ntt;
  int sms = 148, dev = 0;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  int nz = 1;
  if (c.ws && c.tickets && tiles < sms) nz = std::max(1, std::min(p.nsb, sms / tiles));
  while (nz > 1 && tiles * nz > QG_WS_CTAS) --nz;
  p.ws = c.ws;
  p.tickets = c.tickets;
  static const bool trace = getenv("INFERNO_QG_TRACE") != nullptr;
  p.trace = trace ? 1 : 0;
  if (trace) {
    static const unsigned long long zeros[16] = {};
    cudaMemcpyToSymbolAsync(qg_trace, zeros, sizeof zeros, 0, cudaMemcpyHostToDevice, st);
  }
  static const int dbgmode = getenv("INFERNO_QG_DBGMODE") ? atoi(getenv("INFERNO_QG_DBGMODE")) : 0;
  p.dbgmode = dbgmode;
  QgMaps maps;
  memset(&maps, 0, sizeof maps);
  int rc;
  // the activation rows are padded (zeros) to whole BN tiles
  const int Tpad = qgemm_rows_padded(c.T);
  if ((rc = make_act_map(&maps.hi, (const __half*)c.xhi, c.K, Tpad, BN))) return rc;
  if ((rc = make_act_map(&maps.lo, (const __half*)(c.split ? c.xlo : c.xhi), c.K, Tpad, BN))) return rc;
  const dim3 grid(mt, ntt, nz);
  cudaError_t e;
  switch (c.type) {
    case T_Q4_K: e = qg_launch<T_Q4_K>(p, maps, BN, grid, smem, st, pdl); break;
    case T_Q5_K: e = qg_launch<T_Q5_K>(p, maps, BN, grid, smem, st, pdl); break;
    case T_Q6_K: e = qg_launch<T_Q6_K>(p, maps, BN, grid, smem, st, pdl); break;
    default: e = qg_launch<T_Q8_0>(p, maps, BN, grid, smem, st, pdl); break;
  }
  return e == cudaSuccess ? 0 : set_error(INFERNO_ECUDA, "qgemm launch: %s", cudaGetErrorString(e));
}

}  // namespace inf

namespace inf {

int qgemm_from_gemv(const GemvCall& c, cudaStream_t st) {
  static const bool off = getenv("INFERNO_NO_TC_GEMM") != nullptr;
  static const bool fast = getenv("INFERNO_TC_GEMM_FP16") != nullptr;
  if (off || c.nb < 16 || !qgemm_supported(c.type) || c.inner % 256 || c.nxv != 1 || c.xch_wk >= 0 ||
      c.xch_rk >= 0 || c.force_r || (c.pro != PRO_NONE && c.pro != PRO_RMSNORM) ||
      (c.epi != EPI_STORE && c.epi != EPI_ADD && c.epi != EPI_SWIGLU) || c.x_stride % 2)
    return 1;
  for (int i = 0; i < c.nmats; ++i)
    if (c.mats[i].indirect || !c.mats[i].y && !(c.epi == EPI_SWIGLU && i == 1)) return 1;
  const int T = c.nb, K = c.inner, Tpad = qgemm_rows_padded(T);
  // stream-ordered scratch: fp16 hi / lo activations (padded to whole token
  // tiles), token exponents, the weight bound
  const size_t act = (size_t)Tpad * K * 2;
  const size_t wsb = qgemm_ws_bytes();
  const size_t bytes = 2 * act + (size_t)Tpad * 4 + 256 + wsb + QGEMM_TICKETS * 4;
  char* buf = nullptr;
  INF_CUDA_TRY(cudaMallocAsync((void**)&buf, bytes, st));
  __half* xhi = (__half*)buf;
  __half* xlo = (__half*)(buf + act);
  float* xexp = (float*)(buf + 2 * act);
  float* wb = xexp + Tpad;
  float* ws = (float*)(buf + 2 * act + (size_t)Tpad * 4 + 256);
  int* tickets = (int*)((char*)ws + wsb);
  INF_CUDA_TRY(cudaMemsetAsync(tickets, 0, QGEMM_TICKETS * 4, st));
  int rc = launch_qgemm_act(c.x, c.x_stride, K, T, c.pro, c.pro_w, c.pro_z, c.pro_group, c.eps, xhi, xlo, xexp, st,
                            false);
  // one bound over every matrix of the call (a common weight scale): the
  // bound kernel folds into its output with atomicMax
  for (int i = 0; i < c.nmats && !rc; ++i)
    rc = launch_qgemm_wbound(c.type, c.mats[i].W, c.mats[i].rows, K, wb, st, i == 0);
  if (!rc) {
    QgemmCall q;
    q.type = c.type;
    q.K = K;
    for (int i = 0; i < c.nmats; ++i) q.mats[i] = c.mats[i];
    q.nmats = c.nmats;
    q.T = T;
    q.xhi = xhi;
    q.xlo = xlo;
    q.xexp = xexp;
    q.y_stride = c.y_stride ? c.y_stride : c.mats[0].rows;
    q.epi = c.epi == EPI_ADD ? 1 : c.epi == EPI_SWIGLU ? 2 : 0;
    q.wbound = wb;
    q.err = c.err ? c.err : device_error_word(0);
    q.split = !fast;
    q.ws = ws;
    q.tickets = tickets;
    rc = launch_qgemm(q, st, false);
  }
  cudaError_t ef = cudaFreeAsync(buf, st);
  if (!rc && ef != cudaSuccess) rc = set_error(INFERNO_ECUDA, "qgemm scratch: %s", cudaGetErrorString(ef));
  return rc;
}

}  // namespace inf
