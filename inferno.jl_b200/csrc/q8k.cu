// The Q8_K activation path of the reference's quantized C kernels
// (src/kernels/quant_kernels.c): quantize_row_q8_K (:166-196) and the block
// dot products vec_dot_q{4,5,6}_K_q8_K (:204-519) and vec_dot_q8_0_q8_0
// (:531-559), exported with the same symbols by the compatibility tier.
//
// Results are bit-identical to the reference's AVX2 + FMA build: a block's
// 256-bit integer lanes (lane k of a 32-byte chunk = bytes 4k..4k+3) are
// exact int32 sums, every lane keeps its own fp32 accumulator updated with one
// fma per block in block order, and the eight lanes are combined in
// hsum_float_8's order.  Lane sums are computed in parallel (one thread per
// block x lane); the per-lane fma chains run serially in block order.  These
// are per-call helpers of the compatibility tier, not the decode hot path.
#include "internal.h"
#include "common.cuh"

namespace inf {

namespace {

constexpr int Q8K_BYTES = 292;  // float d; int8 qs[256]; int16 bsums[16]
constexpr int TILE = 32;        // blocks per tile: 32 blocks x 8 lanes = 256 threads

__device__ __forceinline__ uint16_t q_ld16(const uint8_t* p) { return (uint16_t)(p[0] | (p[1] << 8)); }
__device__ __forceinline__ float q_ldf(const uint8_t* p) {
  return __uint_as_float((uint32_t)p[0] | ((uint32_t)p[1] << 8) | ((uint32_t)p[2] << 16) | ((uint32_t)p[3] << 24));
}
__device__ __forceinline__ int16_t q_ldi16(const uint8_t* p) { return (int16_t)q_ld16(p); }

__device__ __forceinline__ void k4_scale_min(const uint8_t* s, int j, int& sc, int& m) {
  if (j < 4) { sc = s[j] & 63; m = s[j + 4] & 63; }
  else { sc = (s[j + 4] & 15) | ((s[j - 4] >> 6) << 4); m = (s[j + 4] >> 4) | ((s[j] >> 6) << 4); }
}

__global__ void q8k_quantize_kernel(const float* __restrict__ x, uint8_t* __restrict__ y) {
  __shared__ float red[8];
  const int t = threadIdx.x, w = t >> 5, ln = t & 31;
  const float v = x[(size_t)blockIdx.x * 256 + t];
  float a = fabsf(v);
#pragma unroll
  for (int o = 16; o; o >>= 1) a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, o));
  if (!ln) red[w] = a;
  __syncthreads();
  float amax = red[0];
#pragma unroll
  for (int i = 1; i < 8; ++i) amax = fmaxf(amax, red[i]);
  const float d = __fdiv_rn(amax, 127.0f);
  const float id = d != 0.0f ? __frcp_rn(d) : 0.0f;
  const int q = (int)(int8_t)(int)roundf(__fmul_rn(v, id));
  uint8_t* yb = y + (size_t)blockIdx.x * Q8K_BYTES;
  yb[4 + t] = (uint8_t)q;
  int s = q;
#pragma unroll
  for (int o = 8; o; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  if ((t & 15) == 0) {
    const uint16_t u = (uint16_t)(int16_t)s;
    yb[260 + 2 * (t >> 4)] = (uint8_t)u;
    yb[261 + 2 * (t >> 4)] = (uint8_t)(u >> 8);
  }
  if (t == 0) {
    const uint32_t u = __float_as_uint(d);
    yb[0] = (uint8_t)u; yb[1] = (uint8_t)(u >> 8); yb[2] = (uint8_t)(u >> 16); yb[3] = (uint8_t)(u >> 24);
  }
}

// integer lane k of block xb / yb; *mins gets the min-term lane (Q4_K / Q5_K, k < 4)
template <int TYPE>
__device__ int32_t lane_sum(const uint8_t* xb, const uint8_t* yb, int k, int32_t* mins) {
  int32_t lane = 0;
  if (TYPE == T_Q4_K || TYPE == T_Q5_K) {
    const bool q5 = TYPE == T_Q5_K;
    const int8_t* q8 = (const int8_t*)(yb + 4);
    const uint8_t* qh = xb + 16;
    const uint8_t* qs = xb + (q5 ? 48 : 16);
    for (int j = 0; j < 4; ++j) {
      int sc0, sc1, m0, m1;
      k4_scale_min(xb + 4, 2 * j, sc0, m0);
      k4_scale_min(xb + 4, 2 * j + 1, sc1, m1);
      int lo = 0, hi = 0;
#pragma unroll
      for (int b = 4 * k; b < 4 * k + 4; ++b) {
        int ql = qs[32 * j + b] & 15, qhh = qs[32 * j + b] >> 4;
        if (q5) { ql |= ((qh[b] >> (2 * j)) & 1) << 4; qhh |= ((qh[b] >> (2 * j + 1)) & 1) << 4; }
        lo += ql * q8[64 * j + b];
        hi += qhh * q8[64 * j + 32 + b];
      }
      lane += sc0 * lo + sc1 * hi;
    }
    if (k < 4) {
      int sa, sb, ma, mb;
      k4_scale_min(xb + 4, 2 * k, sa, ma);
      k4_scale_min(xb + 4, 2 * k + 1, sb, mb);
      // _mm_hadd_epi16 of the bsums wraps at 16 bits
      const int16_t s0 = (int16_t)(q_ldi16(yb + 260 + 8 * k) + q_ldi16(yb + 262 + 8 * k));
      const int16_t s1 = (int16_t)(q_ldi16(yb + 264 + 8 * k) + q_ldi16(yb + 266 + 8 * k));
      *mins = ma * s0 + mb * s1;
    }
  } else if (TYPE == T_Q6_K) {
    const int8_t* q8 = (const int8_t*)(yb + 4);
    const uint8_t *ql = xb, *qh = xb + 128;
    const int8_t* sc = (const int8_t*)(xb + 192);
    for (int j = 0; j < 2; ++j)
      for (int t = 0; t < 4; ++t) {
        int s = 0;
#pragma unroll
        for (int b = 4 * k; b < 4 * k + 4; ++b) {
          const uint8_t lb = ql[64 * j + (t & 1) * 32 + b];
          const int q = ((t < 2 ? lb : lb >> 4) & 15) | (((qh[32 * j + b] >> (2 * t)) & 3) << 4);
          s += (q - 32) * q8[128 * j + 32 * t + b];
        }
        lane += sc[8 * j + 2 * t + (k >= 4)] * s;
      }
  } else {  // Q8_0 x Q8_0: |x| times y with x's sign (int8 wrap), pair sums saturated to int16
    const int8_t *qx = (const int8_t*)(xb + 2), *qy = (const int8_t*)(yb + 2);
    for (int p = 0; p < 2; ++p) {
      int pair = 0;
      for (int b = 4 * k + 2 * p; b < 4 * k + 2 * p + 2; ++b) {
        const int ax = qx[b] < 0 ? -(int)qx[b] : qx[b];
        const int sy = qx[b] < 0 ? (int)(int8_t)(-qy[b]) : (qx[b] == 0 ? 0 : qy[b]);
        pair += ax * sy;
      }
      lane += min(32767, max(-32768, pair));
    }
  }
  return lane;
}

template <int TYPE>
__global__ void __launch_bounds__(256) q8k_vec_dot_kernel(const uint8_t* __restrict__ x,
                                                          const uint8_t* __restrict__ y, int nb,
                                                          float* __restrict__ out) {
  constexpr int XB = TYPE == T_Q4_K ? 144 : TYPE == T_Q5_K ? 176 : TYPE == T_Q6_K ? 210 : 34;
  constexpr int YB = TYPE == T_Q8_0 ? 34 : Q8K_BYTES;
  constexpr bool MINS = TYPE == T_Q4_K || TYPE == T_Q5_K;
  __shared__ int32_t s_lane[TILE][8];
  __shared__ int32_t s_min[TILE][4];
  __shared__ float s_acc[12];
  const int t = threadIdx.x, ib = t >> 3, k = t & 7;
  float acc = 0.0f;  // thread c < 8: lane c; thread 8..11: Q4_K min lane c-8; thread 8: Q5_K summs
  for (int i0 = 0; i0 < nb; i0 += TILE) {
    const int i = i0 + ib;
    if (i < nb) {
      int32_t m = 0;
      s_lane[ib][k] = lane_sum<TYPE>(x + (size_t)i * XB, y + (size_t)i * YB, k, &m);
      if (MINS && k < 4) s_min[ib][k] = m;
    }
    __syncthreads();
    const int n = min(TILE, nb - i0);
    if (t < 8) {
      for (int b = 0; b < n; ++b) {
        const uint8_t *xb = x + (size_t)(i0 + b) * XB, *yb = y + (size_t)(i0 + b) * YB;
        float d;
        if (TYPE == T_Q8_0) d = __fmul_rn(h2f_bits(q_ld16(xb)), h2f_bits(q_ld16(yb)));
        else d = __fmul_rn(q_ldf(yb), h2f_bits(q_ld16(xb + (TYPE == T_Q6_K ? 208 : 0))));
        acc = fmaf(d, (float)s_lane[b][t], acc);
      }
    } else if (MINS && t < 12) {
      for (int b = 0; b < n; ++b) {
        const uint8_t *xb = x + (size_t)(i0 + b) * XB, *yb = y + (size_t)(i0 + b) * YB;
        const float dmin = -__fmul_rn(q_ldf(yb), h2f_bits(q_ld16(xb + 2)));
        if (TYPE == T_Q4_K) {
          acc = fmaf(dmin, (float)s_min[b][t - 8], acc);
        } else if (t == 8) {
          const int32_t h = (s_min[b][0] + s_min[b][1]) + (s_min[b][2] + s_min[b][3]);
          acc = fmaf(dmin, (float)h, acc);
        }
      }
    }
    __syncthreads();
  }
  if (t < 12) s_acc[t] = acc;
  __syncthreads();
  if (t == 0) {
    const float* a = s_acc;
    const float s0 = a[4] + a[0], s1 = a[5] + a[1], s2 = a[6] + a[2], s3 = a[7] + a[3];
    float r = (s0 + s2) + (s1 + s3);
    if (TYPE == T_Q4_K) r = r + ((a[8] + a[10]) + (a[9] + a[11]));
    if (TYPE == T_Q5_K) r = r + a[8];
    *out = r;
  }
}

// q{4,5,6}_k_gemv of the reference (quant_kernels.c:602-650): out[row] =
// vec_dot(row, quantize_row_q8_K(x)).  One warp per row; lane (b, k) = (lane
// / 8, lane % 8) computes integer lane k of block c0 + b, and every thread
// with lane % 8 == k replays the fma chain of lane k in block order through
// shuffles, so each row's result equals the reference's vec_dot bit for bit.
template <int TYPE>
__global__ void __launch_bounds__(256) q8k_gemv_kernel(const uint8_t* __restrict__ W,
                                                       const uint8_t* __restrict__ y8, int nb, int rows,
                                                       float* __restrict__ out) {
  constexpr int XB = TYPE == T_Q4_K ? 144 : TYPE == T_Q5_K ? 176 : 210;
  constexpr bool MINS = TYPE == T_Q4_K || TYPE == T_Q5_K;
  const int lane = threadIdx.x & 31, b = lane >> 3, k = lane & 7;
  const int row = blockIdx.x * 8 + (threadIdx.x >> 5);
  if (row >= rows) return;
  const uint8_t* wr = W + (size_t)row * nb * XB;
  float acc = 0.0f, accm = 0.0f;
  for (int c0 = 0; c0 < nb; c0 += 4) {
    const int i = c0 + b;
    int32_t v = 0, m = 0;
    float d = 0.0f, dmin = 0.0f;
    if (i < nb) {
      const uint8_t *xb = wr + (size_t)i * XB, *yb = y8 + (size_t)i * Q8K_BYTES;
      v = lane_sum<TYPE>(xb, yb, k, &m);
      d = __fmul_rn(q_ldf(yb), h2f_bits(q_ld16(xb + (TYPE == T_Q6_K ? 208 : 0))));
      if (MINS) dmin = -__fmul_rn(q_ldf(yb), h2f_bits(q_ld16(xb + 2)));
    }
    const int n = min(4, nb - c0);
    for (int bb = 0; bb < 4; ++bb) {
      const int vb = __shfl_sync(0xffffffffu, v, bb * 8 + k);
      const float db = __shfl_sync(0xffffffffu, d, bb * 8);
      int mb = 0;
      float dmb = 0.0f;
      if (MINS) {
        dmb = __shfl_sync(0xffffffffu, dmin, bb * 8);
        if (TYPE == T_Q4_K) {
          mb = __shfl_sync(0xffffffffu, m, bb * 8 + (k & 3));
        } else {
          const int m0 = __shfl_sync(0xffffffffu, m, bb * 8), m1 = __shfl_sync(0xffffffffu, m, bb * 8 + 1);
          const int m2 = __shfl_sync(0xffffffffu, m, bb * 8 + 2), m3 = __shfl_sync(0xffffffffu, m, bb * 8 + 3);
          mb = (m0 + m1) + (m2 + m3);
        }
      }
      if (bb < n) {
        acc = fmaf(db, (float)vb, acc);
        if (MINS) accm = fmaf(dmb, (float)mb, accm);
      }
    }
  }
  float a[8], am[4];
#pragma unroll
  for (int j = 0; j < 8; ++j) a[j] = __shfl_sync(0xffffffffu, acc, j);
#pragma unroll
  for (int j = 0; j < 4; ++j) am[j] = __shfl_sync(0xffffffffu, accm, j);
  if (lane == 0) {
    const float s0 = a[4] + a[0], s1 = a[5] + a[1], s2 = a[6] + a[2], s3 = a[7] + a[3];
    float r = (s0 + s2) + (s1 + s3);
    if (TYPE == T_Q4_K) r = r + ((am[0] + am[2]) + (am[1] + am[3]));
    if (TYPE == T_Q5_K) r = r + am[0];
    out[row] = r;
  }
}

// q8_0_gemv of the reference (quant_kernels.c:658-680), fp32 activations:
// lane k of the accumulator takes, per block and per 8-value chunk c in
// order, fma(d, q[8c + k] * x[8c + k], acc).  One warp per row; thread
// (c, k) forms the product of chunk c, the chain replays through shuffles.
__global__ void __launch_bounds__(256) q80_ref_gemv_kernel(const uint8_t* __restrict__ W,
                                                           const float* __restrict__ x, int nb, int rows,
                                                           float* __restrict__ out) {
  const int lane = threadIdx.x & 31, c = lane >> 3, k = lane & 7;
  const int row = blockIdx.x * 8 + (threadIdx.x >> 5);
  if (row >= rows) return;
  const uint8_t* wr = W + (size_t)row * nb * 34;
  float acc = 0.0f;
  for (int i = 0; i < nb; ++i) {
    const uint8_t* blk = wr + (size_t)i * 34;
    const float d = h2f_bits(q_ld16(blk));
    const float p = __fmul_rn((float)(int8_t)blk[2 + 8 * c + k], x[(size_t)i * 32 + 8 * c + k]);
#pragma unroll
    for (int cc = 0; cc < 4; ++cc) acc = fmaf(d, __shfl_sync(0xffffffffu, p, cc * 8 + k), acc);
  }
  float a[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) a[j] = __shfl_sync(0xffffffffu, acc, j);
  if (lane == 0) {
    const float s0 = a[4] + a[0], s1 = a[5] + a[1], s2 = a[6] + a[2], s3 = a[7] + a[3];
    out[row] = (s0 + s2) + (s1 + s3);
  }
}

}  // namespace

int launch_ref_gemv(int type, const void* W, const float* x, void* y8, int inner, int rows, float* out,
                    cudaStream_t st) {
  if (rows <= 0) return 0;
  const unsigned grid = (unsigned)((rows + 7) / 8);
  const uint8_t* w = (const uint8_t*)W;
  if (type == T_Q8_0) {
    q80_ref_gemv_kernel<<<grid, 256, 0, st>>>(w, x, inner / 32, rows, out);
  } else {
    int rc = launch_quantize_q8k(x, y8, inner / 256, st);
    if (rc) return rc;
    const uint8_t* y = (const uint8_t*)y8;
    switch (type) {
      case T_Q4_K: q8k_gemv_kernel<T_Q4_K><<<grid, 256, 0, st>>>(w, y, inner / 256, rows, out); break;
      case T_Q5_K: q8k_gemv_kernel<T_Q5_K><<<grid, 256, 0, st>>>(w, y, inner / 256, rows, out); break;
      case T_Q6_K: q8k_gemv_kernel<T_Q6_K><<<grid, 256, 0, st>>>(w, y, inner / 256, rows, out); break;
      default: return set_error(-1, "reference-numerics gemv: unsupported type %d", type);
    }
  }
  INF_CUDA_TRY(cudaGetLastError());
  return 0;
}

int launch_quantize_q8k(const float* x, void* y, long long nblocks, cudaStream_t st) {
  if (nblocks <= 0) return 0;
  if (nblocks > 0x7fffffffLL) return set_error(-1, "quantize_row_q8_K: %lld blocks", nblocks);
  q8k_quantize_kernel<<<(unsigned)nblocks, 256, 0, st>>>(x, (uint8_t*)y);
  INF_CUDA_TRY(cudaGetLastError());
  return 0;
}

int launch_vec_dot_q8k(int type, const void* x, const void* y, int nb, float* out, cudaStream_t st) {
  const uint8_t *xp = (const uint8_t*)x, *yp = (const uint8_t*)y;
  switch (type) {
    case T_Q4_K: q8k_vec_dot_kernel<T_Q4_K><<<1, 256, 0, st>>>(xp, yp, nb, out); break;
    case T_Q5_K: q8k_vec_dot_kernel<T_Q5_K><<<1, 256, 0, st>>>(xp, yp, nb, out); break;
    case T_Q6_K: q8k_vec_dot_kernel<T_Q6_K><<<1, 256, 0, st>>>(xp, yp, nb, out); break;
    case T_Q8_0: q8k_vec_dot_kernel<T_Q8_0><<<1, 256, 0, st>>>(xp, yp, nb, out); break;
    default: return set_error(-1, "vec_dot: unsupported type %d", type);
  }
  INF_CUDA_TRY(cudaGetLastError());
  return 0;
}

}  // namespace inf
