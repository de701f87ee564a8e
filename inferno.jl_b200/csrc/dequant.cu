#include <algorithm>
// Bit-exact dequantization of GGUF super-blocks to fp32.
//
// Follows Inferno.jl src/Dequant.jl:12-54 (IQ2_XXS), :304-321 (Q8_0),
// :325-375 (Q4_K), :379-441 (Q5_K), :558-601 (Q6_K) operation by operation;
// every multiply / subtract is an explicitly rounded __fmul_rn / __fsub_rn so
// nvcc cannot contract them into an FMA (Julia does not fuse a*b-c either).
// One thread produces one 32-element run; loads are byte loads because the
// 210/66/34-byte blocks are not word aligned (this kernel is load-time only).
#include "internal.h"
#include "gemv.cuh"

namespace inf {

__device__ __forceinline__ uint16_t ld16(const uint8_t* p) { return (uint16_t)(p[0] | (p[1] << 8)); }
__device__ __forceinline__ uint32_t ld32(const uint8_t* p) {
  return (uint32_t)p[0] | ((uint32_t)p[1] << 8) | ((uint32_t)p[2] << 16) | ((uint32_t)p[3] << 24);
}

__device__ __forceinline__ void kscale_b(const uint8_t* sc, int is, uint32_t& s, uint32_t& m) {
  if (is < 4) {
    s = sc[is] & 63u;
    m = sc[is + 4] & 63u;
  } else {
    s = (sc[is + 4] & 0x0fu) | ((sc[is - 4] >> 6) << 4);
    m = (sc[is + 4] >> 4) | ((sc[is] >> 6) << 4);
  }
}

template <int TYPE>
__global__ void dequant_kernel(const uint8_t* __restrict__ src, float* __restrict__ dst, long long nruns) {
  long long r = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= nruns) return;
  float* o = dst + r * 32;
  if (TYPE == T_Q8_0) {
    const uint8_t* b = src + r * 34;
    float d = h2f_bits(ld16(b));
    for (int j = 0; j < 32; ++j) o[j] = __fmul_rn(d, (float)(int8_t)b[2 + j]);
  } else if (TYPE == T_Q4_K || TYPE == T_Q5_K) {
    // run r: block r>>3, q = r&7 -> sub-block pair j = q>>1, lo/hi = q&1
    long long blk = r >> 3;
    int q = (int)(r & 7), j = q >> 1, hi = q & 1;
    const uint8_t* b = src + blk * (TYPE == T_Q4_K ? 144 : 176);
    float d = h2f_bits(ld16(b)), dmin = h2f_bits(ld16(b + 2));
    uint32_t s, m;
    kscale_b(b + 4, 2 * j + hi, s, m);
    float d1 = __fmul_rn(d, (float)s), mn = __fmul_rn(dmin, (float)m);
    o = dst + blk * 256 + j * 64 + hi * 32;
    const uint8_t* qs = b + (TYPE == T_Q4_K ? 16 : 48) + j * 32;
    for (int l = 0; l < 32; ++l) {
      uint32_t v = hi ? (qs[l] >> 4) : (qs[l] & 0x0fu);
      if (TYPE == T_Q5_K) {
        uint32_t u = 1u << (2 * j + hi);
        v += (b[16 + l] & u) ? 16u : 0u;
      }
      o[l] = __fsub_rn(__fmul_rn(d1, (float)v), mn);
    }
  } else if (TYPE == T_Q6_K) {
    // run r: block r>>3, q = r&7 -> half n = q>>2, group k = q&3 (q1..q4)
    long long blk = r >> 3;
    int q = (int)(r & 7), n = q >> 2, k = q & 3;
    const uint8_t* b = src + blk * 210;
    const uint8_t* ql = b + n * 64;
    const uint8_t* qh = b + 128 + n * 32;
    const int8_t* sc = (const int8_t*)(b + 192 + n * 8);
    float d = h2f_bits(ld16(b + 208));
    o = dst + blk * 256 + n * 128 + k * 32;
    for (int l = 0; l < 32; ++l) {
      uint32_t lo = (k & 1) ? ql[l + 32] : ql[l];
      uint32_t nib = (k >= 2) ? (lo >> 4) : (lo & 0x0fu);
      int qv = (int)(nib | (((qh[l] >> (2 * k)) & 3u) << 4)) - 32;
      int is = l / 16;
      o[l] = __fmul_rn(__fmul_rn(d, (float)sc[is + 2 * k]), (float)qv);
    }
  } else if (TYPE == T_IQ2_XXS) {
    long long blk = r >> 3;
    int ib = (int)(r & 7);
    const uint8_t* b = src + blk * 66;
    float d = h2f_bits(ld16(b));
    uint32_t a1 = ld32(b + 2 + ib * 8), a2 = ld32(b + 6 + ib * 8);
    float db = __fmul_rn(__fmul_rn(d, __fadd_rn(0.5f, (float)(a2 >> 28))), 0.25f);
    for (int l = 0; l < 4; ++l) {
      uint64_t g = c_iq2xxs_grid_init[(a1 >> (8 * l)) & 0xffu];
      uint32_t sg = (a2 >> (7 * l)) & 127u;
      sg |= (uint32_t)(__popc(sg) & 1) << 7;
      for (int jj = 0; jj < 8; ++jj) {
        int v = (int)((g >> (8 * jj)) & 0xffu) - 8;
        float sgn = ((sg >> jj) & 1u) ? -1.0f : 1.0f;
        o[l * 8 + jj] = __fmul_rn(__fmul_rn(db, (float)v), sgn);
      }
    }
  } else if (TYPE == T_F32) {
    const float* s = (const float*)src + r * 32;
    for (int j = 0; j < 32; ++j) o[j] = s[j];
  }
}

int launch_dequant(int type, const void* src, long long n, float* dst, cudaStream_t st) {
  if (n % 32) return -1;
  long long runs = n / 32;
  if (runs == 0) return 0;
  int threads = 256;
  unsigned blocks = (unsigned)((runs + threads - 1) / threads);
  const uint8_t* s = (const uint8_t*)src;
  switch (type) {
    case T_Q8_0: dequant_kernel<T_Q8_0><<<blocks, threads, 0, st>>>(s, dst, runs); break;
    case T_Q4_K: dequant_kernel<T_Q4_K><<<blocks, threads, 0, st>>>(s, dst, runs); break;
    case T_Q5_K: dequant_kernel<T_Q5_K><<<blocks, threads, 0, st>>>(s, dst, runs); break;
    case T_Q6_K: dequant_kernel<T_Q6_K><<<blocks, threads, 0, st>>>(s, dst, runs); break;
    case T_IQ2_XXS: dequant_kernel<T_IQ2_XXS><<<blocks, threads, 0, st>>>(s, dst, runs); break;
    case T_F32: dequant_kernel<T_F32><<<blocks, threads, 0, st>>>(s, dst, runs); break;
    default: return -2;
  }
  return cudaGetLastError() == cudaSuccess ? 0 : -3;
}

// Dequantize row row_ptr[b] of a (rows x inner) matrix into dst[b][inner],
// one CTA per b (token-embedding lookup: src/ModelCPU.jl:973-976).  The rows
// are read from device memory so the launch can sit inside a captured graph.
template <int TYPE>
__global__ void embed_row_kernel(const uint8_t* __restrict__ W, long long row_bytes, int inner,
                                 const int* __restrict__ row_ptr, float* __restrict__ dst, int vocab) {
  pdl_wait();
  pdl_trigger();
  int row = row_ptr[blockIdx.x];
  if (row < 0 || row >= vocab) row = 0;
  dst += (long long)blockIdx.x * inner;
  // eight threads per 32-value run, four values each (the same arithmetic
  // per value as dequant_kernel)
  const int runs = inner / 32;
  const uint8_t* src = W + (long long)row * row_bytes;
  for (int item = threadIdx.x; item < runs * 8; item += blockDim.x) {
  const int r = item >> 3, l0 = (item & 7) * 4;
  if (TYPE == T_Q6_K) {
    const int blk = r >> 3, q = r & 7, n = q >> 2, k = q & 3;
    const uint8_t* b = src + (long long)blk * 210;
    const uint8_t* ql = b + n * 64;
    const uint8_t* qh = b + 128 + n * 32;
    const int8_t* sc = (const int8_t*)(b + 192 + n * 8);
    const float d = h2f_bits(ld16(b + 208));
    float* o = dst + (long long)blk * 256 + n * 128 + k * 32;
#pragma unroll
    for (int l = l0; l < l0 + 4; ++l) {
      const uint32_t lo = (k & 1) ? ql[l + 32] : ql[l];
      const uint32_t nib = (k >= 2) ? (lo >> 4) : (lo & 0x0fu);
      const int qv = (int)(nib | (((qh[l] >> (2 * k)) & 3u) << 4)) - 32;
      o[l] = __fmul_rn(__fmul_rn(d, (float)sc[l / 16 + 2 * k]), (float)qv);
    }
  } else if (TYPE == T_Q8_0) {
    const uint8_t* b = src + (long long)r * 34;
    const float d = h2f_bits(ld16(b));
#pragma unroll
    for (int jj = l0; jj < l0 + 4; ++jj) dst[r * 32 + jj] = __fmul_rn(d, (float)(int8_t)b[2 + jj]);
  } else if (TYPE == T_Q4_K || TYPE == T_Q5_K) {
    const int blk = r >> 3, q = r & 7, j = q >> 1, hi = q & 1;
    const uint8_t* b = src + (long long)blk * (TYPE == T_Q4_K ? 144 : 176);
    const float d = h2f_bits(ld16(b)), dmin = h2f_bits(ld16(b + 2));
    uint32_t sv, m;
    kscale_b(b + 4, 2 * j + hi, sv, m);
    const float d1 = __fmul_rn(d, (float)sv), mn = __fmul_rn(dmin, (float)m);
    float* o = dst + (long long)blk * 256 + j * 64 + hi * 32;
    const uint8_t* qs = b + (TYPE == T_Q4_K ? 16 : 48) + j * 32;
#pragma unroll
    for (int l = l0; l < l0 + 4; ++l) {
      uint32_t v = hi ? (qs[l] >> 4) : (qs[l] & 0x0fu);
      if (TYPE == T_Q5_K) v += (b[16 + l] & (1u << (2 * j + hi))) ? 16u : 0u;
      o[l] = __fsub_rn(__fmul_rn(d1, (float)v), mn);
    }
  } else if (TYPE == T_F32) {
    const float* sp = (const float*)src;
#pragma unroll
    for (int jj = l0; jj < l0 + 4; ++jj) dst[r * 32 + jj] = sp[r * 32 + jj];
  }
  }
}

int launch_embed_row(int type, const void* W, long long row_bytes, int inner, const int* row_ptr, float* dst,
                     int vocab, cudaStream_t st, bool pdl, int nrows) {
  if (inner % 256 || nrows < 1) return -1;
  const int threads = std::min(1024, inner / 32 * 8);     // 8 threads per 32-value run
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(nrows);
  cfg.blockDim = dim3(threads);
  cfg.stream = st;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = pdl ? 1 : 0;
  const uint8_t* w = (const uint8_t*)W;
  cudaError_t e;
  switch (type) {
    case T_Q6_K: e = cudaLaunchKernelEx(&cfg, embed_row_kernel<T_Q6_K>, w, row_bytes, inner, row_ptr, dst, vocab); break;
    case T_Q4_K: e = cudaLaunchKernelEx(&cfg, embed_row_kernel<T_Q4_K>, w, row_bytes, inner, row_ptr, dst, vocab); break;
    case T_Q5_K: e = cudaLaunchKernelEx(&cfg, embed_row_kernel<T_Q5_K>, w, row_bytes, inner, row_ptr, dst, vocab); break;
    case T_Q8_0: e = cudaLaunchKernelEx(&cfg, embed_row_kernel<T_Q8_0>, w, row_bytes, inner, row_ptr, dst, vocab); break;
    case T_F32: e = cudaLaunchKernelEx(&cfg, embed_row_kernel<T_F32>, w, row_bytes, inner, row_ptr, dst, vocab); break;
    default: return -2;
  }
  return e == cudaSuccess ? 0 : -3;
}

}  // namespace inf
