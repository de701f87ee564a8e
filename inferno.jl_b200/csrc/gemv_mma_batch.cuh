// Batched integer tensor-core GEMV: up to MMA_NBT input columns (the prompt
// tokens of one prefill chunk) against Q4_K / Q6_K rows.
//
// Same operator and fixed-point scheme as gemv_mma_kernel (one column), with
// the weight decode shared by the columns: each 16-row x 32-k A fragment is
// unpacked once and multiplied with the B fragment of every column, so the
// per-weight integer work is amortised over the tokens and the MMA count
// grows with them.  Each column keeps its own fixed-point scale (max|v| of
// that token), RMSNorm factor and sub-block sums.
//
// Activations are held compactly: per column and k step 128 bytes (limb l,
// k-half p, lane quad c -> word (2l + p) * 4 + c, i.e. lane * 4), and the zero
// half of the B fragment is made in registers.  The prologue runs one warp per
// column in two passes over the column's input (statistics, then limbs) so no
// fp32 staging array is needed.
#pragma once
#include "gemv_mma.cuh"

namespace inf {

constexpr int MMA_NBT = 8;            // columns per launch
constexpr int MMA_KSC_BYTES = 128;    // compact B bytes per k step and column
constexpr int MMA_MAX_HEADS = 64;     // PRO_HEADNORM_GATE heads per column (n / group)

__device__ __forceinline__ uint2 mma_bfrag(const uint8_t* xq_ks, int lane) {
  const uint32_t w = *(const uint32_t*)(xq_ks + lane * 4);
  return ((lane >> 2) & 1) ? make_uint2(0u, w) : make_uint2(w, 0u);
}

// Input value of element quad u (elements 4u..4u+3) of column v after the
// prologue fusion (RMSNorm weight, head norm + SiLU gate, or none).  `hsc`
// holds the column's per-head scales (head-norm only).
__device__ __forceinline__ float4 mma_batch_u(const GemvParams& p, int v, int u, const float* hsc) {
  const float* x = p.x + (long long)v * p.x_stride;
  float4 a = ((const float4*)x)[u];
  if (p.pro == PRO_RMSNORM) {
    const float4 w4 = ((const float4*)p.pro_w)[u];
    a.x *= w4.x; a.y *= w4.y; a.z *= w4.z; a.w *= w4.w;
  } else if (p.pro == PRO_HEADNORM_GATE) {
    const int G = p.pro_group, e0 = 4 * u, hh = e0 / G, i0 = e0 - hh * G;
    const float scale = hsc[hh];
    const float4 z4 = ((const float4*)(p.pro_z + (long long)v * p.x_stride))[u];
    const float4 w4 = *(const float4*)(p.pro_w + i0);
    const float vv[4] = {a.x, a.y, a.z, a.w}, zz[4] = {z4.x, z4.y, z4.z, z4.w}, ww[4] = {w4.x, w4.y, w4.z, w4.w};
    float o[4];
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      const float q = vv[t] * scale * ww[t];
      o[t] = q * zz[t] * (1.0f / (1.0f + expf(-zz[t])));
    }
    a = make_float4(o[0], o[1], o[2], o[3]);
  }
  return a;
}

// Warp `v` prepares column v: statistics pass (sum of squares / head norms,
// max|u|), then the limbs and sub-block sums.  cs[v] gets the column factor
// (1/rms or 1), vmax[v] max|u|; bad[v] flags a non-finite input.
template <int TYPE>
__device__ void gemv_mma_batch_prologue(const GemvParams& p, uint8_t* xq, float* xsum, float* cs, float* vmax,
                                        float* hsc_all, int* bad_all, int v, int lane) {
  const int n = p.inner, nf4 = n >> 2;
  const int nsb = n >> 8;
  float* hsc = hsc_all + v * MMA_MAX_HEADS;
  bool bad = false;
  float ss = 0.f, amax = 0.f;
  if (p.pro == PRO_HEADNORM_GATE) {
    const int G = p.pro_group, per = G >> 2;     // float4 items per head
    const float* x = p.x + (long long)v * p.x_stride;
    for (int hh = 0; hh < n / G; ++hh) {
      float hs = 0.f;
      for (int i = lane; i < per; i += 32) {
        const float4 a = ((const float4*)(x + hh * G))[i];
        hs = fmaf(a.x, a.x, fmaf(a.y, a.y, fmaf(a.z, a.z, fmaf(a.w, a.w, hs))));
      }
      hs = warp_sum(hs);
      if (lane == 0) hsc[hh] = 1.0f / sqrtf(hs / (float)G + p.eps);
    }
    __syncwarp();
  }
  for (int u = lane; u < nf4; u += 32) {
    const float4 a = mma_batch_u(p, v, u, hsc);
    if (p.pro == PRO_RMSNORM) {
      const float4 r = ((const float4*)(p.x + (long long)v * p.x_stride))[u];
      ss = fmaf(r.x, r.x, fmaf(r.y, r.y, fmaf(r.z, r.z, fmaf(r.w, r.w, ss))));
    }
    amax = fmaxf(amax, fmaxf(fmaxf(fabsf(a.x), fabsf(a.y)), fmaxf(fabsf(a.z), fabsf(a.w))));
  }
  ss = warp_sum(ss);
  amax = warp_max(amax);
  if (!(amax <= 3.0e38f)) bad = true;
  const float up = mma_pow2(mma_exp2_scale(amax));
  uint8_t* xqv = xq + (size_t)v * nsb * 8 * MMA_KSC_BYTES;
  float* xs = xsum + (size_t)v * nsb * 16;
  // nf4 is a multiple of 64 (n % 256 == 0): every lane runs every iteration
  for (int u = lane; u < nf4; u += 32) {
    const float4 a = mma_batch_u(p, v, u, hsc);
    const int e0 = 4 * u, sb = e0 >> 8, r = e0 & 255;
    int ks, cc, hp;
    if (TYPE == T_Q4_K) {
      ks = sb * 8 + 2 * (r >> 6) + ((r >> 2) & 1);
      cc = (r >> 3) & 3;
      hp = (r >> 5) & 1;
    } else {
      ks = sb * 8 + 4 * (r >> 7) + ((r >> 5) & 3);
      cc = (r >> 2) & 3;
      hp = (r >> 4) & 1;
    }
    const float vv[4] = {a.x, a.y, a.z, a.w};
    uint32_t limb[4] = {0u, 0u, 0u, 0u};
    float sum = 0.f;
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      if (vv[t] != vv[t]) bad = true;
      int xi = __float2int_rn(vv[t] * up);
      sum += (float)xi;
#pragma unroll
      for (int l = 0; l < 3; ++l) {
        const int d = (int)(int8_t)(xi & 0xff);
        limb[l] |= (uint32_t)(d & 0xff) << (8 * t);
        xi = (xi - d) >> 8;
      }
      limb[3] |= (uint32_t)(xi & 0xff) << (8 * t);
    }
#pragma unroll
    for (int l = 0; l < 4; ++l)
      *(uint32_t*)(xqv + (size_t)ks * MMA_KSC_BYTES + ((2 * l + hp) * 4 + cc) * 4) = limb[l];
    sum += __shfl_xor_sync(0xffffffffu, sum, 1);
    sum += __shfl_xor_sync(0xffffffffu, sum, 2);
    if (TYPE == T_Q4_K) sum += __shfl_xor_sync(0xffffffffu, sum, 4);
    if ((u & (TYPE == T_Q4_K ? 7 : 3)) == 0) xs[TYPE == T_Q4_K ? (e0 >> 5) : (e0 >> 4)] = sum;
  }
  bad = __any_sync(0xffffffffu, bad);
  if (lane == 0) {
    cs[v] = p.pro == PRO_RMSNORM ? 1.0f / sqrtf(ss / (float)n + p.eps) : 1.0f;
    vmax[v] = amax;
    bad_all[v] = bad ? 1 : 0;
  }
}

// Super-block bodies for MMA_NBT columns (rows g and g + 8 of the warp's 16).
// xq_sb / xs_sb point at column 0; columns are xq_col / xs_col apart.
__device__ __forceinline__ void mma_sb_q4k_batch(const uint8_t* ra, const uint8_t* rb, const uint8_t* xq_sb,
                                                 size_t xq_col, const float* xs_sb, int xs_col, int ncol, int lane,
                                                 float (&acc)[MMA_NBT][2], float (&corr)[MMA_NBT][2]) {
  const int c = lane & 3;
  const uint4 ha = *(const uint4*)ra, hb = *(const uint4*)rb;
  const uint32_t sla = ha.y & 0x3f3f3f3fu, sha = (ha.w & 0x0f0f0f0fu) | ((ha.y >> 2) & 0x30303030u);
  const uint32_t slb = hb.y & 0x3f3f3f3fu, shb = (hb.w & 0x0f0f0f0fu) | ((hb.y >> 2) & 0x30303030u);
  int S0[MMA_NBT], S1[MMA_NBT];
#pragma unroll
  for (int v = 0; v < MMA_NBT; ++v) S0[v] = S1[v] = 0;
#pragma unroll 1
  for (int j = 0; j < 4; ++j) {
    const uint2 qa = *(const uint2*)(ra + 16 + 32 * j + 8 * c);
    const uint2 qb = *(const uint2*)(rb + 16 + 32 * j + 8 * c);
    const uint32_t wsa = j < 2 ? sla : sha, wsb = j < 2 ? slb : shb;
    const int s0a = ubyte<0>(wsa >> (16 * (j & 1))), s1a = ubyte<1>(wsa >> (16 * (j & 1)));
    const int s0b = ubyte<0>(wsb >> (16 * (j & 1))), s1b = ubyte<1>(wsb >> (16 * (j & 1)));
#pragma unroll
    for (int wd = 0; wd < 2; ++wd) {
      const uint32_t wa = wd ? qa.y : qa.x, wb = wd ? qb.y : qb.x;
      const uint32_t a0 = wa & 0x0f0f0f0fu, a1 = wb & 0x0f0f0f0fu;
      const uint32_t a2 = (wa >> 4) & 0x0f0f0f0fu, a3 = (wb >> 4) & 0x0f0f0f0fu;
      const uint8_t* xk = xq_sb + (2 * j + wd) * MMA_KSC_BYTES;
#pragma unroll
      for (int v = 0; v < MMA_NBT; ++v) {
        if (v < ncol) {
          const uint2 bv = mma_bfrag(xk + v * xq_col, lane);
          int d[4];
          imma_k32(d, a0, a1, a2, a3, bv.x, bv.y);
          S0[v] += s0a * d[0] + s1a * d[1];
          S1[v] += s0b * d[2] + s1b * d[3];
        }
      }
    }
  }
  const float2 dda = __half22float2(*(const __half2*)&ha.x), ddb = __half22float2(*(const __half2*)&hb.x);
  const uint32_t mla = ha.z & 0x3f3f3f3fu, mha = ((ha.w >> 4) & 0x0f0f0f0fu) | ((ha.z >> 2) & 0x30303030u);
  const uint32_t mlb = hb.z & 0x3f3f3f3fu, mhb = ((hb.w >> 4) & 0x0f0f0f0fu) | ((hb.z >> 2) & 0x30303030u);
  const int sh = 16 * (c & 1);
  const uint32_t ma = (c < 2 ? mla : mha) >> sh, mb = (c < 2 ? mlb : mhb) >> sh;
  const float ma0 = (float)ubyte<0>(ma), ma1 = (float)ubyte<1>(ma);
  const float mb0 = (float)ubyte<0>(mb), mb1 = (float)ubyte<1>(mb);
#pragma unroll
  for (int v = 0; v < MMA_NBT; ++v) {
    if (v < ncol) {
      acc[v][0] = fmaf(dda.x, (float)S0[v], acc[v][0]);
      acc[v][1] = fmaf(ddb.x, (float)S1[v], acc[v][1]);
      const float2 X = *(const float2*)(xs_sb + v * xs_col + 2 * c);
      corr[v][0] = fmaf(dda.y, ma0 * X.x + ma1 * X.y, corr[v][0]);
      corr[v][1] = fmaf(ddb.y, mb0 * X.x + mb1 * X.y, corr[v][1]);
    }
  }
}

__device__ __forceinline__ void mma_sb_q6k_batch(const uint8_t* ra, const uint8_t* rb, const uint8_t* xq_sb,
                                                 size_t xq_col, const float* xs_sb, int xs_col, int ncol, int lane,
                                                 float (&acc)[MMA_NBT][2], float (&corr)[MMA_NBT][2]) {
  const int c = lane & 3;
  int S0[MMA_NBT], S1[MMA_NBT];
#pragma unroll
  for (int v = 0; v < MMA_NBT; ++v) S0[v] = S1[v] = 0;
  uint32_t sca[4], scb[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    sca[i] = lds_u32_any(ra + 192 + 4 * i);
    scb[i] = lds_u32_any(rb + 192 + 4 * i);
  }
#pragma unroll 1
  for (int n6 = 0; n6 < 2; ++n6) {
    const uint32_t ha0 = lds_u32_any(ra + 128 + 32 * n6 + 4 * c);
    const uint32_t ha1 = lds_u32_any(ra + 128 + 32 * n6 + 16 + 4 * c);
    const uint32_t hb0 = lds_u32_any(rb + 128 + 32 * n6 + 4 * c);
    const uint32_t hb1 = lds_u32_any(rb + 128 + 32 * n6 + 16 + 4 * c);
#pragma unroll
    for (int kk = 0; kk < 2; ++kk) {
      const uint32_t la0 = lds_u32_any(ra + 64 * n6 + 32 * kk + 4 * c);
      const uint32_t la1 = lds_u32_any(ra + 64 * n6 + 32 * kk + 16 + 4 * c);
      const uint32_t lb0 = lds_u32_any(rb + 64 * n6 + 32 * kk + 4 * c);
      const uint32_t lb1 = lds_u32_any(rb + 64 * n6 + 32 * kk + 16 + 4 * c);
#pragma unroll
      for (int hi = 0; hi < 2; ++hi) {
        const int k = kk + 2 * hi;
        const int sh = 4 * hi;
        const uint32_t ua0 = ((la0 >> sh) & 0x0f0f0f0fu) | qh_bits(ha0, k);
        const uint32_t ua1 = ((la1 >> sh) & 0x0f0f0f0fu) | qh_bits(ha1, k);
        const uint32_t ub0 = ((lb0 >> sh) & 0x0f0f0f0fu) | qh_bits(hb0, k);
        const uint32_t ub1 = ((lb1 >> sh) & 0x0f0f0f0fu) | qh_bits(hb1, k);
        const int is = 8 * n6 + 2 * k;
        const int s0a = sbyte<0>(sca[is >> 2] >> (8 * (is & 3))), s1a = sbyte<0>(sca[is >> 2] >> (8 * (is & 3) + 8));
        const int s0b = sbyte<0>(scb[is >> 2] >> (8 * (is & 3))), s1b = sbyte<0>(scb[is >> 2] >> (8 * (is & 3) + 8));
        const uint8_t* xk = xq_sb + (4 * n6 + k) * MMA_KSC_BYTES;
#pragma unroll
        for (int v = 0; v < MMA_NBT; ++v) {
          if (v < ncol) {
            const uint2 bv = mma_bfrag(xk + v * xq_col, lane);
            int d[4];
            imma_k32(d, ua0, ub0, ua1, ub1, bv.x, bv.y);
            S0[v] += s0a * d[0] + s1a * d[1];
            S1[v] += s0b * d[2] + s1b * d[3];
          }
        }
      }
    }
  }
  const float da = h2f_bits(lds_u16_any(ra + 208)), db = h2f_bits(lds_u16_any(rb + 208));
  const uint32_t wa = c == 0 ? sca[0] : c == 1 ? sca[1] : c == 2 ? sca[2] : sca[3];
  const uint32_t wb = c == 0 ? scb[0] : c == 1 ? scb[1] : c == 2 ? scb[2] : scb[3];
#pragma unroll
  for (int v = 0; v < MMA_NBT; ++v) {
    if (v < ncol) {
      acc[v][0] = fmaf(da, (float)S0[v], acc[v][0]);
      acc[v][1] = fmaf(db, (float)S1[v], acc[v][1]);
      const float4 X = *(const float4*)(xs_sb + v * xs_col + 4 * c);
      const float ta = (float)sbyte<0>(wa) * X.x + (float)sbyte<1>(wa) * X.y + (float)sbyte<2>(wa) * X.z +
                       (float)sbyte<3>(wa) * X.w;
      const float tb = (float)sbyte<0>(wb) * X.x + (float)sbyte<1>(wb) * X.y + (float)sbyte<2>(wb) * X.z +
                       (float)sbyte<3>(wb) * X.w;
      corr[v][0] = fmaf(32.0f * da, ta, corr[v][0]);
      corr[v][1] = fmaf(32.0f * db, tb, corr[v][1]);
    }
  }
}

// Smem layout: [full][empty][cs 8][vmax 8][bad 8][hsc 8 x 64][kpart NBT x NW x 16][xsum][xq][stages]
template <int NW>
__host__ __device__ constexpr size_t mma_batch_fixed_bytes() {
  return 16 * GEMV_MAX_STAGES + 3 * MMA_NBT * 4 + MMA_NBT * MMA_MAX_HEADS * 4 + (size_t)MMA_NBT * NW * 16 * 4;
}

template <int TYPE, int NW>
__global__ void __launch_bounds__((NW + 1) * 32, 1) gemv_mma_batch_kernel(const __grid_constant__ GemvParams p) {
  static_assert(NW == MMA_NBT, "one prologue warp per column");
  extern __shared__ __align__(128) uint8_t smem[];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  constexpr int BB = TYPE == T_Q4_K ? 144 : 210;
  constexpr int XS_PER_SB = TYPE == T_Q4_K ? 8 : 16;
  uint64_t* full = (uint64_t*)smem;
  uint64_t* empty = full + GEMV_MAX_STAGES;
  float* cs = (float*)(empty + GEMV_MAX_STAGES);
  float* vmax = cs + MMA_NBT;
  int* bad = (int*)(vmax + MMA_NBT);
  float* hsc = (float*)(bad + MMA_NBT);
  float* kpart = hsc + MMA_NBT * MMA_MAX_HEADS;
  float* xsum = kpart + MMA_NBT * NW * 16;
  const int nsb = p.inner >> 8;
  uint8_t* xq = (uint8_t*)(xsum + (size_t)MMA_NBT * nsb * 16);
  const size_t xq_col = (size_t)nsb * 8 * MMA_KSC_BYTES;
  uint8_t* stage0 = (uint8_t*)(((uintptr_t)(xq + MMA_NBT * xq_col) + 127) & ~(uintptr_t)127);
  const int ncol = p.nb;

  if (tid == 0) {
    for (int s = 0; s < p.stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], NW);
    }
    fence_mbar_init();
  }
  __syncthreads();
  const int G = gridDim.x;
  const int n_items = (p.ntiles - (int)blockIdx.x + G - 1) / G;
  if (warp == NW) {
    gemv_producer<false>(p, full, empty, stage0, lane, n_items);
    return;
  }

  pdl_wait();
  if (warp < ncol) gemv_mma_batch_prologue<TYPE>(p, xq, xsum, cs, vmax, hsc, bad, warp, lane);
  named_bar_sync(1, NW * 32);
  float fscale[MMA_NBT];
#pragma unroll
  for (int v = 0; v < MMA_NBT; ++v)
    fscale[v] = v < ncol ? (bad[v] ? __int_as_float(0x7fc00000) : cs[v] * mma_pow2(-mma_exp2_scale(vmax[v])))
                         : 0.f;

  const bool paired = (p.epi == EPI_SWIGLU);
  const int nrg = p.TR >> 4;
  const int nkg = NW / nrg;
  const int rg = warp % nrg, wk = warp / nrg;
  const int g = lane >> 2, c = lane & 3;
  const float limbw = c == 0 ? 1.0f : c == 1 ? 256.0f : c == 2 ? 65536.0f : 16777216.0f;

  for (int it = 0; it < n_items; ++it) {
    const int s = it % p.stages;
    if (!mbar_wait(&full[s], (it / p.stages) & 1, p.err)) return;
    int sg, row0;
    tile_locate(p, blockIdx.x + it * G, sg, row0);
    const uint8_t* st = stage0 + (long long)s * p.stage_bytes;
    const uint8_t *ra, *rb;
    if (paired) {
      const uint32_t m0 = (uint32_t)((uintptr_t)seg_row_ptr<false>(p, 0, row0) & 15);
      const uint32_t m1 = (uint32_t)((uintptr_t)seg_row_ptr<false>(p, 1, row0) & 15);
      ra = st + m0 + (long long)(rg * 8 + g) * p.row_bytes;
      rb = st + p.part1_off + m1 + (long long)(rg * 8 + g) * p.row_bytes;
    } else {
      const uint32_t m0 = (uint32_t)((uintptr_t)seg_row_ptr<false>(p, sg, row0) & 15);
      ra = st + m0 + (long long)(rg * 16 + g) * p.row_bytes;
      rb = ra + 8ll * p.row_bytes;
    }
    float acc[MMA_NBT][2], corr[MMA_NBT][2];
#pragma unroll
    for (int v = 0; v < MMA_NBT; ++v) acc[v][0] = acc[v][1] = corr[v][0] = corr[v][1] = 0.f;
    for (int sb = wk; sb < nsb; sb += nkg) {
      if constexpr (TYPE == T_Q4_K)
        mma_sb_q4k_batch(ra + sb * BB, rb + sb * BB, xq + (size_t)sb * 8 * MMA_KSC_BYTES, xq_col,
                         xsum + sb * XS_PER_SB, nsb * 16, ncol, lane, acc, corr);
      else
        mma_sb_q6k_batch(ra + sb * BB, rb + sb * BB, xq + (size_t)sb * 8 * MMA_KSC_BYTES, xq_col,
                         xsum + sb * XS_PER_SB, nsb * 16, ncol, lane, acc, corr);
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);

    float ta[MMA_NBT], tb[MMA_NBT];
#pragma unroll
    for (int v = 0; v < MMA_NBT; ++v) {
      ta[v] = limbw * acc[v][0] - corr[v][0];
      tb[v] = limbw * acc[v][1] - corr[v][1];
      ta[v] += __shfl_xor_sync(0xffffffffu, ta[v], 1);
      tb[v] += __shfl_xor_sync(0xffffffffu, tb[v], 1);
      ta[v] += __shfl_xor_sync(0xffffffffu, ta[v], 2);
      tb[v] += __shfl_xor_sync(0xffffffffu, tb[v], 2);
    }
    if (nkg > 1) {
      if (wk > 0 && c == 0) {
#pragma unroll
        for (int v = 0; v < MMA_NBT; ++v) {
          kpart[(v * NW + wk * nrg + rg) * 16 + g] = ta[v];
          kpart[(v * NW + wk * nrg + rg) * 16 + g + 8] = tb[v];
        }
      }
      named_bar_sync(2, NW * 32);
      if (wk == 0 && c == 0)
        for (int k = 1; k < nkg; ++k) {
#pragma unroll
          for (int v = 0; v < MMA_NBT; ++v) {
            ta[v] += kpart[(v * NW + k * nrg + rg) * 16 + g];
            tb[v] += kpart[(v * NW + k * nrg + rg) * 16 + g + 8];
          }
        }
      named_bar_sync(2, NW * 32);
    }
    if (wk != 0 || c != 0) continue;
#pragma unroll
    for (int v = 0; v < MMA_NBT; ++v) {
      if (v >= ncol) break;
      const float a = ta[v] * fscale[v], b = tb[v] * fscale[v];
      if (paired) {
        const int row = row0 + rg * 8 + g;
        if (row < p.seg[0].rows) {
          const float sg_ = a / (1.0f + expf(-a));      // mlp_forward (src/ModelCPU.jl:455-468)
          p.seg[0].y[(long long)v * p.y_stride + row] = sg_ * b;
        }
      } else {
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int row = row0 + rg * 16 + g + 8 * h;
          if (row < p.seg[sg].rows && p.seg[sg].y) {
            float* y = p.seg[sg].y + (long long)v * p.y_stride + row;
            const float t = h ? b : a;
            if (p.epi == EPI_ADD) *y += t;
            else *y = t;
          }
        }
      }
    }
  }
}

}  // namespace inf
