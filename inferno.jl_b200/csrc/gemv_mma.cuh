// Integer tensor-core GEMV for Q4_K and Q6_K rows (single column).
//
// Same operator as gemv_kernel (ModelCPU.mul! / mul_quant_mat_vec, Inferno.jl
// src/ModelCPU.jl:284-444; dequant formulas of src/Dequant.jl:345-362 and
// :585-596), restructured so that the per-weight work is a few integer
// instructions instead of an int->float conversion plus an FMA:
//
//  * The activation vector v (after the fused prologue) is written as an
//    exact fixed-point integer  x'_i = rint(v_i * 2^s)  with |x'| < 2^30
//    (s from max|v|), split into four balanced int8 "limbs"
//      x' = t0 + 2^8 t1 + 2^16 t2 + 2^24 t3,   t_l in [-128, 127].
//    The representation error is 2^-31 of max|v| per element, below fp32
//    rounding of the reference's own dot products.
//  * Weight codes (4-bit Q4_K nibbles, 6-bit Q6_K values) are the A operand
//    of mma.sync.m16n8k32 u8 x s8 -> s32 as they sit in shared memory (one
//    mask / shift per four codes); the limbs are the B operand.  A warp
//    multiplies 16 rows by one 32-wide k step per instruction; the 8 B
//    columns are (limb l, half p): column 2l+p holds limb l of the 16
//    elements of k-half p and zeros in the other half, so each column's
//    integer result belongs to one sub-block and takes that sub-block's
//    integer scale with one IMAD.  All integer sums are exact (bounded by
//    256 * 63 * 128 * 128 < 2^31 per super-block and row).
//  * Per super-block and row:  acc += d * float(sum_j sc_j * D_j), and the
//    offset terms (Q4_K: dmin * sum_j m_j X_j; Q6_K: 32 d sum_j sc_j X_j,
//    X_j = sum of x' over sub-block j) are accumulated separately in fp32.
//  * The row total is  2^-s * sum_l 2^{8l} acc_l  (lane c of a quad owns limb
//    c), times the RMSNorm 1/rms column factor.
//
// Tiles, the TMA ring, the producer warp, prologue fusions and epilogues are
// those of gemv_kernel.  A warp owns 16 rows (SwiGLU: 8 gate rows as MMA rows
// 0-7 and the matching 8 up rows as rows 8-15) and a K group of super-blocks.
#pragma once
#include "gemv.cuh"

namespace inf {

constexpr int MMA_KS_BYTES = 256;     // B bytes per k step (8 columns x 32 k)
// Kernel variants: the per-token GEMVs run MMA_PLAIN, whose code holds none
// of the MoE (expert-indirect rows, several input vectors) or tensor-parallel
// exchange paths -- every launch fetches its instructions cold, and unused
// branches inlined into the hot path cost measurable time per launch.
// The plain per-token GEMVs are split further by what they run: MMA_PLAIN
// (register prologue, one row per tile row: store / add / argmax),
// MMA_SWIGLU (register prologue, gate and up rows paired), MMA_GATE (the
// general prologue, e.g. head-norm x SiLU(z) of the ssm_out input).
enum MmaMode : int { MMA_PLAIN = 0, MMA_MOE = 1, MMA_XCH = 2, MMA_GATE = 3, MMA_SWIGLU = 4 };
// The super-block bodies' outer loops are not unrolled: the per-layer GEMVs
// are latency-bound and every launch fetches its code cold, so code size
// matters more than loop overhead.

__device__ __forceinline__ void imma_k32(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%10,%10,%10,%10};"
      : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(0));
}

template <int K>
__device__ __forceinline__ int sbyte(uint32_t w) {   // signed byte K of w
  return (int)(w << (24 - 8 * K)) >> 24;
}
// bits 2K, 2K+1 of each byte of a Q6_K qh word, moved to bits 4, 5
// (k is a constant after unrolling)
__device__ __forceinline__ uint32_t qh_bits(uint32_t h, int k) {
  return (k < 2 ? (h << (4 - 2 * k)) : (h >> (2 * k - 4))) & 0x30303030u;
}
template <int K>
__device__ __forceinline__ int ubyte(uint32_t w) {   // unsigned byte K of w
  return (int)((w >> (8 * K)) & 0xffu);
}

__device__ __forceinline__ unsigned long long ld_relaxed_sys_u64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_relaxed_sys_u64(unsigned long long* p, unsigned long long v) {
  asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

// Element (within the vector) of k-half p, position t of the quad (ks, cc),
// and the sub-block sum slot it belongs to.
template <int TYPE>
__device__ __forceinline__ int mma_elem(int ks, int cc, int p) {
  const int sb = ks >> 3, r = ks & 7;
  if constexpr (TYPE == T_Q4_K) return sb * 256 + (r >> 1) * 64 + 32 * p + 8 * cc + 4 * (r & 1);
  else return sb * 256 + (r >> 2) * 128 + (r & 3) * 32 + 16 * p + 4 * cc;
}
template <int TYPE>
__device__ __forceinline__ int mma_xsum_slot(int ks, int p) {
  const int sb = ks >> 3, r = ks & 7;
  if constexpr (TYPE == T_Q4_K) return sb * 8 + (r >> 1) * 2 + p;          // 32-element sub-blocks
  else return sb * 16 + (r >> 2) * 8 + (r & 3) * 2 + p;                     // 16-element sub-blocks
}

// Prologue: v (RMSNorm x*w, head-norm gate, or x) into xf, then the limbs
// into xq ([vector][ks][8 columns][4 lanes][8 bytes]) and sub-block sums into
// xsum.  vmax[v] receives max|v| of each input vector (its fixed-point scale
// is derived from it), red[0..NW) the RMSNorm partial sums; returns the column
// factor (1/rms or 1).  A non-finite input sets the flag red[2*NW] and makes
// every output NaN (as the reference's fp32 arithmetic would).
// vmax[] and the flag must be zero on entry.
__device__ __forceinline__ int mma_exp2_scale(float vmax) {
  int e = 0;
  if (vmax > 0.f && vmax <= 3.0e38f) {
    // frexp exponent (vmax < 2^e): from the IEEE exponent field for normal
    // numbers, the library routine for subnormals
    const int be = (__float_as_int(vmax) >> 23) & 0xff;
    if (be > 0) e = be - 126;
    else frexpf(vmax, &e);
  }
  return max(-120, min(120, 30 - e));
}
// 2^k for |k| <= 120 (a normal float), built from its exponent field
__device__ __forceinline__ float mma_pow2(int k) { return __int_as_float((k + 127) << 23); }

template <int TYPE, int NW, int MODE>
__device__ float gemv_mma_prologue(const GemvParams& p, float* xf, uint8_t* xq, float* xsum, float* red,
                                   float* vmax, int tid) {
  const int n = p.inner;
  const int lane = tid & 31, w = tid >> 5;
  constexpr int NT = NW * 32;
  const int nxv = p.nxv;
  const float* x = p.x;
  float ss = 0.f, amax = 0.f;
  bool bad = false;
  if (MODE == MMA_XCH && p.pro == PRO_RMSNORM && p.xch_rk >= 0) {
    // residual stream = x + the ranks' partials of sync point xch_rk, summed
    // in rank order (bit-identical on every rank); CTA 0 stores it for later
    // kernels.  Every word is polled until its tag is this sync's (bounded).
    const uint32_t tag = (uint32_t)(*p.xch_seq + (unsigned long long)p.xch_rk + 1ull);
    const unsigned long long* parts = p.xch_parts[p.xch_rank] + (size_t)(p.xch_rk & 1) * p.xch_n * n;
    constexpr int PER = 8192 / NT;          // hidden <= 8192
    float v[PER];
#pragma unroll
    for (int j = 0; j < PER; ++j) {
      const int i = tid + j * NT;
      v[j] = i < n ? __ldcg(x + i) : 0.f;
    }
    for (int r = 0; r < p.xch_n; ++r) {
      unsigned long long w[PER];
#pragma unroll
      for (int j = 0; j < PER; ++j) {
        const int i = tid + j * NT;
        w[j] = i < n ? ld_relaxed_sys_u64(parts + (size_t)r * n + i) : ((unsigned long long)tag << 32);
      }
#pragma unroll
      for (int j = 0; j < PER; ++j) {
        const int i = tid + j * NT;
        unsigned it = 0;
        // after one word timed out the others are not waited for
        while (!bad && (uint32_t)(w[j] >> 32) != tag) {
          if (++it > p.xch_spin) {
            if (p.err) atomicExch(p.err, DERR_MBAR_TIMEOUT);
            bad = true;
            break;
          }
          if (it > 1024) __nanosleep(32);
          w[j] = ld_relaxed_sys_u64(parts + (size_t)r * n + i);
        }
        v[j] += __uint_as_float((uint32_t)w[j]);
      }
    }
#pragma unroll
    for (int j = 0; j < PER; ++j) {
      const int i = tid + j * NT;
      if (i < n) {
        if (blockIdx.x == 0) p.x_next[i] = v[j];
        ss = fmaf(v[j], v[j], ss);
        const float u = v[j] * p.pro_w[i];
        amax = fmaxf(amax, fabsf(u));
        xf[i] = u;
      }
    }
  } else if (p.pro == PRO_RMSNORM) {
    for (int i = tid; i < n; i += NT) {
      const float v = x[i];
      ss = fmaf(v, v, ss);
      const float u = v * p.pro_w[i];
      amax = fmaxf(amax, fabsf(u));
      xf[i] = u;
    }
  } else if (p.pro == PRO_HEADNORM_GATE) {
    const int G = p.pro_group;
    const int per = G >> 5;
#pragma unroll
    for (int hh = w; hh < n / G; hh += NW) {
      float yv[8], zv[8], wv[8];
      float hs = 0.f;
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        const bool ok = q < per;
        const int i = hh * G + q * 32 + lane;
        yv[q] = ok ? x[i] : 0.f;
        zv[q] = ok ? p.pro_z[i] : 0.f;
        wv[q] = ok ? p.pro_w[q * 32 + lane] : 0.f;
      }
#pragma unroll
      for (int q = 0; q < 8; ++q) hs = fmaf(yv[q], yv[q], hs);
      hs = warp_sum(hs);
      const float scale = 1.0f / sqrtf(hs / (float)G + p.eps);
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        if (q >= per) break;
        const float v = yv[q] * scale * wv[q];
        const float u = v * zv[q] * (1.0f / (1.0f + expf(-zv[q])));
        amax = fmaxf(amax, fabsf(u));
        xf[hh * G + q * 32 + lane] = u;
      }
    }
  } else if (MODE == MMA_MOE && nxv > 1) {
    // several vectors (n % 32 == 0): a warp's 32 elements share one vector
    for (int i = tid; i < nxv * n; i += NT) {
      const int v = i / n;
      const float u = x[(long long)v * p.x_stride + (i - v * n)];
      xf[i] = u;
      const float m = warp_max(fabsf(u));
      if (lane == 0) atomicMax((int*)&vmax[v], __float_as_int(m));
      if (u != u) bad = true;
    }
  } else {
    for (int i = tid; i < n; i += NT) {
      const float u = x[i];
      amax = fmaxf(amax, fabsf(u));
      xf[i] = u;
    }
  }
  if (nxv == 1 || p.pro != PRO_NONE) {
    ss = warp_sum(ss);
    amax = warp_max(amax);      // fmaxf drops NaN: NaN is caught per element below
    if (lane == 0) {
      red[w] = ss;
      atomicMax((int*)&vmax[0], __float_as_int(amax));
    }
  }
  named_bar_sync(1, NT);
  float colscale = 1.0f;
  if (p.pro == PRO_RMSNORM) {
    float tss = 0.f;
#pragma unroll
    for (int i = 0; i < NW; ++i) tss += red[i];
    colscale = 1.0f / sqrtf(tss / (float)n + p.eps);
  }

  // limbs: one thread per quad (ks, cc) = 4 elements of each k-half
  const int nqv = n >> 3;
  const size_t xq_vec = (size_t)(n >> 8) * 8 * MMA_KS_BYTES;
  const float up0 = mma_pow2(mma_exp2_scale(vmax[0]));
  if (!(vmax[0] <= 3.0e38f)) bad = true;
  for (int qq = tid; qq < nxv * nqv; qq += NT) {
    const int v = MODE == MMA_MOE ? qq / nqv : 0, q = qq - v * nqv;
    float up = up0;
    if (MODE == MMA_MOE) {
      const float vm = vmax[v];
      if (!(vm <= 3.0e38f)) bad = true;
      up = mma_pow2(mma_exp2_scale(vm));
    }
    const int ks = q >> 2, cc = q & 3;
    const float* xfv = xf + (size_t)v * n;
    uint8_t* xqv = xq + v * xq_vec;
    float part[2];
#pragma unroll
    for (int hp = 0; hp < 2; ++hp) {
      const int e0 = mma_elem<TYPE>(ks, cc, hp);
      const float4 v4 = *(const float4*)&xfv[e0];
      const float vv[4] = {v4.x, v4.y, v4.z, v4.w};
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
      for (int l = 0; l < 4; ++l) {
        uint2 v2 = hp == 0 ? make_uint2(limb[l], 0u) : make_uint2(0u, limb[l]);
        *(uint2*)(xqv + (size_t)ks * MMA_KS_BYTES + (2 * l + hp) * 32 + cc * 8) = v2;
      }
      part[hp] = sum;
    }
    // sub-block sums: Q4_K sums 8 quads (2 ks x 4 cc), Q6_K 4 quads
#pragma unroll
    for (int hp = 0; hp < 2; ++hp) {
      part[hp] += __shfl_xor_sync(0xffffffffu, part[hp], 1);
      part[hp] += __shfl_xor_sync(0xffffffffu, part[hp], 2);
      if (TYPE == T_Q4_K) part[hp] += __shfl_xor_sync(0xffffffffu, part[hp], 4);
    }
    if ((q & (TYPE == T_Q4_K ? 7 : 3)) == 0) {
      float* xs = xsum + (size_t)v * (n >> 8) * 16;
      xs[mma_xsum_slot<TYPE>(ks, 0)] = part[0];
      xs[mma_xsum_slot<TYPE>(ks, 1)] = part[1];
    }
  }
  if (bad) *(volatile int*)&red[2 * NW] = 1;
  named_bar_sync(1, NT);   // also the barrier before the tiles
  return colscale;
}

// Register prologue (RMSNorm or plain input, one vector): thread u holds the
// four consecutive elements 4u..4u+3 from the load to the limb stores, so no
// fp32 staging pass is needed; the sub-blocks (32 elements for Q4_K, 16 for
// Q6_K) are 8 / 4 consecutive lanes, summed with shuffles.  Same outputs as
// gemv_mma_prologue.
template <int NW>
constexpr int mma_pro_items() { return 8192 / 4 / (NW * 32); }   // float4 items per thread (n <= 8192)

// RMSNorm weights of the register prologue: constants, so they are loaded
// before griddepcontrol.wait (their L2 round trip overlaps the previous kernel)
template <int NW>
__device__ __forceinline__ void gemv_mma_prologue_weights(const GemvParams& p, int tid,
                                                          float4 (&w4)[mma_pro_items<NW>()]) {
  constexpr int NT = NW * 32, IT = mma_pro_items<NW>();
  const int nf4 = p.inner >> 2;
#pragma unroll
  for (int j = 0; j < IT; ++j) {
    const int u = tid + j * NT;
    // RMSNorm: weight of each element; head norm (groups of 128): the
    // group's weights, element 4u lying at 4 (u % 32) of its group
    w4[j] = (p.pro == PRO_RMSNORM && u < nf4)          ? ((const float4*)p.pro_w)[u]
            : (p.pro == PRO_HEADNORM_GATE && u < nf4) ? ((const float4*)p.pro_w)[u & 31]
                                                      : make_float4(0.f, 0.f, 0.f, 0.f);
  }
}

template <int TYPE, int NW, int MODE>
__device__ float gemv_mma_prologue_reg(const GemvParams& p, uint8_t* xq, float* xsum, float* red, float* vmax,
                                       int tid, const float4 (&wpre)[mma_pro_items<NW>()]) {
  constexpr int NT = NW * 32;
  constexpr int IT = mma_pro_items<NW>();
  const int n = p.inner, nf4 = n >> 2;
  const int lane = tid & 31, w = tid >> 5;
  const bool rms = p.pro == PRO_RMSNORM;
  const bool xch = MODE == MMA_XCH && p.xch_rk >= 0;
  // head norm x SiLU(z) of the ssm_out input, heads of 128 elements: a warp's
  // 32 float4 items are one head (MMA_GATE kernels only)
  constexpr bool HNG = MODE == MMA_GATE;
  bool bad = false;
  float4 v[IT];
  float4 z4[HNG ? IT : 1];
  float ss = 0.f, amax = 0.f;
  uint32_t tag = 0;
  const unsigned long long* parts = nullptr;
  if (xch) {
    tag = (uint32_t)(*p.xch_seq + (unsigned long long)p.xch_rk + 1ull);
    parts = p.xch_parts[p.xch_rank] + (size_t)(p.xch_rk & 1) * p.xch_n * n;
  }
#pragma unroll
  for (int j = 0; j < IT; ++j) {
    const int u = tid + j * NT;
    v[j] = make_float4(0.f, 0.f, 0.f, 0.f);
    if (u < nf4) v[j] = xch ? __ldcg((const float4*)p.x + u) : ((const float4*)p.x)[u];
    if constexpr (HNG) z4[j] = u < nf4 ? ((const float4*)p.pro_z)[u] : make_float4(0.f, 0.f, 0.f, 0.f);
  }
  if (xch) {
    // residual = x + the ranks' tagged partials of sync xch_rk (rank order)
    for (int r = 0; r < p.xch_n; ++r) {
#pragma unroll
      for (int j = 0; j < IT; ++j) {
        const int u = tid + j * NT;
        if (u >= nf4) continue;
        float pr[4];
#pragma unroll
        for (int t = 0; t < 4; ++t) {
          const unsigned long long* a = parts + (size_t)r * n + 4 * u + t;
          unsigned long long wv = ld_relaxed_sys_u64(a);
          unsigned it = 0;
          // after one word timed out the others are not waited for
          while (!bad && (uint32_t)(wv >> 32) != tag) {
            if (++it > p.xch_spin) {
              if (p.err) atomicExch(p.err, DERR_MBAR_TIMEOUT);
              bad = true;
              break;
            }
            if (it > 1024) __nanosleep(32);
            wv = ld_relaxed_sys_u64(a);
          }
          pr[t] = __uint_as_float((uint32_t)wv);
        }
        v[j].x += pr[0]; v[j].y += pr[1]; v[j].z += pr[2]; v[j].w += pr[3];
      }
    }
  }
#pragma unroll
  for (int j = 0; j < IT; ++j) {
    const int u = tid + j * NT;
    if (u >= nf4) continue;
    if (xch && blockIdx.x == 0) ((float4*)p.x_next)[u] = v[j];
    if constexpr (HNG) {
      float hs = fmaf(v[j].x, v[j].x, fmaf(v[j].y, v[j].y, fmaf(v[j].z, v[j].z, v[j].w * v[j].w)));
      hs = warp_sum(hs);                 // whole warps take this branch together
      const float sc = 1.0f / sqrtf(hs / (float)p.pro_group + p.eps);
      const float4 w4 = wpre[j], zz = z4[j];
      v[j].x = v[j].x * sc * w4.x * zz.x * (1.0f / (1.0f + expf(-zz.x)));
      v[j].y = v[j].y * sc * w4.y * zz.y * (1.0f / (1.0f + expf(-zz.y)));
      v[j].z = v[j].z * sc * w4.z * zz.z * (1.0f / (1.0f + expf(-zz.z)));
      v[j].w = v[j].w * sc * w4.w * zz.w * (1.0f / (1.0f + expf(-zz.w)));
    } else if (rms) {
      ss = fmaf(v[j].x, v[j].x, fmaf(v[j].y, v[j].y, fmaf(v[j].z, v[j].z, fmaf(v[j].w, v[j].w, ss))));
      const float4 w4 = wpre[j];
      v[j].x *= w4.x; v[j].y *= w4.y; v[j].z *= w4.z; v[j].w *= w4.w;
    }
    amax = fmaxf(amax, fmaxf(fmaxf(fabsf(v[j].x), fabsf(v[j].y)), fmaxf(fabsf(v[j].z), fabsf(v[j].w))));
  }
  if (tid == 0) KT_LAST(p.trace, 7);
  if (tid == 0) GEMV_DBG(p, 3);
  ss = warp_sum(ss);
  amax = warp_max(amax);
  if (lane == 0) {
    red[w] = ss;
    red[NW + w] = amax;              // per-warp maxima (no shared atomics)
  }
  named_bar_sync(1, NT);
  float colscale = 1.0f;
  if (rms) {
    float tss = 0.f;
#pragma unroll
    for (int i = 0; i < NW; ++i) tss += red[i];
    colscale = 1.0f / sqrtf(tss / (float)n + p.eps);
  }
  float vm = 0.f;
#pragma unroll
  for (int i = 0; i < NW; ++i) vm = fmaxf(vm, red[NW + i]);
  if (tid == 0) vmax[0] = vm;      // read by the tiles after the next barrier
  if (!(vm <= 3.0e38f)) bad = true;
  const float up = mma_pow2(mma_exp2_scale(vm));
#pragma unroll
  for (int j = 0; j < IT; ++j) {
    const int u = tid + j * NT;
    if (j * NT >= nf4) break;                // whole warps leave together
    const bool ok = u < nf4;
    const int e0 = 4 * u;
    // (k step, lane quad, k half) of elements e0..e0+3 (inverse of mma_elem)
    const int sb = e0 >> 8, r = e0 & 255;
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
    const float vv[4] = {v[j].x, v[j].y, v[j].z, v[j].w};
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
    if (ok) {
#pragma unroll
      for (int l = 0; l < 4; ++l) {
        const uint2 v2 = hp == 0 ? make_uint2(limb[l], 0u) : make_uint2(0u, limb[l]);
        *(uint2*)(xq + (size_t)ks * MMA_KS_BYTES + (2 * l + hp) * 32 + cc * 8) = v2;
      }
    }
    // sub-block sum: 8 (Q4_K) / 4 (Q6_K) consecutive items
    sum += __shfl_xor_sync(0xffffffffu, sum, 1);
    sum += __shfl_xor_sync(0xffffffffu, sum, 2);
    if (TYPE == T_Q4_K) sum += __shfl_xor_sync(0xffffffffu, sum, 4);
    if (ok && (u & (TYPE == T_Q4_K ? 7 : 3)) == 0) xsum[TYPE == T_Q4_K ? (e0 >> 5) : (e0 >> 4)] = sum;
  }
  if (bad) *(volatile int*)&red[2 * NW] = 1;
  named_bar_sync(1, NT);
  return colscale;
}

// ---------------------------------------------------------------------------
// super-block bodies: rows g (ra) and g+8 (rb) of the warp's 16, lane quad c.
// S[0], S[1]: exact integer sums for the two rows; corr: fp32 offset terms.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void mma_sb_q4k(const uint8_t* ra, const uint8_t* rb, const uint8_t* xq_sb,
                                           const float* xs_sb, int lane, float (&acc)[2], float (&corr)[2]) {
  const int c = lane & 3;
  const uint4 ha = *(const uint4*)ra, hb = *(const uint4*)rb;
  // 6-bit scales s0..s7 and mins m0..m7 as bytes (Dequant.jl:345-362)
  const uint32_t sla = ha.y & 0x3f3f3f3fu, sha = (ha.w & 0x0f0f0f0fu) | ((ha.y >> 2) & 0x30303030u);
  const uint32_t slb = hb.y & 0x3f3f3f3fu, shb = (hb.w & 0x0f0f0f0fu) | ((hb.y >> 2) & 0x30303030u);
  int S0 = 0, S1 = 0;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const uint2 qa = *(const uint2*)(ra + 16 + 32 * j + 8 * c);
    const uint2 qb = *(const uint2*)(rb + 16 + 32 * j + 8 * c);
    const uint32_t wsa = j < 2 ? sla : sha, wsb = j < 2 ? slb : shb;
    const int s0a = ubyte<0>(wsa >> (16 * (j & 1))), s1a = ubyte<1>(wsa >> (16 * (j & 1)));
    const int s0b = ubyte<0>(wsb >> (16 * (j & 1))), s1b = ubyte<1>(wsb >> (16 * (j & 1)));
#pragma unroll
    for (int wd = 0; wd < 2; ++wd) {
      const uint32_t wa = wd ? qa.y : qa.x, wb = wd ? qb.y : qb.x;
      const uint2 bv = *(const uint2*)(xq_sb + (2 * j + wd) * MMA_KS_BYTES + lane * 8);
      int d[4];
      imma_k32(d, wa & 0x0f0f0f0fu, wb & 0x0f0f0f0fu, (wa >> 4) & 0x0f0f0f0fu, (wb >> 4) & 0x0f0f0f0fu, bv.x, bv.y);
      S0 += s0a * d[0] + s1a * d[1];
      S1 += s0b * d[2] + s1b * d[3];
    }
  }
  const float2 dda = __half22float2(*(const __half2*)&ha.x), ddb = __half22float2(*(const __half2*)&hb.x);
  acc[0] = fmaf(dda.x, (float)S0, acc[0]);
  acc[1] = fmaf(ddb.x, (float)S1, acc[1]);
  // mins of sub-blocks 2c, 2c+1 (this lane's share of the offset term)
  const uint32_t mla = ha.z & 0x3f3f3f3fu, mha = ((ha.w >> 4) & 0x0f0f0f0fu) | ((ha.z >> 2) & 0x30303030u);
  const uint32_t mlb = hb.z & 0x3f3f3f3fu, mhb = ((hb.w >> 4) & 0x0f0f0f0fu) | ((hb.z >> 2) & 0x30303030u);
  const int sh = 16 * (c & 1);
  const uint32_t ma = (c < 2 ? mla : mha) >> sh, mb = (c < 2 ? mlb : mhb) >> sh;
  const float2 X = *(const float2*)(xs_sb + 2 * c);
  corr[0] = fmaf(dda.y, (float)ubyte<0>(ma) * X.x + (float)ubyte<1>(ma) * X.y, corr[0]);
  corr[1] = fmaf(ddb.y, (float)ubyte<0>(mb) * X.x + (float)ubyte<1>(mb) * X.y, corr[1]);
}

__device__ __forceinline__ void mma_sb_q6k(const uint8_t* ra, const uint8_t* rb, const uint8_t* xq_sb,
                                           const float* xs_sb, int lane, float (&acc)[2], float (&corr)[2]) {
  const int c = lane & 3;
  int S0 = 0, S1 = 0;
  // int8 scales sc[0..15] (four words per row)
  uint32_t sca[4], scb[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    sca[i] = lds_u32_any(ra + 192 + 4 * i);
    scb[i] = lds_u32_any(rb + 192 + 4 * i);
  }
#pragma unroll
  for (int n6 = 0; n6 < 2; ++n6) {
    // qh words for l = 4c.. (h = 0) and 16 + 4c.. (h = 1)
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
        const int k = kk + 2 * hi;      // q group (Dequant.jl:585-596)
        const int sh = 4 * hi;
        const uint32_t ua0 = ((la0 >> sh) & 0x0f0f0f0fu) | qh_bits(ha0, k);
        const uint32_t ua1 = ((la1 >> sh) & 0x0f0f0f0fu) | qh_bits(ha1, k);
        const uint32_t ub0 = ((lb0 >> sh) & 0x0f0f0f0fu) | qh_bits(hb0, k);
        const uint32_t ub1 = ((lb1 >> sh) & 0x0f0f0f0fu) | qh_bits(hb1, k);
        const uint2 bv = *(const uint2*)(xq_sb + (4 * n6 + k) * MMA_KS_BYTES + lane * 8);
        int d[4];
        imma_k32(d, ua0, ub0, ua1, ub1, bv.x, bv.y);
        const int is = 8 * n6 + 2 * k;  // scale index of h = 0; h = 1 is is + 1
        const int s0a = sbyte<0>(sca[is >> 2] >> (8 * (is & 3))), s1a = sbyte<0>(sca[is >> 2] >> (8 * (is & 3) + 8));
        const int s0b = sbyte<0>(scb[is >> 2] >> (8 * (is & 3))), s1b = sbyte<0>(scb[is >> 2] >> (8 * (is & 3) + 8));
        S0 += s0a * d[0] + s1a * d[1];
        S1 += s0b * d[2] + s1b * d[3];
      }
    }
  }
  const float da = h2f_bits(lds_u16_any(ra + 208)), db = h2f_bits(lds_u16_any(rb + 208));
  acc[0] = fmaf(da, (float)S0, acc[0]);
  acc[1] = fmaf(db, (float)S1, acc[1]);
  // offset term 32 * d * sum_j sc_j X_j over sub-blocks 4c..4c+3
  const float4 X = *(const float4*)(xs_sb + 4 * c);
  const uint32_t wa = c == 0 ? sca[0] : c == 1 ? sca[1] : c == 2 ? sca[2] : sca[3];
  const uint32_t wb = c == 0 ? scb[0] : c == 1 ? scb[1] : c == 2 ? scb[2] : scb[3];
  const float ta = (float)sbyte<0>(wa) * X.x + (float)sbyte<1>(wa) * X.y + (float)sbyte<2>(wa) * X.z +
                   (float)sbyte<3>(wa) * X.w;
  const float tb = (float)sbyte<0>(wb) * X.x + (float)sbyte<1>(wb) * X.y + (float)sbyte<2>(wb) * X.z +
                   (float)sbyte<3>(wb) * X.w;
  corr[0] = fmaf(32.0f * da, ta, corr[0]);
  corr[1] = fmaf(32.0f * db, tb, corr[1]);
}

// Q6_K regrouped per 16 rows (T_Q6_KR): for row group G and super-block sb a
// 3360-byte block (= 16 x 210) holds
//   [6 chunks][32 lanes][16 B]  the ql / qh words lane (g, c) reads for rows
//                               g and g + 8 (12 words each, order below),
//   [16 rows][16 B]             int8 scales,   [16 rows][2 B]  fp16 d.
// Word w of a row: w < 8 -> ql at 64*(w>>2) + 32*((w>>1)&1) + 16*(w&1) + 4c,
// w >= 8 -> qh at 128 + 32*((w-8)>>1) + 16*((w-8)&1) + 4c (Dequant.jl:585-596
// offsets).  Every load is an aligned, conflict-free 16-byte access.
constexpr int Q6R_BLOCK = 3360;

__device__ __forceinline__ void mma_sb_q6kr(const uint8_t* gb, const uint8_t* xq_sb, const float* xs_sb, int lane,
                                            float (&acc)[2], float (&corr)[2]) {
  const int c = lane & 3, g = lane >> 2;
  uint32_t wa[12], wb[12];
  {
    const uint4* ch = (const uint4*)gb;
    uint4 t[6];
#pragma unroll
    for (int i = 0; i < 6; ++i) t[i] = ch[i * 32 + lane];
#pragma unroll
    for (int i = 0; i < 3; ++i) {
      wa[4 * i] = t[i].x; wa[4 * i + 1] = t[i].y; wa[4 * i + 2] = t[i].z; wa[4 * i + 3] = t[i].w;
      wb[4 * i] = t[3 + i].x; wb[4 * i + 1] = t[3 + i].y; wb[4 * i + 2] = t[3 + i].z; wb[4 * i + 3] = t[3 + i].w;
    }
  }
  const uint4 sa4 = *(const uint4*)(gb + 3072 + g * 16), sb4 = *(const uint4*)(gb + 3072 + (g + 8) * 16);
  const uint32_t sca[4] = {sa4.x, sa4.y, sa4.z, sa4.w}, scb[4] = {sb4.x, sb4.y, sb4.z, sb4.w};
  int S0 = 0, S1 = 0;
#pragma unroll
  for (int n6 = 0; n6 < 2; ++n6) {
#pragma unroll
    for (int kk = 0; kk < 2; ++kk) {
#pragma unroll
      for (int hi = 0; hi < 2; ++hi) {
        const int k = kk + 2 * hi;
        const int sh = 4 * hi;
        const uint32_t la0 = wa[n6 * 4 + kk * 2], la1 = wa[n6 * 4 + kk * 2 + 1];
        const uint32_t lb0 = wb[n6 * 4 + kk * 2], lb1 = wb[n6 * 4 + kk * 2 + 1];
        const uint32_t ua0 = ((la0 >> sh) & 0x0f0f0f0fu) | qh_bits(wa[8 + n6 * 2], k);
        const uint32_t ua1 = ((la1 >> sh) & 0x0f0f0f0fu) | qh_bits(wa[8 + n6 * 2 + 1], k);
        const uint32_t ub0 = ((lb0 >> sh) & 0x0f0f0f0fu) | qh_bits(wb[8 + n6 * 2], k);
        const uint32_t ub1 = ((lb1 >> sh) & 0x0f0f0f0fu) | qh_bits(wb[8 + n6 * 2 + 1], k);
        const uint2 bv = *(const uint2*)(xq_sb + (4 * n6 + k) * MMA_KS_BYTES + lane * 8);
        int d[4];
        imma_k32(d, ua0, ub0, ua1, ub1, bv.x, bv.y);
        const int is = 8 * n6 + 2 * k;
        const int s0a = sbyte<0>(sca[is >> 2] >> (8 * (is & 3))), s1a = sbyte<0>(sca[is >> 2] >> (8 * (is & 3) + 8));
        const int s0b = sbyte<0>(scb[is >> 2] >> (8 * (is & 3))), s1b = sbyte<0>(scb[is >> 2] >> (8 * (is & 3) + 8));
        S0 += s0a * d[0] + s1a * d[1];
        S1 += s0b * d[2] + s1b * d[3];
      }
    }
  }
  const float da = h2f_bits(*(const uint16_t*)(gb + 3328 + g * 2));
  const float db = h2f_bits(*(const uint16_t*)(gb + 3328 + (g + 8) * 2));
  acc[0] = fmaf(da, (float)S0, acc[0]);
  acc[1] = fmaf(db, (float)S1, acc[1]);
  const float4 X = *(const float4*)(xs_sb + 4 * c);
  const uint32_t wsa = c == 0 ? sca[0] : c == 1 ? sca[1] : c == 2 ? sca[2] : sca[3];
  const uint32_t wsb = c == 0 ? scb[0] : c == 1 ? scb[1] : c == 2 ? scb[2] : scb[3];
  const float ta = (float)sbyte<0>(wsa) * X.x + (float)sbyte<1>(wsa) * X.y + (float)sbyte<2>(wsa) * X.z +
                   (float)sbyte<3>(wsa) * X.w;
  const float tb = (float)sbyte<0>(wsb) * X.x + (float)sbyte<1>(wsb) * X.y + (float)sbyte<2>(wsb) * X.z +
                   (float)sbyte<3>(wsb) * X.w;
  corr[0] = fmaf(32.0f * da, ta, corr[0]);
  corr[1] = fmaf(32.0f * db, tb, corr[1]);
}

template <int TYPE, int NW, int MODE>
__global__ void __launch_bounds__((NW + 1) * 32, NW == 8 ? 2 : 1) gemv_mma_kernel(const __grid_constant__ GemvParams p) {
  extern __shared__ __align__(128) uint8_t smem[];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  if (tid == 0) {
    KT_KIND(p.trace, KT_GEMV_MMA);
    KT_FIRST(p.trace, 1);
    GEMV_DBG(p, 0);
  }
  constexpr int BB = TYPE == T_Q4_K ? 144 : TYPE == T_Q6_KR ? Q6R_BLOCK : 210;
  constexpr int XS_PER_SB = TYPE == T_Q4_K ? 8 : 16;
  // layout: [full][empty][red 2*NW+4][vmax 16][kpart NW*16][xsum][xf][xq][stages]
  uint64_t* full = (uint64_t*)smem;
  uint64_t* empty = full + GEMV_MAX_STAGES;
  float* red = (float*)(empty + GEMV_MAX_STAGES);
  float* vmax = red + 2 * NW + 4;
  float* kpart = vmax + 16;
  float* xsum = kpart + NW * 16;
  const int nsb = p.inner >> 8;
  const int nxv = MODE == MMA_MOE ? p.nxv : 1;
  float* xf = xsum + nxv * nsb * 16;
  uint8_t* xq = (uint8_t*)(xf + (size_t)nxv * p.inner);
  const size_t xq_vec = (size_t)nsb * 8 * MMA_KS_BYTES;
  uint8_t* stage0 = (uint8_t*)(((uintptr_t)(xq + nxv * xq_vec) + 127) & ~(uintptr_t)127);

  if (tid == 0) {
    for (int s = 0; s < p.stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], NW);
    }
    fence_mbar_init();
    *(volatile int*)&red[2 * NW] = 0;   // non-finite input flag
  }
  if (tid < 16) vmax[tid] = 0.f;
  __syncthreads();
  const int G = gridDim.x;
  const int n_items = (p.ntiles - (int)blockIdx.x + G - 1) / G;
  if (warp == NW) {
    gemv_producer<MODE == MMA_MOE>(p, full, empty, stage0, lane, n_items);
    return;
  }

  const bool reg_pro = (MODE == MMA_PLAIN || MODE == MMA_SWIGLU) ||
                       (MODE == MMA_XCH && (p.pro == PRO_RMSNORM || p.pro == PRO_NONE)) ||
                       (MODE == MMA_GATE && p.pro == PRO_HEADNORM_GATE && p.pro_group == 128 && p.inner % 128 == 0);
  float4 wpre[mma_pro_items<NW>()];
  if (reg_pro) gemv_mma_prologue_weights<NW>(p, tid, wpre);
  pdl_wait();
  if (tid == 0) {
    KT_FIRST(p.trace, 2);
    KT_LAST(p.trace, 3);
    if (INFERNO_KTRACE && p.dbg && blockIdx.x == 0) gemv_dbg[30] = gemv_dbg[16 + 7];
    GEMV_DBG(p, 2);
  }
  // residual add (EPI_ADD): the old values of the first tile's rows are
  // loaded now, so their L2 round trip overlaps the prologue instead of
  // sitting between the MMAs and the store
  constexpr bool PRE_ADD_MODE = MODE == MMA_PLAIN || MODE == MMA_GATE;
  float yold[2] = {0.f, 0.f};
  if (PRE_ADD_MODE && p.epi == EPI_ADD && n_items > 0) {
    const int nrg0 = p.TR >> 4, lg0 = __ffs(nrg0) - 1;
    if ((warp >> lg0) == 0 && (lane & 3) == 0) {
      int sg0, r00;
      tile_locate(p, blockIdx.x, sg0, r00);
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int row = r00 + (warp & (nrg0 - 1)) * 16 + (lane >> 2) + 8 * h;
        if (row < p.seg[sg0].rows) yold[h] = p.seg[sg0].y[row];
      }
    }
  }
  const float colscale = reg_pro ? gemv_mma_prologue_reg<TYPE == T_Q6_KR ? T_Q6_K : TYPE, NW, MODE>(p, xq, xsum, red,
                                                                                                     vmax, tid, wpre)
                                 : gemv_mma_prologue<TYPE, NW, MODE>(p, xf, xq, xsum, red, vmax, tid);
  if (tid == 0) KT_LAST(p.trace, 4);
  if (tid == 0) GEMV_DBG(p, 4);
  const bool nonfinite = *(volatile int*)&red[2 * NW] != 0;
  const uint32_t xtag =
      (MODE == MMA_XCH && p.xch_wk >= 0) ? (uint32_t)(*p.xch_seq + (unsigned long long)p.xch_wk + 1ull) : 0u;
  const float fscale0 = nonfinite ? __int_as_float(0x7fc00000) : colscale * mma_pow2(-mma_exp2_scale(vmax[0]));

  const bool paired = MODE == MMA_SWIGLU || ((MODE == MMA_MOE || MODE == MMA_XCH) && p.epi == EPI_SWIGLU);
  const int nrg = p.TR >> 4;            // 16-row groups per tile (1, 2, 4 or 8)
  const int lg_nrg = __ffs(nrg) - 1;
  const int nkg = NW >> lg_nrg;
  const int rg = warp & (nrg - 1), wk = warp >> lg_nrg;
  const int g = lane >> 2, c = lane & 3;
  const float limbw = c == 0 ? 1.0f : c == 1 ? 256.0f : c == 2 ? 65536.0f : 16777216.0f;
  float best_v = -INFINITY;
  int best_i = 0x7fffffff;

  int s = 0, sph = 0;                   // ring stage and its phase parity
  for (int it = 0; it < n_items; ++it, s = (s + 1 == p.stages) ? 0 : s + 1, sph ^= (s == 0)) {
    if (tid == 0 && it == 0) GEMV_DBG(p, 10);
    if (!mbar_wait(&full[s], sph, p.err)) return;
    if (tid == 0 && it == 0) KT_LAST(p.trace, 5);
    if (tid == 0 && it == 0) GEMV_DBG(p, 5);
    int sg, row0;
    tile_locate(p, blockIdx.x + it * G, sg, row0);
    const uint8_t* st = stage0 + (long long)s * p.stage_bytes;
    const uint8_t *ra, *rb;
    if (paired) {
      const uint32_t m0 = (uint32_t)((uintptr_t)seg_row_ptr<MODE == MMA_MOE>(p, 0, row0) & 15);
      const uint32_t m1 = (uint32_t)((uintptr_t)seg_row_ptr<MODE == MMA_MOE>(p, 1, row0) & 15);
      ra = st + m0 + (long long)(rg * 8 + g) * p.row_bytes;
      rb = st + p.part1_off + m1 + (long long)(rg * 8 + g) * p.row_bytes;
    } else if (TYPE == T_Q6_KR) {
      // 16-row groups of nsb 3360-byte blocks, 16-byte aligned
      ra = st + (long long)rg * nsb * Q6R_BLOCK;
      rb = ra;
    } else {
      const uint32_t m0 = (uint32_t)((uintptr_t)seg_row_ptr<MODE == MMA_MOE>(p, sg, row0) & 15);
      ra = st + m0 + (long long)(rg * 16 + g) * p.row_bytes;
      rb = ra + 8ll * p.row_bytes;
    }
    // input vector of this tile and its fixed-point descale
    const int slot = (MODE == MMA_MOE && nxv > 1) ? p.seg[sg].xslot0 + row0 / p.erows : 0;
    const uint8_t* xq_t = xq + slot * xq_vec;
    const float* xsum_t = xsum + slot * nsb * 16;
    const float fscale = (MODE == MMA_MOE && slot) ? (nonfinite ? __int_as_float(0x7fc00000)
                                                                : colscale * mma_pow2(-mma_exp2_scale(vmax[slot])))
                                                   : fscale0;
    float acc[2] = {0.f, 0.f}, corr[2] = {0.f, 0.f};
    const bool skip_tile = seg_skipped<MODE == MMA_MOE>(p, sg, row0);
    for (int sb = wk; sb < nsb && !skip_tile; sb += nkg) {
      if constexpr (TYPE == T_Q4_K)
        mma_sb_q4k(ra + sb * BB, rb + sb * BB, xq_t + (size_t)sb * 8 * MMA_KS_BYTES, xsum_t + sb * XS_PER_SB, lane,
                   acc, corr);
      else if constexpr (TYPE == T_Q6_KR)
        mma_sb_q6kr(ra + sb * BB, xq_t + (size_t)sb * 8 * MMA_KS_BYTES, xsum_t + sb * XS_PER_SB, lane, acc, corr);
      else
        mma_sb_q6k(ra + sb * BB, rb + sb * BB, xq_t + (size_t)sb * 8 * MMA_KS_BYTES, xsum_t + sb * XS_PER_SB, lane,
                   acc, corr);
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);

    // quad reduction: lane c holds limb c of the integer dots and a share of
    // the offset terms
    float ta = limbw * acc[0] - corr[0], tb = limbw * acc[1] - corr[1];
    ta += __shfl_xor_sync(0xffffffffu, ta, 1);
    tb += __shfl_xor_sync(0xffffffffu, tb, 1);
    ta += __shfl_xor_sync(0xffffffffu, ta, 2);
    tb += __shfl_xor_sync(0xffffffffu, tb, 2);
    if (nkg > 1) {
      if (wk > 0 && c == 0) {
        kpart[(wk * nrg + rg) * 16 + g] = ta;
        kpart[(wk * nrg + rg) * 16 + g + 8] = tb;
      }
      named_bar_sync(2, NW * 32);
      if (wk == 0 && c == 0)
        for (int k = 1; k < nkg; ++k) {
          ta += kpart[(k * nrg + rg) * 16 + g];
          tb += kpart[(k * nrg + rg) * 16 + g + 8];
        }
      if (it + 1 < n_items) named_bar_sync(2, NW * 32);   // kpart is reused by the next tile
    }
    if (wk != 0 || c != 0) continue;
    ta *= fscale;
    tb *= fscale;
    if (paired) {
      const int row = row0 + rg * 8 + g;
      if (row < p.seg[0].rows) {
        const float sg_ = ta / (1.0f + expf(-ta));      // mlp_forward (src/ModelCPU.jl:455-468)
        p.seg[0].y[row] = sg_ * tb;
      }
    } else {
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int row = row0 + rg * 16 + g + 8 * h;
        const float t = h ? tb : ta;
        if (row < p.seg[sg].rows) {
          if ((MODE == MMA_PLAIN || MODE == MMA_XCH) && p.epi == EPI_ARGMAX) {
            if (t > best_v || (t == best_v && row < best_i)) { best_v = t; best_i = row; }
            if (p.seg[sg].y) p.seg[sg].y[row] = t;
          } else if (MODE == MMA_XCH && p.xch_wk >= 0) {
            // this rank's partial of sync point xch_wk, to every rank, tagged
            const size_t off = ((size_t)(p.xch_wk & 1) * p.xch_n + p.xch_rank) * p.seg[0].rows + row;
            const unsigned long long wv = ((unsigned long long)xtag << 32) | __float_as_uint(t);
            for (int q = 0; q < p.xch_n; ++q) st_relaxed_sys_u64(p.xch_parts[q] + off, wv);
          } else {
            float* y = p.seg[sg].y + row;
            if (p.epi == EPI_ADD) *y = (PRE_ADD_MODE && it == 0 ? yold[h] : *y) + t;
            else *y = t;
          }
        }
      }
    }
  }
  if (tid == 0) KT_LAST(p.trace, 6);
  if (tid == 0) GEMV_DBG(p, 6);
  if (INFERNO_KTRACE && p.dbg == 2 && reg_pro) {
    // debug: the register prologue once more, with its code now in the
    // instruction cache (slots 8 / 9 around it)
    named_bar_sync(1, NW * 32);
    if (tid == 0) GEMV_DBG(p, 8);
    GemvParams q = p;
    q.dbg = 0;
    (void)gemv_mma_prologue_reg<TYPE == T_Q6_KR ? T_Q6_K : TYPE, NW, MODE>(q, xq, xsum, red, vmax, tid, wpre);
    if (tid == 0) GEMV_DBG(p, 9);
  }
  if ((MODE == MMA_PLAIN || MODE == MMA_XCH) && p.epi == EPI_ARGMAX && wk == 0) {
    float v = best_v;
    int i = best_i;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, v, o);
      const int oi = __shfl_xor_sync(0xffffffffu, i, o);
      if (ov > v || (ov == v && oi < i)) { v = ov; i = oi; }
    }
    if (lane == 0 && i != 0x7fffffff) {
      const unsigned long long key = ((unsigned long long)float_ordered(v) << 32) |
                                     (unsigned long long)(0xffffffffu - (uint32_t)(i + p.argmax_row0));
      atomicMax(&p.argmax[0], key);
    }
  }
  if (tid == 0) GEMV_DBG(p, 7);
}

}  // namespace inf
