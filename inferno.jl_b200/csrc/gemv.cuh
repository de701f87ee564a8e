// Fused dequant-GEMV over GGUF super-blocks in their native byte layout.
//
// Replaces ModelCPU.mul! / mul_quant_mat_vec (Inferno.jl src/ModelCPU.jl:284-444)
// and the C kernels behind QuantizedKernels.jl (src/kernels/quant_kernels.c:602-697),
// with the reference's fp32 numerics (exact dequant, fp32 activations; no int8
// activation quantization).
//
// Design (HBM-bound streaming kernel, one CTA per SM-slot):
//  * A "tile" is TR = 8*R consecutive rows of one matrix; a "chunk" is 1024
//    input elements of those rows.  The producer warp streams (tile, chunk)
//    items into a ring of shared-memory stages with 1-D TMA bulk copies
//    (cp.async.bulk + mbarrier complete_tx), one copy per row segment.  Row
//    segments of 210-, 66- and 34-byte block formats are not 16-byte aligned,
//    so each copy covers the aligned superset and consumers index from the
//    remainder.
//  * 8 consumer warps; warp w owns R rows of the tile and each lane owns one
//    32-element fragment of the chunk, so the fragment's activations sit in
//    registers and are reused for all R rows.
//  * Sub-block scales are applied once per fragment run: for Q4_K/Q5_K
//    sum(w*x) = d1*sum(q*x) - min1*sum(x) with sum(x) precomputed per 16
//    elements in the prologue.  Integers become floats through the 2^23
//    magic-exponent trick (byte_perm + fsub), exact for these ranges.
//  * Weight streaming starts before griddepcontrol.wait, so under
//    programmatic dependent launch it overlaps the previous kernel's tail.
//  * Prologues fuse the input transform (RMSNorm, or per-head RMSNorm x
//    SiLU(z) gate of the Gated DeltaNet output); epilogues fuse the residual
//    add, SwiGLU of paired gate/up rows, or first-max argmax for lm_head.
#pragma once
#include "common.cuh"

namespace inf {

enum Pro : int { PRO_NONE = 0, PRO_RMSNORM = 1, PRO_HEADNORM_GATE = 2 };
enum Epi : int { EPI_STORE = 0, EPI_ADD = 1, EPI_SWIGLU = 2, EPI_ARGMAX = 3 };

// Consumer warps per CTA (template NW): 8 for the per-layer matrices (two
// CTAs fit on an SM, so the next kernel can be resident under programmatic
// dependent launch), 16 for large matrices (lm_head).
constexpr int GEMV_CHUNK = 1024;              // elements per chunk (32 lanes x 32)
constexpr int GEMV_MAX_SEG = 4;
constexpr int GEMV_MAX_STAGES = 8;

struct GemvSeg {
  const uint8_t* W;   // matrix base (16-byte aligned, readable to the next 16 B)
  float* y;           // output rows (EPI_SWIGLU: only seg[0].y is used)
  int rows;
  int tile0;          // first global tile index of this segment
  int indirect;       // rows gathered through GemvParams::eidx (MoE experts)
  int xslot0;         // input-vector slot of row 0 (nxv > 1)
};

struct GemvParams {
  GemvSeg seg[GEMV_MAX_SEG];
  int nseg, ntiles;
  int inner, row_bytes, nkc;
  int TR, slot, stages;
  int nkg;                        // K groups: warps splitting a tile's chunks
  int contig;                     // 1: a tile's rows are copied as one range (nkc == 1)
  int stage_bytes;
  int part1_off;                  // contig + SwiGLU: stage offset of the up-rows range
  int nb;                         // batch columns
  const float* x;                 // [nb][x_stride]
  long long x_stride, y_stride;
  int pro;
  const float* pro_w;             // norm weight
  const float* pro_z;             // gate input (PRO_HEADNORM_GATE)
  float eps;
  int pro_group;                  // head size for PRO_HEADNORM_GATE
  int epi;
  unsigned long long* argmax;     // [nb] packed (ordered value, ~index)
  int argmax_row0;                // global index of row 0 (vocab-split lm_head)
  int* err;
  int l2_evict_first;             // stream weights with an L2 evict_first policy
  // 1: the producer warp lets the next kernel launch at once (it reads only
  // weights, which no kernel writes), so under programmatic dependent launch
  // the next kernel's CTAs become resident and start streaming their own
  // weights while this kernel still computes
  int early_trigger;
  const int* eidx;                // MoE: expert id per erows-row block of an indirect segment
  long long estride;              // bytes between experts
  int erows;                      // rows per expert block (also the input-slot period)
  int n_experts;                  // valid ids are [0, n_experts)
  int nxv;                        // input vectors (tensor-core path, PRO_NONE)
  // Tensor-parallel residual exchange over NVLink peer memory (tensor-core
  // path), low-latency protocol: every element travels as one 64-bit word
  // {fp32 value, 32-bit tag}, tag = *xch_seq + k + 1 for sync point k, so the
  // data is its own flag (no fences, counters or flag words).
  // Writer (xch_wk >= 0): the output rows are this rank's partial of sync k
  // and go to parts[k & 1][rank][row] on every rank.  Reader (xch_rk >= 0):
  // polls parts[k & 1][r][i] until the tags match, uses x + sum_r partial_r
  // (rank order: bit-identical on every rank) and CTA 0 stores it in x_next.
  int xch_n, xch_rank, xch_wk, xch_rk;
  unsigned xch_spin;              // polls of one word before the reader gives up (DERR_MBAR_TIMEOUT)
  const unsigned long long* xch_seq;
  unsigned long long* xch_parts[8];  // each rank's [2][n][H] words
  float* x_next;
  unsigned long long* trace;      // debug: 8 timeline slots of this launch (KT_*; null = off)
  int dbg;                        // debug (-DINFERNO_KTRACE=1 builds): stamps into gemv_dbg (INFERNO_GEMV_DBG)
};

// debug timeline of the tensor-core GEMV (GemvParams::dbg): slots 0-15 CTA 0,
// 16-31 the last CTA, %globaltimer ns; slot 30 = the previous launch's
// last-CTA exit as seen after this launch's griddepcontrol.wait
static __device__ unsigned long long gemv_dbg[32];
#define GEMV_DBG(p, i)                                                             \
  do {                                                                             \
    if (INFERNO_KTRACE && (p).dbg) {                                               \
      if (blockIdx.x == 0) gemv_dbg[i] = gtimer();                                 \
      else if (blockIdx.x == gridDim.x - 1) gemv_dbg[16 + (i)] = gtimer();         \
    }                                                                              \
  } while (0)

__device__ __constant__ uint64_t c_iq2xxs_grid_init[256] = {
#include "iq2xxs_grid.inc"
};

// ---------------------------------------------------------------------------
// packed fp32x2 helpers (sm_100: add/sub/fma .f32x2 on 64-bit register pairs)
// ---------------------------------------------------------------------------
typedef unsigned long long f2_t;
__device__ __forceinline__ f2_t pk2(uint32_t a, uint32_t b) {
  f2_t r;
  asm("mov.b64 %0, {%1,%2};" : "=l"(r) : "r"(a), "r"(b));
  return r;
}
__device__ __forceinline__ f2_t pk2f(float a, float b) { return pk2(__float_as_uint(a), __float_as_uint(b)); }
__device__ __forceinline__ float2 upk2(f2_t v) {
  uint32_t a, b;
  asm("mov.b64 {%0,%1}, %2;" : "=r"(a), "=r"(b) : "l"(v));
  return make_float2(__uint_as_float(a), __uint_as_float(b));
}
__device__ __forceinline__ f2_t ffma2(f2_t a, f2_t b, f2_t c) {
  f2_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ f2_t fadd2(f2_t a, f2_t b) {
  f2_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ f2_t fsub2(f2_t a, f2_t b) {
  f2_t d;
  asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ float hsum2(f2_t v) {
  float2 f = upk2(v);
  return f.x + f.y;
}

constexpr float MAGIC = 8388608.0f;
// two bytes (k, k+1) of w as exact floats minus `off`, packed
template <int K>
__device__ __forceinline__ f2_t bytes2(uint32_t w, f2_t magic_off) {
  uint32_t a = __byte_perm(w, 0x4B000000u, 0x7650u | K);
  uint32_t b = __byte_perm(w, 0x4B000000u, 0x7650u | (K + 1));
  return fsub2(pk2(a, b), magic_off);
}

// ---------------------------------------------------------------------------
// per-type fragment dot products.  rowp = start of this row's chunk in smem
// (block 0 of the chunk).  x = the lane's 32 activations as 16 packed pairs
// (type-specific order), xs_* = run sums where a type needs them.
// ---------------------------------------------------------------------------
template <int TYPE>
struct Frag;

// Q4_K/Q5_K 6-bit scales and mins of sub-blocks 2j and 2j+1 (the unpack of
// Inferno.jl src/Dequant.jl:345-362, done on byte pairs): returns the packed
// float pairs (sc_2j, sc_2j+1) and (m_2j, m_2j+1).
__device__ __forceinline__ void kscale_pair(uint4 hd, int j, f2_t& sc, f2_t& mn) {
  const int sh = ((2 * j) & 3) * 8;
  uint32_t a = hd.y >> sh, b = hd.z >> sh, c = hd.w >> sh;
  uint32_t sc_lo = a & 0x3f3fu, m_lo = b & 0x3f3fu;
  uint32_t sc_hi = (c & 0x0f0fu) | ((a >> 2) & 0x3030u);
  uint32_t m_hi = ((c >> 4) & 0x0f0fu) | ((b >> 2) & 0x3030u);
  uint32_t s = j < 2 ? sc_lo : sc_hi, m = j < 2 ? m_lo : m_hi;
  const f2_t MM = pk2f(MAGIC, MAGIC);
  sc = bytes2<0>(s, MM);
  mn = bytes2<0>(m, MM);
}

template <>
struct Frag<T_Q4_K> {
  // lane -> block lane>>3, sub-block pair j=(lane>>1)&3, half h=lane&1:
  // lo run = elements j*64+16h+[0,16), hi run = j*64+32+16h+[0,16)
  __device__ static int xpos(int lane, int i) {
    int b = lane >> 3, j = (lane >> 1) & 3, h = lane & 1;
    return b * 256 + j * 64 + 16 * h + (i < 16 ? i : 16 + i);
  }
  static constexpr bool kNeedSums = true;
  __device__ static float dot(const uint8_t* rowp, int lane, const f2_t* x, float xs_lo, float xs_hi) {
    const uint8_t* blk = rowp + (lane >> 3) * 144;
    const int j = (lane >> 1) & 3, h = lane & 1;
    const uint4 hd = *(const uint4*)blk;
    const uint4 qv = *(const uint4*)(blk + 16 + j * 32 + 16 * h);
    const uint32_t w4[4] = {qv.x, qv.y, qv.z, qv.w};
    const f2_t MM = pk2f(MAGIC, MAGIC);
    f2_t slo = 0ull, shi = 0ull;
#pragma unroll
    for (int w = 0; w < 4; ++w) {
      uint32_t lo = w4[w] & 0x0f0f0f0fu, hi = (w4[w] >> 4) & 0x0f0f0f0fu;
      slo = ffma2(bytes2<0>(lo, MM), x[2 * w], slo);
      shi = ffma2(bytes2<0>(hi, MM), x[8 + 2 * w], shi);
      slo = ffma2(bytes2<2>(lo, MM), x[2 * w + 1], slo);
      shi = ffma2(bytes2<2>(hi, MM), x[8 + 2 * w + 1], shi);
    }
    f2_t sc, mn;
    kscale_pair(hd, j, sc, mn);
    const float2 dd = h2f_pair(hd.x);
    const float2 s2 = upk2(sc), m2 = upk2(mn);
    const float d1 = dd.x * s2.x, mn1 = dd.y * m2.x, d2 = dd.x * s2.y, mn2 = dd.y * m2.y;
    return (d1 * hsum2(slo) - mn1 * xs_lo) + (d2 * hsum2(shi) - mn2 * xs_hi);
  }
  __device__ static float2 h2f_pair(uint32_t w) {
    return make_float2(h2f_bits((uint16_t)(w & 0xffffu)), h2f_bits((uint16_t)(w >> 16)));
  }
};

template <>
struct Frag<T_Q5_K> {
  __device__ static int xpos(int lane, int i) { return Frag<T_Q4_K>::xpos(lane, i); }
  static constexpr bool kNeedSums = true;
  __device__ static float dot(const uint8_t* rowp, int lane, const f2_t* x, float xs_lo, float xs_hi) {
    const uint8_t* blk = rowp + (lane >> 3) * 176;
    const int j = (lane >> 1) & 3, h = lane & 1;
    const uint4 hd = *(const uint4*)blk;
    const uint4 qv = *(const uint4*)(blk + 48 + j * 32 + 16 * h);
    const uint4 hv = *(const uint4*)(blk + 16 + 16 * h);
    const uint32_t w4[4] = {qv.x, qv.y, qv.z, qv.w};
    const uint32_t h4[4] = {hv.x, hv.y, hv.z, hv.w};
    const f2_t MM = pk2f(MAGIC, MAGIC);
    f2_t slo = 0ull, shi = 0ull;
#pragma unroll
    for (int w = 0; w < 4; ++w) {
      uint32_t lo = (w4[w] & 0x0f0f0f0fu) | (((h4[w] >> (2 * j)) & 0x01010101u) << 4);
      uint32_t hi = ((w4[w] >> 4) & 0x0f0f0f0fu) | (((h4[w] >> (2 * j + 1)) & 0x01010101u) << 4);
      slo = ffma2(bytes2<0>(lo, MM), x[2 * w], slo);
      shi = ffma2(bytes2<0>(hi, MM), x[8 + 2 * w], shi);
      slo = ffma2(bytes2<2>(lo, MM), x[2 * w + 1], slo);
      shi = ffma2(bytes2<2>(hi, MM), x[8 + 2 * w + 1], shi);
    }
    f2_t sc, mn;
    kscale_pair(hd, j, sc, mn);
    const float2 dd = Frag<T_Q4_K>::h2f_pair(hd.x);
    const float2 s2 = upk2(sc), m2 = upk2(mn);
    const float d1 = dd.x * s2.x, mn1 = dd.y * m2.x, d2 = dd.x * s2.y, mn2 = dd.y * m2.y;
    return (d1 * hsum2(slo) - mn1 * xs_lo) + (d2 * hsum2(shi) - mn2 * xs_hi);
  }
};

template <>
struct Frag<T_Q6_K> {
  // lane -> block lane>>3, half n=(lane>>2)&1, l-run m=lane&3: four runs
  // n*128 + 32k + 8m + [0,8), k = 0..3 (the q1..q4 groups of Dequant.jl:585-596)
  __device__ static int xpos(int lane, int i) {
    int b = lane >> 3, n = (lane >> 2) & 1, m = lane & 3;
    return b * 256 + n * 128 + 32 * (i >> 3) + 8 * m + (i & 7);
  }
  static constexpr bool kNeedSums = false;
  __device__ static float dot(const uint8_t* rowp, int lane, const f2_t* x, float, float) {
    const uint8_t* blk = rowp + (lane >> 3) * 210;
    const int n = (lane >> 2) & 1, m = lane & 3;
    const uint8_t* A = blk + n * 64 + 8 * m;
    const uint8_t* Hq = blk + 128 + n * 32 + 8 * m;
    const f2_t MO = pk2f(MAGIC + 32.0f, MAGIC + 32.0f);
    f2_t s0 = 0ull, s1 = 0ull, s2 = 0ull, s3 = 0ull;
#pragma unroll
    for (int w = 0; w < 2; ++w) {
      uint32_t a = lds_u32_any(A + 4 * w), b = lds_u32_any(A + 32 + 4 * w), hh = lds_u32_any(Hq + 4 * w);
      uint32_t q1 = (a & 0x0f0f0f0fu) | ((hh & 0x03030303u) << 4);
      uint32_t q2 = (b & 0x0f0f0f0fu) | (((hh >> 2) & 0x03030303u) << 4);
      uint32_t q3 = ((a >> 4) & 0x0f0f0f0fu) | (((hh >> 4) & 0x03030303u) << 4);
      uint32_t q4 = ((b >> 4) & 0x0f0f0f0fu) | (((hh >> 6) & 0x03030303u) << 4);
      s0 = ffma2(bytes2<0>(q1, MO), x[2 * w], s0);
      s0 = ffma2(bytes2<2>(q1, MO), x[2 * w + 1], s0);
      s1 = ffma2(bytes2<0>(q2, MO), x[4 + 2 * w], s1);
      s1 = ffma2(bytes2<2>(q2, MO), x[4 + 2 * w + 1], s1);
      s2 = ffma2(bytes2<0>(q3, MO), x[8 + 2 * w], s2);
      s2 = ffma2(bytes2<2>(q3, MO), x[8 + 2 * w + 1], s2);
      s3 = ffma2(bytes2<0>(q4, MO), x[12 + 2 * w], s3);
      s3 = ffma2(bytes2<2>(q4, MO), x[12 + 2 * w + 1], s3);
    }
    // int8 scales sc[is], sc[is+2], sc[is+4], sc[is+6], is = n*8 + m/2
    const uint32_t scw = lds_u32_any(blk + 192 + n * 8 + (m >> 1));
    const uint32_t scw2 = lds_u32_any(blk + 192 + n * 8 + (m >> 1) + 4);
    const float d = h2f_bits(lds_u16_any(blk + 208));
    const float c0 = (float)(int8_t)(scw & 0xffu), c1 = (float)(int8_t)((scw >> 16) & 0xffu);
    const float c2 = (float)(int8_t)(scw2 & 0xffu), c3 = (float)(int8_t)((scw2 >> 16) & 0xffu);
    return ((d * c0) * hsum2(s0) + (d * c1) * hsum2(s1)) + ((d * c2) * hsum2(s2) + (d * c3) * hsum2(s3));
  }
};

template <>
struct Frag<T_Q8_0> {
  __device__ static int xpos(int lane, int i) { return lane * 32 + i; }
  static constexpr bool kNeedSums = false;
  __device__ static float dot(const uint8_t* rowp, int lane, const f2_t* x, float, float) {
    const uint8_t* blk = rowp + lane * 34;
    const float d = h2f_bits(lds_u16_any(blk));
    const f2_t MO = pk2f(MAGIC + 128.0f, MAGIC + 128.0f);
    f2_t s0 = 0ull, s1 = 0ull;
#pragma unroll
    for (int w = 0; w < 8; ++w) {
      uint32_t q = lds_u32_any(blk + 2 + 4 * w) ^ 0x80808080u;
      s0 = ffma2(bytes2<0>(q, MO), x[2 * w], s0);
      s1 = ffma2(bytes2<2>(q, MO), x[2 * w + 1], s1);
    }
    return d * (hsum2(s0) + hsum2(s1));
  }
};

template <>
struct Frag<T_IQ2_XXS> {
  __device__ static int xpos(int lane, int i) { return (lane >> 3) * 256 + (lane & 7) * 32 + i; }
  static constexpr bool kNeedSums = false;
  // grid: 256 x uint64 codebook in shared memory
  __device__ static float dot_grid(const uint8_t* rowp, int lane, const f2_t* x, const uint2* grid) {
    const uint8_t* blk = rowp + (lane >> 3) * 66;
    const int ib = lane & 7;
    const float d = h2f_bits(lds_u16_any(blk));
    const uint32_t a1 = lds_u32_any(blk + 2 + ib * 8), a2 = lds_u32_any(blk + 6 + ib * 8);
    const float db = d * (0.5f + (float)(a2 >> 28)) * 0.25f;   // Dequant.jl:36
    const f2_t MO = pk2f(MAGIC + 8.0f, MAGIC + 8.0f);
    f2_t s = 0ull;
#pragma unroll
    for (int l = 0; l < 4; ++l) {
      const uint2 g = grid[(a1 >> (8 * l)) & 0xffu];
      uint32_t sg = (a2 >> (7 * l)) & 127u;
      sg |= (uint32_t)(__popc(sg) & 1) << 7;            // KSIGNS_IQ2XS
      // sign bits j -> bit 31 of the matching float
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const uint32_t word = q < 2 ? g.x : g.y;
        f2_t v = (q & 1) ? bytes2<2>(word, MO) : bytes2<0>(word, MO);
        const uint32_t s0 = ((sg >> (2 * q)) & 1u) << 31, s1 = ((sg >> (2 * q + 1)) & 1u) << 31;
        v ^= pk2(s0, s1);
        s = ffma2(v, x[l * 4 + q], s);
      }
    }
    return db * hsum2(s);
  }
};

template <>
struct Frag<T_F32> {
  __device__ static int xpos(int lane, int i) { return lane * 32 + i; }
  static constexpr bool kNeedSums = false;
  __device__ static float dot(const uint8_t* rowp, int lane, const f2_t* x, float, float) {
    const f2_t* w = (const f2_t*)(rowp + lane * 128);
    f2_t s0 = 0ull, s1 = 0ull;
#pragma unroll
    for (int k = 0; k < 16; k += 2) {
      s0 = ffma2(w[k], x[k], s0);
      s1 = ffma2(w[k + 1], x[k + 1], s1);
    }
    return hsum2(s0) + hsum2(s1);
  }
};

// Multi-row warp reduction: R per-lane partial sums -> lane L holds the full
// sum of row reduce_row<R>(L) (transpose-reduce: R-1 + 5 - log2 R shuffles).
template <int R>
__device__ __forceinline__ float reduce_rows(float (&v)[R], int lane) {
  if constexpr (R == 4) {
    const bool u16 = lane & 16, u8 = lane & 8;
    float a = u16 ? v[2] : v[0], b = u16 ? v[0] : v[2];
    float c = u16 ? v[3] : v[1], d = u16 ? v[1] : v[3];
    a += __shfl_xor_sync(0xffffffffu, b, 16);
    c += __shfl_xor_sync(0xffffffffu, d, 16);
    float e = u8 ? c : a, f = u8 ? a : c;
    e += __shfl_xor_sync(0xffffffffu, f, 8);
    e += __shfl_xor_sync(0xffffffffu, e, 4);
    e += __shfl_xor_sync(0xffffffffu, e, 2);
    e += __shfl_xor_sync(0xffffffffu, e, 1);
    return e;
  } else if constexpr (R == 2) {
    const bool u16 = lane & 16;
    float a = u16 ? v[1] : v[0], b = u16 ? v[0] : v[1];
    a += __shfl_xor_sync(0xffffffffu, b, 16);
    a += __shfl_xor_sync(0xffffffffu, a, 8);
    a += __shfl_xor_sync(0xffffffffu, a, 4);
    a += __shfl_xor_sync(0xffffffffu, a, 2);
    a += __shfl_xor_sync(0xffffffffu, a, 1);
    return a;
  } else {
    return warp_sum(v[0]);
  }
}
// row index whose total lane `lane` holds after reduce_rows<R>
template <int R>
__device__ __forceinline__ int reduce_row_of(int lane) {
  if constexpr (R == 4) return ((lane >> 4) & 1) * 2 + ((lane >> 3) & 1);
  else if constexpr (R == 2) return (lane >> 4) & 1;
  else return 0;
}
// lanes that write a row after reduce_rows<R> (one per row)
template <int R>
__device__ __forceinline__ bool reduce_writer(int lane) {
  if constexpr (R == 4) return (lane & 7) == 0;
  else if constexpr (R == 2) return (lane & 15) == 0;
  else return lane == 0;
}

// Shared-memory activation layout ("fragment-interleaved"): element e of
// chunk kc, held by lane L in fragment slot q (e == Frag::xpos(L, q)), lives at
// float index  kc*1024 + (q/4)*128 + L*4 + q%4  so that for every float4 k a
// warp's 32 lanes read 512 consecutive bytes (no bank conflicts).
template <int TYPE>
__device__ __forceinline__ int xperm(int i) {
  const int kc = i >> 10, e = i & 1023;
  int lane, q;
  if (TYPE == T_Q4_K || TYPE == T_Q5_K) {
    const int bb = e >> 8, r = e & 255, j = r >> 6, rr = r & 63, hi = rr >> 5, t = rr & 31;
    lane = bb * 8 + j * 2 + (t >> 4);
    q = hi * 16 + (t & 15);
  } else if (TYPE == T_Q6_K) {
    const int bb = e >> 8, r = e & 255, n = r >> 7, r2 = r & 127, k = r2 >> 5, r3 = r2 & 31;
    lane = bb * 8 + n * 4 + (r3 >> 3);
    q = k * 8 + (r3 & 7);
  } else {
    lane = e >> 5;
    q = e & 31;
  }
  return (kc << 10) + (q >> 2) * 128 + lane * 4 + (q & 3);
}

// Prologue: the input vector(s) in the permuted layout, in one pass and one
// barrier.  For RMSNorm the stored value is x*w (norm weight) and the 1/rms
// factor, a scalar per batch column, is applied to each row's dot product in
// the epilogue: scale * sum_i W[r,i] x[i] w[i] == sum_i W[r,i] (x[i]*scale*w[i])
// (rmsnorm_cpu!, src/ModelCPU.jl:110-122, reassociated).  red[b*NW + warp]
// receives the per-warp partial sums of x^2.
template <int TYPE, int NW>
__device__ void gemv_prologue(const GemvParams& p, float* xs, float* red, int tid) {
  const int n = p.inner;
  const int npad = p.nkc * GEMV_CHUNK;
  const int lane = tid & 31, w = tid >> 5;
  for (int b = 0; b < p.nb; ++b) {
    const float* x = p.x + (long long)b * p.x_stride;
    float* o = xs + (long long)b * npad;
    if (p.pro == PRO_RMSNORM) {
      float ss = 0.f;
      for (int i = tid; i < n; i += NW * 32) {
        const float v = x[i];
        ss = fmaf(v, v, ss);
        o[xperm<TYPE>(i)] = v * p.pro_w[i];
      }
      ss = warp_sum(ss);
      if (lane == 0) red[b * NW + w] = ss;
    } else if (p.pro == PRO_HEADNORM_GATE) {
      // per-head rmsnorm of the GDN output, then * z * sigmoid(z)
      // (src/ModelCPU.jl:682-692); warp per head, loads first, compact code
      const int G = p.pro_group;
      const float* z = p.pro_z + (long long)b * p.x_stride;
      const int per = G >> 5;                 // elements per lane (G <= 256)
#pragma unroll 1
      for (int hh = w; hh < n / G; hh += NW) {
        float yv[8], zv[8], wv[8];
        float ss = 0.f;
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          const bool ok = q < per;
          const int i = hh * G + q * 32 + lane;
          yv[q] = ok ? x[i] : 0.f;
          zv[q] = ok ? z[i] : 0.f;
          wv[q] = ok ? p.pro_w[q * 32 + lane] : 0.f;
        }
#pragma unroll
        for (int q = 0; q < 8; ++q) ss = fmaf(yv[q], yv[q], ss);
        ss = warp_sum(ss);
        const float scale = 1.0f / sqrtf(ss / (float)G + p.eps);
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          if (q >= per) break;
          const float v = yv[q] * scale * wv[q];
          o[xperm<TYPE>(hh * G + q * 32 + lane)] = v * zv[q] * (1.0f / (1.0f + expf(-zv[q])));
        }
      }
    } else {
      for (int i = tid; i < n; i += NW * 32) o[xperm<TYPE>(i)] = x[i];
    }
  }
  named_bar_sync(1, NW * 32);
}

// ---------------------------------------------------------------------------
// the kernel
// ---------------------------------------------------------------------------
__device__ __forceinline__ void tile_locate(const GemvParams& p, int tile, int& seg, int& row0) {
  seg = 0;
#pragma unroll
  for (int s = 1; s < GEMV_MAX_SEG; ++s)
    if (s < p.nseg && tile >= p.seg[s].tile0) seg = s;
  const int half = (p.epi == EPI_SWIGLU) ? p.TR / 2 : p.TR;
  row0 = (tile - p.seg[seg].tile0) * half;
}

// Address of row `row0` of segment `sg`.  Indirect (MoE) segments map row r to
// row r % erows of expert eidx[r / erows]; a tile never straddles two experts.
// An out-of-range id is reported and replaced by expert 0.
template <bool IND = true>
__device__ __forceinline__ const uint8_t* seg_row_ptr(const GemvParams& p, int sg, int row0) {
  const GemvSeg& s = p.seg[sg];
  if (!IND || !s.indirect) return s.W + (long long)row0 * p.row_bytes;
  const int slot = row0 / p.erows;
  int e = p.eidx[slot];
  if (e >= p.n_experts) {
    if (p.err) atomicExch(p.err, DERR_BAD_ARG);
    e = 0;
  }
  if (e < 0) e = 0;     // an expert of another rank (seg_skipped): never read
  return s.W + (long long)e * p.estride + (long long)(row0 - slot * p.erows) * p.row_bytes;
}

// Expert parallelism: a negative id marks a selected expert held by another
// rank; its tiles are neither copied nor computed and their outputs are 0.
template <bool IND = true>
__device__ __forceinline__ bool seg_skipped(const GemvParams& p, int sg, int row0) {
  return IND && p.seg[sg].indirect && p.eidx[row0 / p.erows] < 0;
}

// Producer warp of the GEMV kernels: one bulk copy per tile (two for paired
// gate/up tiles) into the ring of stages.  Weights stream before
// griddepcontrol.wait; dependents are released only after it.
template <bool IND = true>
__device__ __forceinline__ void gemv_producer(const GemvParams& p, uint64_t* full, uint64_t* empty, uint8_t* stage0,
                                              int lane, int n_items) {
  const int G = gridDim.x;
  const bool paired = (p.epi == EPI_SWIGLU);
  const int TR = p.TR, half_tr = TR / 2;
  bool waited = false;
  if (p.early_trigger && !(IND && p.eidx)) {
    pdl_trigger();
    waited = true;
  }
  if (IND && p.eidx) {
    // expert ids come from the preceding kernel: no weight prefetch before the wait
    pdl_wait();
    pdl_trigger();
    waited = true;
  }
  int s = 0, sph = 1;                   // ring stage; parity of its previous use
  for (int it = 0; it < n_items; ++it, s = (s + 1 == p.stages) ? 0 : s + 1, sph ^= (s == 0)) {
    if (it >= p.stages) {
      if (!mbar_wait(&empty[s], sph, p.err)) break;
    }
    int sg, row0;
    tile_locate(p, blockIdx.x + it * G, sg, row0);
    uint8_t* st = stage0 + (long long)s * p.stage_bytes;
    if (lane < (paired ? 2 : 1)) {
      const int sgr = paired ? lane : sg;
      const int nrows = seg_skipped<IND>(p, sgr, row0) ? 0 : min(paired ? half_tr : TR, p.seg[sgr].rows - row0);
      uint32_t bytes = 0;
      uintptr_t a0 = 0;
      if (nrows > 0) {
        const uintptr_t src = (uintptr_t)seg_row_ptr<IND>(p, sgr, row0);
        a0 = src & ~(uintptr_t)15;
        const uintptr_t a1 = (src + (long long)nrows * p.row_bytes + 15) & ~(uintptr_t)15;
        bytes = (uint32_t)(a1 - a0);
      }
      const uint32_t other = __shfl_down_sync(paired ? 3u : 1u, bytes, 1, paired ? 2 : 1);
      if (lane == 0) mbar_arrive_expect_tx(&full[s], bytes + (paired ? other : 0u));
      __syncwarp(paired ? 3u : 1u);
      if (bytes) {
        // weights are read once per token: stream them with evict_first
        if (p.l2_evict_first)
          tma_load_1d_hint(st + (lane ? p.part1_off : 0), (const void*)a0, bytes, &full[s], l2_policy_evict_first());
        else
          tma_load_1d(st + (lane ? p.part1_off : 0), (const void*)a0, bytes, &full[s]);
      }
    }
    if (lane == 0 && it == 0) GEMV_DBG(p, 1);
    // weights stream before the wait; dependents launch only after it
    if ((it == p.stages - 1 || it == n_items - 1) && !waited) {
      pdl_wait();
      pdl_trigger();
      waited = true;
    }
  }
  if (!waited) {
    pdl_wait();
    pdl_trigger();
  }
}

template <int TYPE, int NB, int R, int NW>
__global__ void __launch_bounds__((NW + 1) * 32, NW == 8 ? 2 : 1) gemv_kernel(const __grid_constant__ GemvParams p) {
  extern __shared__ __align__(128) uint8_t smem[];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  if (tid == 0) {
    KT_KIND(p.trace, KT_GEMV);
    KT_FIRST(p.trace, 1);
  }
  constexpr bool SUMS = Frag<TYPE>::kNeedSums;
  // layout: [full bars][empty bars][red NB*NW][kpart][grid 2KB][xs][stages]
  uint64_t* full = (uint64_t*)smem;
  uint64_t* empty = full + GEMV_MAX_STAGES;
  float* red = (float*)(empty + GEMV_MAX_STAGES);   // [NB][NW] partial sums of x^2
  float* kpart = red + 128;                         // [NB][8][64] K-group partial row sums
  uint2* grid = (uint2*)(kpart + NB * 8 * 64);
  float* xs = (float*)(grid + 256);
  uint8_t* stage0 = (uint8_t*)(((uintptr_t)(xs + NB * p.nkc * GEMV_CHUNK) + 127) & ~(uintptr_t)127);
  const int stage_bytes = p.stage_bytes;

  if (tid == 0) {
    for (int s = 0; s < p.stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], NW);
    }
    fence_mbar_init();
  }
  __syncthreads();

  const int G = gridDim.x;
  const int n_items = (p.ntiles - (int)blockIdx.x + G - 1) / G;   // one item = one tile, all of K
  const bool paired = (p.epi == EPI_SWIGLU);

  if (warp == NW) {
    gemv_producer(p, full, empty, stage0, lane, n_items);
    return;
  }

  // ---------------- consumer warps ----------------
  pdl_wait();
  if (tid == 0) {
    KT_FIRST(p.trace, 2);
    KT_LAST(p.trace, 3);
  }
  if (TYPE == T_IQ2_XXS) {
    for (int i = tid; i < 256; i += NW * 32) {
      const uint64_t g = c_iq2xxs_grid_init[i];
      grid[i] = make_uint2((uint32_t)g, (uint32_t)(g >> 32));
    }
  }
  gemv_prologue<TYPE, NW>(p, xs, red, tid);
  if (tid == 0) KT_LAST(p.trace, 4);
  // per-column factor applied to the row dots (1/rms for RMSNorm, else 1)
  float colscale[NB];
#pragma unroll
  for (int b = 0; b < NB; ++b) {
    colscale[b] = 1.0f;
    if (p.pro == PRO_RMSNORM && b < p.nb) {
      float ss = 0.f;
#pragma unroll
      for (int i = 0; i < NW; ++i) ss += red[b * NW + i];
      colscale[b] = 1.0f / sqrtf(ss / (float)p.inner + p.eps);
    }
  }

  // warp -> (row group wr, K group wk); the tile's rows are wr*R + r
  const int nwr = NW / p.nkg;
  const int wr = warp % nwr, wk = warp / nwr;
  float best_v[NB];
  int best_i[NB];
#pragma unroll
  for (int b = 0; b < NB; ++b) { best_v[b] = -INFINITY; best_i[b] = 0x7fffffff; }
  const int x0 = Frag<TYPE>::xpos(lane, 0);
  const int blk_mask = ~(qk_of(TYPE) == 256 ? 255 : 31);

  for (int it = 0; it < n_items; ++it) {
    const int s = it % p.stages;
    if (!mbar_wait(&full[s], (it / p.stages) & 1, p.err)) return;
    if (tid == 0 && it == 0) KT_LAST(p.trace, 5);
    int sg, row0;
    tile_locate(p, blockIdx.x + it * G, sg, row0);
    const uint8_t* st = stage0 + (long long)s * stage_bytes;
    // shared-memory address of each of this warp's rows
    const uint8_t* rp[R];
#pragma unroll
    for (int r = 0; r < R; ++r) {
      const int sgr = paired ? (r < R / 2 ? 0 : 1) : sg;
      const int rrel = paired ? wr * (R / 2) + (r % (R >= 2 ? R / 2 : 1)) : wr * R + r;
      const uint32_t mis = (uint32_t)((uintptr_t)seg_row_ptr(p, sgr, row0) & 15);
      rp[r] = st + ((paired && sgr) ? p.part1_off : 0) + mis + (long long)rrel * p.row_bytes;
    }
    float acc[NB][R];
#pragma unroll
    for (int b = 0; b < NB; ++b)
#pragma unroll
      for (int r = 0; r < R; ++r) acc[b][r] = 0.f;
    const bool skip_tile = seg_skipped(p, sg, row0);
    for (int kc = wk; kc < p.nkc && !skip_tile; kc += p.nkg) {
      const int ce = min(GEMV_CHUNK, p.inner - kc * GEMV_CHUNK);
      if ((x0 & blk_mask) >= ce) continue;
      const long long coff = (long long)kc * (GEMV_CHUNK / qk_of(TYPE)) * bb_of(TYPE);
#pragma unroll
      for (int b = 0; b < NB; ++b) {
        if (b >= p.nb) break;
        f2_t xv[16];
        const float4* xb = (const float4*)(xs + ((long long)b * p.nkc + kc) * GEMV_CHUNK) + lane;
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          const ulonglong2 v = *(const ulonglong2*)(xb + k * 32);
          xv[2 * k] = v.x;
          xv[2 * k + 1] = v.y;
        }
        float xs_lo = 0.f, xs_hi = 0.f;
        if (SUMS) {
          // lo run = slots 0..15, hi run = slots 16..31 of the fragment
          f2_t a0 = xv[0], a1 = xv[8];
#pragma unroll
          for (int k = 1; k < 8; ++k) {
            a0 = fadd2(a0, xv[k]);
            a1 = fadd2(a1, xv[8 + k]);
          }
          xs_lo = hsum2(a0);
          xs_hi = hsum2(a1);
        }
#pragma unroll
        for (int r = 0; r < R; ++r) {
          float v;
          if constexpr (TYPE == T_IQ2_XXS) v = Frag<T_IQ2_XXS>::dot_grid(rp[r] + coff, lane, xv, grid);
          else v = Frag<TYPE>::dot(rp[r] + coff, lane, xv, xs_lo, xs_hi);
          acc[b][r] += v;
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);

    // ---- reduce the tile's rows: lanes, then K groups through smem ----
    const int myrow = reduce_row_of<R>(lane);
    const bool writer = reduce_writer<R>(lane);
    float tot[NB];
#pragma unroll
    for (int b = 0; b < NB; ++b) tot[b] = (b < p.nb) ? reduce_rows<R>(acc[b], lane) : 0.f;
    if (p.nkg > 1) {
      if (wk > 0 && writer)
#pragma unroll
        for (int b = 0; b < NB; ++b) kpart[(b * 8 + wk) * 64 + wr * R + myrow] = tot[b];
      named_bar_sync(2, NW * 32);
      if (wk == 0 && writer)
#pragma unroll
        for (int b = 0; b < NB; ++b)
          for (int g = 1; g < p.nkg; ++g) tot[b] += kpart[(b * 8 + g) * 64 + wr * R + myrow];
      named_bar_sync(2, NW * 32);   // kpart reused by the next tile
    }
    if (wk != 0) continue;
#pragma unroll
    for (int b = 0; b < NB; ++b) {
      if (b >= p.nb) break;
      const float t = tot[b] * colscale[b];
      if (paired) {
        // rows r < R/2 are gate rows, r >= R/2 the matching up rows
        const float other = __shfl_xor_sync(0xffffffffu, t, 16);
        const int row = row0 + wr * (R / 2) + (R >= 2 ? myrow % (R >= 2 ? R / 2 : 1) : 0);
        if (writer && myrow < R / 2 && row < p.seg[0].rows) {
          const float sg_ = t / (1.0f + expf(-t));      // mlp_forward (src/ModelCPU.jl:455-468)
          p.seg[0].y[(long long)b * p.y_stride + row] = sg_ * other;
        }
      } else {
        const int row = row0 + wr * R + myrow;
        if (writer && row < p.seg[sg].rows) {
          if (p.epi == EPI_ARGMAX) {
            if (t > best_v[b] || (t == best_v[b] && row < best_i[b])) { best_v[b] = t; best_i[b] = row; }
            if (p.seg[sg].y) p.seg[sg].y[(long long)b * p.y_stride + row] = t;
          } else {
            float* y = p.seg[sg].y + (long long)b * p.y_stride + row;
            if (p.epi == EPI_ADD) *y += t;
            else *y = t;
          }
        }
      }
    }
  }
  if (tid == 0) KT_LAST(p.trace, 6);
  if (p.epi == EPI_ARGMAX && wk == 0) {
#pragma unroll
    for (int b = 0; b < NB; ++b) {
      if (b >= p.nb) break;
      // warp-level first-max, then one atomic per warp
      float v = best_v[b];
      int i = best_i[b];
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, v, o);
        const int oi = __shfl_xor_sync(0xffffffffu, i, o);
        if (ov > v || (ov == v && oi < i)) { v = ov; i = oi; }
      }
      if (lane == 0 && i != 0x7fffffff) {
        const unsigned long long key = ((unsigned long long)float_ordered(v) << 32) |
                                       (unsigned long long)(0xffffffffu - (uint32_t)(i + p.argmax_row0));
        atomicMax(&p.argmax[b], key);
      }
    }
  }
}

}  // namespace inf
