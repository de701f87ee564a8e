// Persistent decode kernel: a whole greedy decode loop in one cooperative
// launch.
//
// The per-token work of Inferno.jl's forward_cpu! (src/ModelCPU.jl:945-989:
// embedding, 24 DecoderLayerCPU calls, final RMSNorm, lm_head, argmax) is a
// fixed program of "stages": per GDN layer [in_proj|attn_gate GEMV], GDN step,
// ssm_out GEMV, ffn gate/up GEMV, ffn_down GEMV; per attention layer
// [wq|wk|wv GEMV], attention, wo GEMV, ffn gate/up, ffn_down; then lm_head.
// One CTA per SM runs every stage; stages are separated by a grid barrier
// (the data dependence of RMSNorm / attention on complete vectors).
//
// Why: at batch 1 every stage moves 1-5 MB, which HBM delivers in < 1 us, so
// separate kernels are bound by launch, dependency release and weight-fetch
// latency (~6 us each, measured).  Here
//   * a producer warp walks the same stage program ahead of the consumers and
//     streams each CTA's weight tiles of the coming stages into a ring of
//     shared-memory slots with 1-D TMA bulk copies (L2 evict_first), bounded
//     only by free slots -- so weights for stage s+1 arrive while stage s
//     computes or waits at the barrier;
//   * 16 consumer warps compute the stage from shared memory (the GEMV tile
//     decoders of gemv.cuh; the GDN and attention bodies of gdn.cu / attn.cu
//     restated for thread subsets of this CTA);
//   * the token loop (argmax -> next token -> embedding) runs on the device:
//     every CTA derives the next token from the lm_head's packed argmax and
//     dequantizes the embedding row itself.
// Activations written by other CTAs are read with ld.global.cg (L2), since L1
// is not coherent within one launch.  Every spin (grid barrier, mbarriers) is
// bounded; on timeout the kernel records an error and all CTAs leave.
#include <algorithm>
#include <climits>
#include "internal.h"
#include "gemv.cuh"
#include "params.h"
#include "persist.h"
#include "../../include/inferno_b200.h"

namespace inf {

constexpr int PK_NW = 16;                     // consumer warps
constexpr int PK_THREADS = (PK_NW + 1) * 32;  // + producer warp
constexpr int PK_NSLOT = 5;                   // weight ring slots
constexpr int PK_GDN_ROWS = 16;
constexpr int PK_DK = 128;
constexpr int PK_HD = 256;

__device__ __forceinline__ float ldcg(const float* p) { return __ldcg(p); }

// bounded grid barrier over the consumer warps of all CTAs (monotonic counter)
__device__ __forceinline__ bool grid_barrier(unsigned* counter, unsigned target, int* abort_flag, int* err) {
  named_bar_sync(1, PK_NW * 32);
  __shared__ int s_ok;
  if (threadIdx.x == 0) {
    __threadfence();
    atomicAdd(counter, 1u);
    int ok = 1;
    unsigned v;
    for (unsigned it = 0;; ++it) {
      asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(counter) : "memory");
      if (v >= target) break;
      if (*(volatile int*)abort_flag) { ok = 0; break; }
      if (it > (1u << 24)) {
        atomicExch(err, DERR_MBAR_TIMEOUT);
        atomicExch(abort_flag, 1);
        ok = 0;
        break;
      }
      if (it > 64) __nanosleep(32);
    }
    s_ok = ok;
  }
  named_bar_sync(1, PK_NW * 32);
  return s_ok;
}

// ---------------------------------------------------------------------------
// GEMV stage: consumer side (prologue from L2, tiles from the ring)
// ---------------------------------------------------------------------------
template <int TYPE>
__device__ void pk_prologue(const PkStage& S, const float* xsrc, float* xs, float* red, int tid) {
  const GemvParams& p = S.g;
  const int n = p.inner, lane = tid & 31, w = tid >> 5;
  constexpr int NT = PK_NW * 32;
  if (p.pro == PRO_RMSNORM) {
    float ss = 0.f;
    for (int i = tid; i < n; i += NT) {
      const float v = S.embed_row ? xsrc[i] : ldcg(xsrc + i);
      ss = fmaf(v, v, ss);
      xs[xperm<TYPE>(i)] = v * p.pro_w[i];
    }
    ss = warp_sum(ss);
    if (lane == 0) red[w] = ss;
  } else if (p.pro == PRO_HEADNORM_GATE) {
    const int G = p.pro_group, per = G >> 5;
    for (int hh = w; hh < n / G; hh += PK_NW) {
      float yv[8], zv[8], wv[8];
      float ss = 0.f;
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        const bool ok = q < per;
        const int i = hh * G + q * 32 + lane;
        yv[q] = ok ? ldcg(xsrc + i) : 0.f;
        zv[q] = ok ? ldcg(p.pro_z + i) : 0.f;
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
        xs[xperm<TYPE>(hh * G + q * 32 + lane)] = v * zv[q] * (1.0f / (1.0f + expf(-zv[q])));
      }
    }
  } else {
    for (int i = tid; i < n; i += NT) xs[xperm<TYPE>(i)] = ldcg(xsrc + i);
  }
  named_bar_sync(1, NT);
}

struct PkRing {
  uint64_t* full;
  uint64_t* empty;
  uint8_t* slots;
  unsigned gi;     // global item counter (same sequence in producer and consumers)
};

template <int TYPE, int R>
__device__ bool pk_gemv_tiles(const PkStage& S, PkRing& rg, const float* xs, const float* red, float* kpart,
                              const uint2* grid, int* err, unsigned long long* best_key, unsigned long long* trp) {
  const GemvParams& p = S.g;
  constexpr bool SUMS = Frag<TYPE>::kNeedSums;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int G = gridDim.x;
  const int n_items = (p.ntiles - (int)blockIdx.x + G - 1) / G;
  const bool paired = p.epi == EPI_SWIGLU;
  float colscale = 1.0f;
  if (p.pro == PRO_RMSNORM) {
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < PK_NW; ++i) ss += red[i];
    colscale = 1.0f / sqrtf(ss / (float)p.inner + p.eps);
  }
  const int nwr = PK_NW / p.nkg;
  const int wr = warp % nwr, wk = warp / nwr;
  const int x0 = Frag<TYPE>::xpos(lane, 0);
  const int blk_mask = ~(qk_of(TYPE) == 256 ? 255 : 31);
  float best_v = -INFINITY;
  int best_i = 0x7fffffff;
  for (int it = 0; it < n_items; ++it, ++rg.gi) {
    const int s = rg.gi % PK_NSLOT;
    if (!mbar_wait(&rg.full[s], (rg.gi / PK_NSLOT) & 1, err)) return false;
    if (trp && it == 0) trp[2] = clock64();
    int sg, row0;
    tile_locate(p, blockIdx.x + it * G, sg, row0);
    const uint8_t* st = rg.slots + (size_t)s * S.slot_bytes;
    const uint8_t* rp[R];
#pragma unroll
    for (int r = 0; r < R; ++r) {
      const int sgr = paired ? (r < R / 2 ? 0 : 1) : sg;
      const int rrel = paired ? wr * (R / 2) + (r % (R / 2)) : wr * R + r;
      const uint32_t mis = (uint32_t)((uintptr_t)(p.seg[sgr].W + (long long)row0 * p.row_bytes) & 15);
      rp[r] = st + ((paired && sgr) ? p.part1_off : 0) + mis + (long long)rrel * p.row_bytes;
    }
    float acc[R];
#pragma unroll
    for (int r = 0; r < R; ++r) acc[r] = 0.f;
    for (int kc = wk; kc < p.nkc; kc += p.nkg) {
      const int ce = min(GEMV_CHUNK, p.inner - kc * GEMV_CHUNK);
      if ((x0 & blk_mask) >= ce) continue;
      const long long coff = (long long)kc * (GEMV_CHUNK / qk_of(TYPE)) * bb_of(TYPE);
      f2_t xv[16];
      const float4* xb = (const float4*)(xs + (long long)kc * GEMV_CHUNK) + lane;
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const ulonglong2 v = *(const ulonglong2*)(xb + k * 32);
        xv[2 * k] = v.x;
        xv[2 * k + 1] = v.y;
      }
      float xs_lo = 0.f, xs_hi = 0.f;
      if (SUMS) {
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
        acc[r] += v;
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&rg.empty[s]);
    const int myrow = reduce_row_of<R>(lane);
    const bool writer = reduce_writer<R>(lane);
    float tot = reduce_rows<R>(acc, lane);
    if (p.nkg > 1) {
      if (wk > 0 && writer) kpart[wk * 64 + wr * R + myrow] = tot;
      named_bar_sync(2, PK_NW * 32);
      if (wk == 0 && writer)
        for (int g = 1; g < p.nkg; ++g) tot += kpart[g * 64 + wr * R + myrow];
      named_bar_sync(2, PK_NW * 32);
    }
    if (wk != 0) continue;
    const float t = tot * colscale;
    if (paired) {
      const float other = __shfl_xor_sync(0xffffffffu, t, 16);
      const int row = row0 + wr * (R / 2) + (myrow % (R / 2));
      if (writer && myrow < R / 2 && row < p.seg[0].rows) {
        const float sg_ = t / (1.0f + expf(-t));      // mlp_forward (src/ModelCPU.jl:455-468)
        p.seg[0].y[row] = sg_ * other;
      }
    } else {
      const int row = row0 + wr * R + myrow;
      if (writer && row < p.seg[sg].rows) {
        if (p.epi == EPI_ARGMAX) {
          if (t > best_v || (t == best_v && row < best_i)) { best_v = t; best_i = row; }
          if (p.seg[sg].y) p.seg[sg].y[row] = t;
        } else {
          float* y = p.seg[sg].y + row;
          if (p.epi == EPI_ADD) *y = __ldcg(y) + t;
          else *y = t;
        }
      }
    }
  }
  if (p.epi == EPI_ARGMAX && wk == 0) {
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
                                     (unsigned long long)(0xffffffffu - (uint32_t)i);
      atomicMax(best_key, key);
    }
  }
  return true;
}

template <int TYPE>
__device__ bool pk_gemv(const PkStage& S, PkRing& rg, const float* xsrc, float* xs, float* red, float* kpart,
                        const uint2* grid, int* err, unsigned long long* key, unsigned long long* trp) {
  const int tid = threadIdx.x;
  pk_prologue<TYPE>(S, xsrc, xs, red, tid);
  if (trp) trp[1] = clock64();
  return S.R == 4 ? pk_gemv_tiles<TYPE, 4>(S, rg, xs, red, kpart, grid, err, key, trp)
                  : pk_gemv_tiles<TYPE, 2>(S, rg, xs, red, kpart, grid, err, key, trp);
}

// ---------------------------------------------------------------------------
// GDN stage on warps 0..3 of the CTAs that own a (head, 16-row block) item
// (restates gdn_step_kernel for a 128-thread subset, reads via L2)
// ---------------------------------------------------------------------------
__device__ void pk_gdn(const GdnParams& p, float* sm) {
  const int tid = threadIdx.x;
  const int items = p.nv * (p.dv / PK_GDN_ROWS);
  if (tid >= 128) return;
  for (int item = blockIdx.x; item < items; item += gridDim.x) {
  const int h = item / (p.dv / PK_GDN_ROWS), r0 = (item % (p.dv / PK_GDN_ROWS)) * PK_GDN_ROWS;
  const int warp = tid >> 5, lane = tid & 31;
  const int g = h % p.nk, K = p.K, C = p.C, H = p.H;
  float* qn = sm;
  float* kn = sm + PK_DK;
  float* vrow = sm + 2 * PK_DK;
  float* red = vrow + PK_GDN_ROWS;      // [3][4]
  const int t = __ldcg(p.step);
  const int cur = t % K;
  const int cq = g * PK_DK + tid, ck = p.nk * PK_DK + g * PK_DK + tid;
  const int cv = 2 * p.nk * PK_DK + h * p.dv + r0 + tid;
  // state rows first (independent loads in flight)
  float4 srow[4];
#pragma unroll
  for (int j = 0; j < 4; ++j)
    srow[j] = __ldcg((const float4*)(p.S + ((long long)h * p.dv + r0 + warp + 4 * j) * PK_DK) + lane);
  float vq = 0.f, vk = 0.f, vvv = 0.f;
  const float nq = ldcg(p.qkv + cq), nk_ = ldcg(p.qkv + ck);
  const float nv_ = tid < PK_GDN_ROWS ? ldcg(p.qkv + cv) : 0.f;
  for (int k = 0; k < K; ++k) {
    int slot = (t - (K - 1) + k) % K;
    if (slot < 0) slot += K;
    const bool last = k == K - 1;
    vq += (last ? nq : ldcg(p.ring + (long long)slot * C + cq)) * p.conv_w[(long long)cq * K + k];
    vk += (last ? nk_ : ldcg(p.ring + (long long)slot * C + ck)) * p.conv_w[(long long)ck * K + k];
    if (tid < PK_GDN_ROWS)
      vvv += (last ? nv_ : ldcg(p.ring + (long long)slot * C + cv)) * p.conv_w[(long long)cv * K + k];
  }
  float a3[3] = {0.f, 0.f, 0.f};
  for (int i = tid; i < H; i += 128) {
    const float xv = ldcg(p.x + i);
    const float xw = xv * p.in_norm[i];
    a3[0] = fmaf(xv, xv, a3[0]);
    a3[1] = fmaf(p.w_alpha[(long long)h * H + i], xw, a3[1]);
    a3[2] = fmaf(p.w_beta[(long long)h * H + i], xw, a3[2]);
  }
  const float qv = vq / (1.0f + expf(-vq));
  const float kv = vk / (1.0f + expf(-vk));
  if (tid < PK_GDN_ROWS) vrow[tid] = vvv / (1.0f + expf(-vvv));
  if (h == g && r0 == 0) {
    p.ring[(long long)cur * C + cq] = nq;
    p.ring[(long long)cur * C + ck] = nk_;
  }
  if (tid < PK_GDN_ROWS) p.ring[(long long)cur * C + cv] = nv_;
  float b5[5] = {a3[0], a3[1], a3[2], qv * qv, kv * kv};
#pragma unroll
  for (int i = 0; i < 5; ++i) b5[i] = warp_sum(b5[i]);
  if (lane == 0)
#pragma unroll
    for (int i = 0; i < 5; ++i) red[i * 4 + warp] = b5[i];
  named_bar_sync(3, 128);
#pragma unroll
  for (int i = 0; i < 5; ++i) b5[i] = (red[i * 4] + red[i * 4 + 1]) + (red[i * 4 + 2] + red[i * 4 + 3]);
  const float scale = 1.0f / sqrtf(b5[0] / (float)H + p.eps);
  const float alpha = b5[1] * scale, beta_raw = b5[2] * scale;
  float dec, bg;
  {
    // gates in Float64 (src/ModelCPU.jl:618-636); every thread computes them
    double a = (double)alpha + (double)p.dt_bias[h];
    a = fmin(20.0, fmax(-20.0, a));
    const double sp = log(1.0 + exp(a));
    const float decay = (float)((double)p.ssm_a[h] * sp);
    dec = expf(decay);
    const double bv = fmin(20.0, fmax(-20.0, (double)beta_raw));
    bg = (float)(1.0 / (1.0 + exp(-bv)));
  }
  const float qnv = 1.0f / (sqrtf(b5[3]) + 1.0e-6f) * (1.0f / sqrtf((float)PK_DK));
  const float knv = 1.0f / (sqrtf(b5[4]) + 1.0e-6f);
  qn[tid] = qv * qnv;
  kn[tid] = kv * knv;
  named_bar_sync(3, 128);
  const float4 k4 = *(const float4*)&kn[lane * 4];
  const float4 q4 = *(const float4*)&qn[lane * 4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int rr = warp + 4 * j, i = r0 + rr;
    float4 s = srow[j];
    s.x *= dec; s.y *= dec; s.z *= dec; s.w *= dec;
    const float sk = warp_sum(s.x * k4.x + s.y * k4.y + s.z * k4.z + s.w * k4.w);
    const float d = bg * (vrow[rr] - sk);
    s.x += d * k4.x; s.y += d * k4.y; s.z += d * k4.z; s.w += d * k4.w;
    const float yv = warp_sum(s.x * q4.x + s.y * q4.y + s.z * q4.z + s.w * q4.w);
    *((float4*)(p.S + ((long long)h * p.dv + i) * PK_DK) + lane) = s;
    if (lane == 0) p.y[h * p.dv + i] = yv;
  }
  named_bar_sync(3, 128);
  if (tid == 0) {
    __threadfence();
    const int prev = atomicAdd(p.done, 1);
    if (prev == items - 1) {
      *p.done = 0;
      *p.step = t + 1;
      __threadfence();
    }
  }
  }
}

// ---------------------------------------------------------------------------
// attention stage on warps 0..7 (256 threads): item = (head, split)
// (restates attn_decode_kernel, reads via L2)
// ---------------------------------------------------------------------------
__device__ void pk_attn(const AttnParams& p, int pos, float* sm) {
  const int d = threadIdx.x;
  if (d >= 256) return;
  const int L = pos + 1;
  const int nact = (L + p.split_len - 1) / p.split_len;
  const int items = p.nh * nact;
  const int lane = d & 31, warp = d >> 5;
  float* qs = sm;
  float* knew = sm + PK_HD;
  float* vnew = sm + 2 * PK_HD;
  float* sc = sm + 3 * PK_HD;          // [32]
  float* red = sc + 32;                // [2][8]
  int* ticket = (int*)(red + 16);
  const float scale = 1.0f / sqrtf((float)PK_HD);
  for (int item = blockIdx.x; item < items; item += gridDim.x) {
    const int h = item / nact, s = item % nact;
    const int kvh = h / (p.nh / p.nkv);
    const int j0 = s * p.split_len, j1 = min(j0 + p.split_len, L);
    const bool has_new = (pos >= j0 && pos < j1);
    const float qv = ldcg(p.qg + (long long)h * 2 * PK_HD + d);
    const float kv = has_new ? ldcg(p.k + kvh * PK_HD + d) : 0.f;
    if (has_new) vnew[d] = ldcg(p.v + kvh * PK_HD + d);
    float a = warp_sum(qv * qv), b = warp_sum(kv * kv);
    if (lane == 0) { red[warp] = a; red[8 + warp] = b; }
    named_bar_sync(4, 256);
    a = 0.f;
    b = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) { a += red[i]; b += red[8 + i]; }
    const float iq = 1.0f / sqrtf(a / (float)PK_HD + p.eps);
    const float ik = 1.0f / sqrtf(b / (float)PK_HD + p.eps);
    qs[d] = qv * iq * p.q_norm[d];
    if (has_new) knew[d] = kv * ik * p.k_norm[d];
    named_bar_sync(4, 256);
    const int half = p.rd / 2;
    if (d < half) {
      const float c = p.rope_cos[(long long)pos * half + d], sn = p.rope_sin[(long long)pos * half + d];
      float x1 = qs[d], x2 = qs[d + half];
      qs[d] = x1 * c - x2 * sn;
      qs[d + half] = x1 * sn + x2 * c;
      if (has_new) {
        x1 = knew[d];
        x2 = knew[d + half];
        knew[d] = x1 * c - x2 * sn;
        knew[d + half] = x1 * sn + x2 * c;
      }
    }
    named_bar_sync(4, 256);
    if (has_new && (h % (p.nh / p.nkv)) == 0) {
      const long long off = ((long long)pos * p.nkv + kvh) * PK_HD + d;
      p.kc[off] = knew[d];
      p.vc[off] = vnew[d];
    }
    const int kk = d >> 3, part = d & 7;
    float4 q8[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) q8[i] = *(const float4*)&qs[part * 32 + 4 * i];
    float m = -INFINITY, l = 0.f, o = 0.f;
    for (int c0 = j0; c0 < j1; c0 += 32) {
      const int cend = min(c0 + 32, j1);
      const int j = c0 + kk;
      float4 kreg[8];
      if (j == pos) {
#pragma unroll
        for (int i = 0; i < 8; ++i) kreg[i] = *(const float4*)&knew[part * 32 + 4 * i];
      } else if (j < cend) {
        const float4* kr = (const float4*)(p.kc + ((long long)j * p.nkv + kvh) * PK_HD + part * 32);
#pragma unroll
        for (int i = 0; i < 8; ++i) kreg[i] = __ldcg(kr + i);
      } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) kreg[i] = make_float4(0.f, 0.f, 0.f, 0.f);
      }
      float vreg[32];
#pragma unroll
      for (int q = 0; q < 32; ++q) {
        const int jj = c0 + q;
        vreg[q] = (jj < cend && jj != pos) ? ldcg(p.vc + ((long long)jj * p.nkv + kvh) * PK_HD + d) : 0.f;
      }
      float dot = 0.f;
#pragma unroll
      for (int i = 0; i < 8; ++i)
        dot += q8[i].x * kreg[i].x + q8[i].y * kreg[i].y + q8[i].z * kreg[i].z + q8[i].w * kreg[i].w;
      dot += __shfl_xor_sync(0xffffffffu, dot, 4);
      dot += __shfl_xor_sync(0xffffffffu, dot, 2);
      dot += __shfl_xor_sync(0xffffffffu, dot, 1);
      named_bar_sync(4, 256);
      if (part == 0) sc[kk] = (j < cend) ? dot * scale : -INFINITY;
      named_bar_sync(4, 256);
      float cm = -INFINITY;
#pragma unroll
      for (int q = 0; q < 32; ++q) cm = fmaxf(cm, sc[q]);
      const float mn = fmaxf(m, cm);
      const float corr = expf(m - mn);
      l *= corr;
      o *= corr;
#pragma unroll
      for (int q = 0; q < 32; ++q) {
        const float e = expf(sc[q] - mn);
        l += e;
        o = fmaf(e, (c0 + q == pos) ? vnew[d] : vreg[q], o);
      }
      m = mn;
    }
    p.part_o[((long long)h * p.nsplit + s) * PK_HD + d] = o;
    if (d == 0) {
      p.part_ml[((long long)h * p.nsplit + s) * 2 + 0] = m;
      p.part_ml[((long long)h * p.nsplit + s) * 2 + 1] = l;
    }
    __threadfence();
    named_bar_sync(4, 256);
    if (d == 0) *ticket = atomicAdd(&p.counters[h], 1);
    named_bar_sync(4, 256);
    if (*ticket == nact - 1) {
      __threadfence();
      if (d == 0) p.counters[h] = 0;
      const float* mlp = p.part_ml + (long long)h * p.nsplit * 2;
      float M = -INFINITY;
      for (int t = 0; t < nact; ++t) M = fmaxf(M, __ldcg(mlp + 2 * t));
      float num = 0.f, den = 0.f;
      for (int t = 0; t < nact; ++t) {
        const float w = expf(__ldcg(mlp + 2 * t) - M);
        num = fmaf(w, __ldcg(p.part_o + ((long long)h * p.nsplit + t) * PK_HD + d), num);
        den = fmaf(w, __ldcg(mlp + 2 * t + 1), den);
      }
      const float g = ldcg(p.qg + (long long)h * 2 * PK_HD + PK_HD + d);
      p.out[(long long)h * PK_HD + d] = (num / den) * (1.0f / (1.0f + expf(-g)));
    }
    named_bar_sync(4, 256);
  }
}

// Q6_K / Q4_K / Q8_0 / F32 embedding row (bit-exact dequant, Dequant.jl)
__device__ void pk_embed(const PkParams& P, int tok, float* out, int tid) {
  const uint8_t* src = P.embd + (long long)tok * P.embd_row_bytes;
  const int runs = P.hidden / 32;
  for (int r = tid; r < runs; r += PK_NW * 32) {
    if (P.embd_type == T_Q6_K) {
      const long long blk = r >> 3;
      const int q = r & 7, n = q >> 2, k = q & 3;
      const uint8_t* b = src + blk * 210;
      const uint8_t* ql = b + n * 64;
      const uint8_t* qh = b + 128 + n * 32;
      const int8_t* sc = (const int8_t*)(b + 192 + n * 8);
      const float d = h2f_bits((uint16_t)(b[208] | (b[209] << 8)));
      float* o = out + blk * 256 + n * 128 + k * 32;
      for (int l = 0; l < 32; ++l) {
        const uint32_t lo = (k & 1) ? ql[l + 32] : ql[l];
        const uint32_t nib = (k >= 2) ? (lo >> 4) : (lo & 0x0fu);
        const int qv = (int)(nib | (((qh[l] >> (2 * k)) & 3u) << 4)) - 32;
        o[l] = __fmul_rn(__fmul_rn(d, (float)sc[l / 16 + 2 * k]), (float)qv);
      }
    } else if (P.embd_type == T_F32) {
      for (int j = 0; j < 32; ++j) out[r * 32 + j] = ((const float*)src)[r * 32 + j];
    } else if (P.embd_type == T_Q8_0) {
      const uint8_t* b = src + (long long)r * 34;
      const float d = h2f_bits((uint16_t)(b[0] | (b[1] << 8)));
      for (int j = 0; j < 32; ++j) out[r * 32 + j] = __fmul_rn(d, (float)(int8_t)b[2 + j]);
    } else {   // Q4_K
      const long long blk = r >> 3;
      const int q = r & 7, j = q >> 1, hi = q & 1;
      const uint8_t* b = src + blk * 144;
      const float d = h2f_bits((uint16_t)(b[0] | (b[1] << 8))), dmin = h2f_bits((uint16_t)(b[2] | (b[3] << 8)));
      const uint8_t* scb = b + 4;
      const int is = 2 * j + hi;
      uint32_t sv, mv;
      if (is < 4) { sv = scb[is] & 63u; mv = scb[is + 4] & 63u; }
      else {
        sv = (scb[is + 4] & 0x0fu) | ((scb[is - 4] >> 6) << 4);
        mv = (scb[is + 4] >> 4) | ((scb[is] >> 6) << 4);
      }
      const float d1 = __fmul_rn(d, (float)sv), mn = __fmul_rn(dmin, (float)mv);
      float* o = out + blk * 256 + j * 64 + hi * 32;
      const uint8_t* qs = b + 16 + j * 32;
      for (int l = 0; l < 32; ++l) o[l] = __fsub_rn(__fmul_rn(d1, (float)(hi ? (qs[l] >> 4) : (qs[l] & 15u))), mn);
    }
  }
}

// ---------------------------------------------------------------------------
// the kernel
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(PK_THREADS, 1) decode_persistent_kernel(const __grid_constant__ PkParams P) {
  extern __shared__ __align__(128) uint8_t smem[];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  uint64_t* full = (uint64_t*)smem;
  uint64_t* empty = full + PK_NSLOT;
  float* red = (float*)(empty + PK_NSLOT);          // 32
  float* kpart = red + 32;                          // 8*64
  float* aux = kpart + 512;                         // 1024: GDN / attention scratch
  uint2* grid = (uint2*)(aux + 1024);               // 256
  PkStage* sbuf = (PkStage*)(grid + 256);          // [2] stage descriptors (double buffer)
  float* emb = (float*)(sbuf + 2);                  // hidden (<= 8192)
  float* xs = emb + P.hidden_pad;                   // activations (<= max inner, padded to 1024)
  uint8_t* slots = (uint8_t*)(((uintptr_t)(xs + P.max_inner_pad) + 127) & ~(uintptr_t)127);

  if (tid == 0) {
    for (int s = 0; s < PK_NSLOT; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], PK_NW);
    }
    fence_mbar_init();
  }
  for (int i = tid; i < 256; i += PK_THREADS) {
    const uint64_t g = c_iq2xxs_grid_init[i];
    grid[i] = make_uint2((uint32_t)g, (uint32_t)(g >> 32));
  }
  __syncthreads();
  const int G = gridDim.x;
  const uint64_t pol = l2_policy_evict_first();

  if (warp == PK_NW) {
    // ---------------- producer: weight tiles of every GEMV stage, in order ----------------
    unsigned gi = 0;
    for (int t = 0; t < P.n_steps; ++t) {
      for (int si = 0; si < P.n_stages; ++si) {
        const PkStage& S = P.stages[si];
        if (S.kind != PK_GEMV) continue;
        const GemvParams& p = S.g;
        const bool paired = p.epi == EPI_SWIGLU;
        const int n_items = (p.ntiles - (int)blockIdx.x + G - 1) / G;
        for (int it = 0; it < n_items; ++it, ++gi) {
          const int s = gi % PK_NSLOT;
          const bool ptr = P.trace && t == 1 && it == 0 && lane == 0 && blockIdx.x == 0;
          if (ptr) P.trace[2048 + 2 * si] = clock64();
          if (gi >= PK_NSLOT && !mbar_wait(&empty[s], ((gi / PK_NSLOT) - 1) & 1, P.err)) return;
          if (*(volatile int*)P.abort_flag) return;
          if (ptr) P.trace[2048 + 2 * si + 1] = clock64();
          int sg, row0;
          tile_locate(p, blockIdx.x + it * G, sg, row0);
          uint8_t* st = slots + (size_t)s * P.slot_bytes;
          if (lane < (paired ? 2 : 1)) {
            const int sgr = paired ? lane : sg;
            const int nrows = min(paired ? p.TR / 2 : p.TR, p.seg[sgr].rows - row0);
            uint32_t bytes = 0;
            uintptr_t a0 = 0;
            if (nrows > 0) {
              const uintptr_t src = (uintptr_t)(p.seg[sgr].W + (long long)row0 * p.row_bytes);
              a0 = src & ~(uintptr_t)15;
              const uintptr_t a1 = (src + (long long)nrows * p.row_bytes + 15) & ~(uintptr_t)15;
              bytes = (uint32_t)(a1 - a0);
            }
            const uint32_t other = __shfl_down_sync(paired ? 3u : 1u, bytes, 1, paired ? 2 : 1);
            if (lane == 0) mbar_arrive_expect_tx(&full[s], bytes + (paired ? other : 0u));
            __syncwarp(paired ? 3u : 1u);
            if (bytes) tma_load_1d_hint(st + (lane ? p.part1_off : 0), (const void*)a0, bytes, &full[s], pol);
          }
        }
      }
    }
    return;
  }

  // ---------------- consumers ----------------
  // The stage descriptor is read from shared memory: descriptor fields read
  // from global memory would put dependent L2 round trips on every stage's
  // critical path.  Warp 0 loads the next descriptor into registers at the
  // start of a stage and stores it into the other buffer just before the grid
  // barrier.
  constexpr int SV = (int)((sizeof(PkStage) + 15) / 16);
  constexpr int SV_LANE = (SV + 31) / 32;
  {
    const uint4* src = (const uint4*)P.stages;
    for (int i = tid; i < SV; i += PK_NW * 32) ((uint4*)sbuf)[i] = src[i];
  }
  named_bar_sync(1, PK_NW * 32);
  unsigned sc = 0;     // running stage counter: descriptor in sbuf[sc & 1]
  PkRing rg{full, empty, slots, 0};
  unsigned nbar = 0;
  int tok = P.tok0;
  for (int t = 0; t < P.n_steps; ++t) {
    const int pos = P.pos0 + t;
    // embedding row of this token, dequantized by every CTA into smem
    pk_embed(P, tok, emb, tid);
    named_bar_sync(1, PK_NW * 32);
    if (blockIdx.x == 0)
      for (int i = tid; i < P.hidden; i += PK_NW * 32) P.x[i] = emb[i];
    for (int si = 0; si < P.n_stages; ++si, ++sc) {
      const PkStage& S = sbuf[sc & 1];
      uint4 nxt[SV_LANE];
      if (warp == 0) {
        const uint4* src = (const uint4*)(P.stages + (si + 1 < P.n_stages ? si + 1 : 0));
#pragma unroll
        for (int j = 0; j < SV_LANE; ++j)
          if (lane + 32 * j < SV) nxt[j] = src[lane + 32 * j];
      }
      const bool tr = P.trace && t == 1 && tid == 0 && (blockIdx.x == 0 || blockIdx.x == G - 1);
      unsigned long long* trp = P.trace ? P.trace + (blockIdx.x == 0 ? 0 : 4096) + 8 * si : nullptr;
      if (tr) {
        trp[0] = clock64();
        trp[5] = S.kind;
        trp[6] = S.kind == PK_GEMV ? S.g.ntiles : 0;
        trp[7] = S.kind == PK_GEMV ? S.g.TR * 100 + S.g.nkg : 0;
      }
      if (S.kind == PK_GEMV) {
        const float* xsrc = S.embed_row ? emb : S.xsrc;
        bool ok;
        switch (S.type) {
          case T_Q4_K: ok = pk_gemv<T_Q4_K>(S, rg, xsrc, xs, red, kpart, grid, P.err, P.argkey, tr ? trp : nullptr); break;
          case T_Q6_K: ok = pk_gemv<T_Q6_K>(S, rg, xsrc, xs, red, kpart, grid, P.err, P.argkey, tr ? trp : nullptr); break;
          case T_Q5_K: ok = pk_gemv<T_Q5_K>(S, rg, xsrc, xs, red, kpart, grid, P.err, P.argkey, tr ? trp : nullptr); break;
          case T_Q8_0: ok = pk_gemv<T_Q8_0>(S, rg, xsrc, xs, red, kpart, grid, P.err, P.argkey, tr ? trp : nullptr); break;
          case T_IQ2_XXS: ok = pk_gemv<T_IQ2_XXS>(S, rg, xsrc, xs, red, kpart, grid, P.err, P.argkey, tr ? trp : nullptr); break;
          default: ok = pk_gemv<T_F32>(S, rg, xsrc, xs, red, kpart, grid, P.err, P.argkey, tr ? trp : nullptr); break;
        }
        if (!ok) {
          atomicExch(P.abort_flag, 1);
          return;
        }
      } else if (S.kind == PK_GDN) {
        pk_gdn(S.d, aux);
      } else if (S.kind == PK_ATTN) {
        pk_attn(S.a, pos, aux);
      }
      if (tr) trp[3] = clock64();
      if (warp == 0) {
        uint4* dst = (uint4*)(sbuf + ((sc + 1) & 1));
#pragma unroll
        for (int j = 0; j < SV_LANE; ++j)
          if (lane + 32 * j < SV) dst[lane + 32 * j] = nxt[j];
      }
      ++nbar;
      if (!grid_barrier(P.barrier, nbar * (unsigned)G, P.abort_flag, P.err)) return;
      if (tr) trp[4] = clock64();
      // the argmax key of the previous token was read by everyone before
      // the first barrier of this token: clear it for this token's lm_head
      if (si == 0 && blockIdx.x == 0 && tid == 0) *P.argkey = 0ull;
    }
    // next token: first-max argmax of this token's logits
    const unsigned long long key = __ldcg(P.argkey);
    const int am = (int)(0xffffffffu - (uint32_t)(key & 0xffffffffull));
    if (blockIdx.x == 0 && tid == 0) {
      const int o = t - (P.n_prompt - 1);
      if (o >= 0 && o < P.max_out) P.out_tokens[o] = am;
      if (t == P.n_steps - 1) {
        P.ctl_last[0] = am;
      }
    }
    tok = (t + 1 < P.n_prompt) ? P.prompt[t + 1] : am;
    // make the argmax key reset (first barrier of the next token) safe: all
    // CTAs have read it once they pass that barrier
  }
}

// ---------------------------------------------------------------------------
// host: stage planning and launch
// ---------------------------------------------------------------------------
int pk_plan_gemv(const GemvCall& c, int slot_cap, int sms, PkStage* S) {
  const int qk = qk_of(c.type), bb = bb_of(c.type);
  const bool paired = c.epi == EPI_SWIGLU;
  const long long row_bytes = (long long)c.inner / qk * bb;
  const int nkc = (c.inner + GEMV_CHUNK - 1) / GEMV_CHUNK;
  auto tile_bytes = [&](int TR) -> size_t {
    if (paired) return 2 * (((size_t)(TR / 2) * row_bytes + 32 + 15) / 16 * 16) + 128;
    return ((size_t)TR * row_bytes + 48 + 127) / 128 * 128;
  };
  int best_r = 0, best_g = 1;
  double best = 1e300;
  for (int R : {4, 2}) {
    for (int g : {1, 2, 4, 8}) {
      if (g > nkc) continue;
      const int TR = R * PK_NW / g;
      if (TR > 64 || (paired && TR % 2)) continue;
      if (tile_bytes(TR) > (size_t)slot_cap) continue;
      const int eff = paired ? TR / 2 : TR;
      long long tiles = 0;
      for (int i = 0; i < (paired ? 1 : c.nmats); ++i) tiles += (c.mats[i].rows + eff - 1) / eff;
      const long long waves = (tiles + sms - 1) / sms;
      const double cost = (double)waves * TR * row_bytes * (R == 4 ? 1.0 : 1.1) * (1.0 + 0.04 * (g - 1));
      if (cost < best) { best = cost; best_r = R; best_g = g; }
    }
  }
  if (!best_r) return set_error(INFERNO_EINVAL, "persistent gemv: rows of %lld bytes exceed a ring slot", row_bytes);
  const int TR = best_r * PK_NW / best_g, eff = paired ? TR / 2 : TR;
  GemvParams& p = S->g;
  p = GemvParams{};
  p.xch_wk = p.xch_rk = -1;
  int ntiles = 0;
  for (int i = 0; i < c.nmats; ++i) {
    p.seg[i].W = (const uint8_t*)c.mats[i].W;
    p.seg[i].y = c.mats[i].y;
    p.seg[i].rows = c.mats[i].rows;
    if (paired && i == 1) p.seg[i].tile0 = INT_MAX;
    else {
      p.seg[i].tile0 = ntiles;
      ntiles += (c.mats[i].rows + eff - 1) / eff;
    }
  }
  p.nseg = c.nmats;
  p.ntiles = ntiles;
  p.inner = c.inner;
  p.row_bytes = (int)row_bytes;
  p.nkc = nkc;
  p.TR = TR;
  p.nkg = best_g;
  p.nb = 1;
  p.pro = c.pro;
  p.pro_w = c.pro_w;
  p.pro_z = c.pro_z;
  p.eps = c.eps;
  p.pro_group = c.pro_group;
  p.epi = c.epi;
  p.part1_off = (int)((((size_t)(TR / 2) * row_bytes + 32 + 15) / 16) * 16);
  S->kind = PK_GEMV;
  S->type = c.type;
  S->R = best_r;
  S->xsrc = c.x;
  S->slot_bytes = slot_cap;
  return 0;
}

size_t pk_smem_bytes(int hidden_pad, int max_inner_pad, int slot_bytes) {
  return 16 * PK_NSLOT + 4 * (32 + 512 + 1024) + 8 * 256 + 2 * sizeof(PkStage) + 4 * (size_t)(hidden_pad + max_inner_pad) + 128 +
         (size_t)PK_NSLOT * slot_bytes;
}

int pk_launch(const PkParams& P, size_t smem, cudaStream_t st) {
  static DeviceOnce once;
  cudaError_t ea = once.run([] {
    return cudaFuncSetAttribute(decode_persistent_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
  });
  if (ea != cudaSuccess)
    return set_error(INFERNO_ECUDA, "persistent kernel attribute: %s", cudaGetErrorString(ea));
  int dev = 0;
  cudaGetDevice(&dev);
  int per_sm = 0;
  cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, decode_persistent_kernel, PK_THREADS, smem);
  const int sms = num_sms(dev);
  if (per_sm < 1) return set_error(INFERNO_ECUDA, "persistent kernel does not fit an SM (smem %zu)", smem);
  void* args[] = {(void*)&P};
  cudaError_t e = cudaLaunchCooperativeKernel((const void*)decode_persistent_kernel, dim3(sms), dim3(PK_THREADS), args,
                                              smem, st);
  return e == cudaSuccess ? 0 : set_error(INFERNO_ECUDA, "persistent launch: %s", cudaGetErrorString(e));
}

}  // namespace inf
