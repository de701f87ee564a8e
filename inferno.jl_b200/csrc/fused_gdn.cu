// Fused [in_proj | attn_gate] GEMV + Gated DeltaNet step for one decode token
// (GatedDeltaNetCPU, Inferno.jl src/ModelCPU.jl:531-700, when every value
// head has its own q/k group, nk == nv).
//
// A thread-block cluster of 8 CTAs per head h.  At finalize the engine
// regroups the head's 512 projection rows as [q_h | k_h | v_h | z_h]
// (128 each); CTA j of the cluster computes rows [64j, 64j+64) with the
// integer tensor-core tile of gemv_mma.cuh (RMSNorm prologue fused) and
// stores them into the shared memory of all 8 CTAs (st.shared::cluster).  After
// one hardware cluster barrier every CTA holds the head's q, k, v, z rows and
// runs the delta-rule update for its 16 state rows (as gdn_step_kernel: conv
// over the ring, SiLU, alpha/beta from the normalised x already staged by the
// GEMV prologue, Float64 gates, L2 norms).  z goes to global memory for the
// ssm_out prologue.  Compared with the two kernels it replaces, the qkv round
// trip through L2, one launch and one dependency release disappear.
#include "internal.h"
#include "gemv_mma.cuh"
#include "params.h"
#include "../../include/inferno_b200.h"

namespace inf {

constexpr int FG_NW = 16;
constexpr int FG_THREADS = (FG_NW + 1) * 32;
constexpr int FG_CLUSTER = 8;
constexpr int FG_DK = 128;
constexpr int FG_ROWS = 16;          // state rows per CTA (128 / 8)
constexpr int FG_MAXK = 4;

__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\nbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ void st_cluster_f32(const float* local, uint32_t cta, float v) {
  uint32_t remote;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(smem_u32(local)), "r"(cta));
  asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(remote), "f"(v) : "memory");
}

struct FusedGdnArgs {
  float* z;        // [nv][dv] gate input of the ssm_out prologue
};

__global__ void __launch_bounds__(FG_THREADS, 1) fused_inproj_gdn_kernel(const __grid_constant__ GemvParams p,
                                                                         const __grid_constant__ GdnParams g,
                                                                         FusedGdnArgs fa) {
  extern __shared__ __align__(128) uint8_t smem[];
  constexpr int NW = FG_NW;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int h = blockIdx.x / FG_CLUSTER, j = blockIdx.x % FG_CLUSTER;   // cluster = head, rank j
  const int H = p.inner, nsb = H >> 8, K = g.K, C = g.C;
  // layout: [full][empty][red 2NW+4][vmax 16][kpart NW*16][xsum][xf][xq][exch 512][gdn scratch 64][wa][wb][stage]
  uint64_t* full = (uint64_t*)smem;
  uint64_t* empty = full + GEMV_MAX_STAGES;
  float* red = (float*)(empty + GEMV_MAX_STAGES);
  float* vmax = red + 2 * NW + 4;
  float* kpart = vmax + 16;
  float* xsum = kpart + NW * 16;
  float* xf = xsum + nsb * 16;
  uint8_t* xq = (uint8_t*)(xf + H);
  float* exch = (float*)(xq + (size_t)nsb * 8 * MMA_KS_BYTES);    // [q 128 | k 128 | v 128 | z 128]
  float* gs = exch + 512;                                           // qn[128] kn[128] vrow[16] red[20] gate[2]
  float* qn = gs;
  float* kn = gs + 128;
  float* vrow = gs + 256;
  float* gred = gs + 272;
  float* wa_s = gs + 304;
  float* wb_s = wa_s + H;
  uint8_t* stage0 = (uint8_t*)(((uintptr_t)(wb_s + H) + 127) & ~(uintptr_t)127);

  if (tid == 0) {
    mbar_init(&full[0], 1);
    mbar_init(&empty[0], NW);
    fence_mbar_init();
    *(volatile int*)&red[2 * NW] = 0;
  }
  if (tid < 16) vmax[tid] = 0.f;
  // ---- pre-wait: GDN state, conv taps and ring history, alpha/beta rows ----
  for (int i = tid * 4; i < H; i += FG_THREADS * 4) {
    *(float4*)&wa_s[i] = *(const float4*)&g.w_alpha[(long long)h * H + i];
    *(float4*)&wb_s[i] = *(const float4*)&g.w_beta[(long long)h * H + i];
  }
  const int t = *g.step;                 // this layer's step (written by its previous token)
  const int cur = t % K;
  const int cq = h * FG_DK + tid, ck = g.nk * FG_DK + h * FG_DK + tid;   // nk == nv: group == head
  const int cv = 2 * g.nk * FG_DK + h * g.dv + FG_ROWS * j + tid;
  float wq[FG_MAXK], wk[FG_MAXK], wv[FG_MAXK], hq[FG_MAXK], hk[FG_MAXK], hv[FG_MAXK];
  float4 srow[4];
  if (tid < 128) {
#pragma unroll
    for (int k = 0; k < FG_MAXK; ++k) {
      wq[k] = wk[k] = wv[k] = hq[k] = hk[k] = hv[k] = 0.f;
      if (k < K) {
        int slot = (t - (K - 1) + k) % K;
        if (slot < 0) slot += K;
        wq[k] = g.conv_w[(long long)cq * K + k];
        wk[k] = g.conv_w[(long long)ck * K + k];
        if (k < K - 1) {
          hq[k] = g.ring[(long long)slot * C + cq];
          hk[k] = g.ring[(long long)slot * C + ck];
        }
        if (tid < FG_ROWS) {
          wv[k] = g.conv_w[(long long)cv * K + k];
          if (k < K - 1) hv[k] = g.ring[(long long)slot * C + cv];
        }
      }
    }
#pragma unroll
    for (int r = 0; r < 4; ++r)
      srow[r] = *((const float4*)(g.S + ((long long)h * g.dv + FG_ROWS * j + warp + 4 * r) * FG_DK) + lane);
  }
  __syncthreads();

  if (warp == NW) {
    gemv_producer<false>(p, full, empty, stage0, lane, 1);
  } else {
    // ---- the projection tile: rows [64j, 64j + 64) of head h ----
    pdl_wait();
    const float colscale = gemv_mma_prologue<T_Q4_K, NW, MMA_PLAIN>(p, xf, xq, xsum, red, vmax, tid);
    const bool nonfinite = *(volatile int*)&red[2 * NW] != 0;
    const float fscale =
        nonfinite ? __int_as_float(0x7fc00000) : colscale * mma_pow2(-mma_exp2_scale(vmax[0]));
    const int nkg = NW / 4, rg = warp % 4, wk = warp / 4;     // TR = 64: 4 row groups x 4 K groups
    const int gq = lane >> 2, c = lane & 3;
    const float limbw = c == 0 ? 1.0f : c == 1 ? 256.0f : c == 2 ? 65536.0f : 16777216.0f;
    bool ok = mbar_wait(&full[0], 0, p.err);
    float acc[2] = {0.f, 0.f}, corr[2] = {0.f, 0.f};
    if (ok) {
      const uint8_t* ra = stage0 + (long long)(rg * 16 + gq) * p.row_bytes;
      const uint8_t* rb = ra + 8ll * p.row_bytes;
      for (int sb = wk; sb < nsb; sb += nkg)
        mma_sb_q4k(ra + sb * 144, rb + sb * 144, xq + (size_t)sb * 8 * MMA_KS_BYTES, xsum + sb * 8, lane, acc, corr);
    }
    float ta = limbw * acc[0] - corr[0], tb = limbw * acc[1] - corr[1];
    ta += __shfl_xor_sync(0xffffffffu, ta, 1);
    tb += __shfl_xor_sync(0xffffffffu, tb, 1);
    ta += __shfl_xor_sync(0xffffffffu, ta, 2);
    tb += __shfl_xor_sync(0xffffffffu, tb, 2);
    if (wk > 0 && c == 0) {
      kpart[(wk * 4 + rg) * 16 + gq] = ta;
      kpart[(wk * 4 + rg) * 16 + gq + 8] = tb;
    }
    named_bar_sync(2, NW * 32);
    if (wk == 0 && c == 0) {
      for (int k = 1; k < nkg; ++k) {
        ta += kpart[(k * 4 + rg) * 16 + gq];
        tb += kpart[(k * 4 + rg) * 16 + gq + 8];
      }
      ta *= fscale;
      tb *= fscale;
      const int r0 = 64 * j + rg * 16 + gq;          // head-local row of ta (tb: + 8)
#pragma unroll
      for (int q = 0; q < FG_CLUSTER; ++q) {
        st_cluster_f32(exch + r0, q, ta);
        st_cluster_f32(exch + r0 + 8, q, tb);
      }
      if (r0 >= 384) {                               // z rows: the ssm_out prologue reads them
        fa.z[(long long)h * g.dv + r0 - 384] = ta;
        fa.z[(long long)h * g.dv + r0 + 8 - 384] = tb;
      }
    }
  }
  cluster_sync_all();
  if (tid >= 128) return;

  // ---- the GDN step for state rows [16j, 16j + 16) of head h (warps 0-3) ----
  float acc3[3] = {0.f, 0.f, 0.f};
  for (int i = tid; i < H; i += 128) {               // xf = x * attn_norm (unscaled)
    const float xw = xf[i];
    acc3[1] = fmaf(wa_s[i], xw, acc3[1]);
    acc3[2] = fmaf(wb_s[i], xw, acc3[2]);
  }
  const float nq = exch[tid], nk_ = exch[128 + tid];
  const float nv_ = tid < FG_ROWS ? exch[256 + FG_ROWS * j + tid] : 0.f;
  float vq = 0.f, vk = 0.f, vvv = 0.f;
#pragma unroll
  for (int k = 0; k < FG_MAXK; ++k) {
    if (k < K - 1) {
      vq += hq[k] * wq[k];
      vk += hk[k] * wk[k];
      vvv += hv[k] * wv[k];
    } else if (k == K - 1) {
      vq += nq * wq[k];
      vk += nk_ * wk[k];
      vvv += nv_ * wv[k];
    }
  }
  const float qv = vq / (1.0f + expf(-vq));
  const float kv = vk / (1.0f + expf(-vk));
  if (tid < FG_ROWS) vrow[tid] = vvv / (1.0f + expf(-vvv));
  // ring: this step's inputs in slot t % K (q/k channels by CTA 0 of the head)
  if (j == 0) {
    g.ring[(long long)cur * C + cq] = nq;
    g.ring[(long long)cur * C + ck] = nk_;
  }
  if (tid < FG_ROWS) g.ring[(long long)cur * C + cv] = nv_;
  float b5[5] = {0.f, acc3[1], acc3[2], qv * qv, kv * kv};
#pragma unroll
  for (int i = 1; i < 5; ++i) b5[i] = warp_sum(b5[i]);
  if (lane == 0)
#pragma unroll
    for (int i = 1; i < 5; ++i) gred[i * 4 + warp] = b5[i];
  named_bar_sync(3, 128);
#pragma unroll
  for (int i = 1; i < 5; ++i) b5[i] = (gred[i * 4] + gred[i * 4 + 1]) + (gred[i * 4 + 2] + gred[i * 4 + 3]);
  // colscale is 1/rms(x) of the same RMSNorm (src/ModelCPU.jl:110-122)
  float scale;
  {
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < FG_NW; ++i) ss += red[i];
    scale = 1.0f / sqrtf(ss / (float)H + p.eps);
  }
  const float alpha = b5[1] * scale, beta_raw = b5[2] * scale;
  double a = (double)alpha + (double)g.dt_bias[h];         // src/ModelCPU.jl:618-636 in Float64
  a = fmin(20.0, fmax(-20.0, a));
  const double sp = log(1.0 + exp(a));
  const float dec = expf((float)((double)g.ssm_a[h] * sp));
  const double bv = fmin(20.0, fmax(-20.0, (double)beta_raw));
  const float bg = (float)(1.0 / (1.0 + exp(-bv)));
  const float qnv = 1.0f / (sqrtf(b5[3]) + 1.0e-6f) * (1.0f / sqrtf((float)FG_DK));
  const float knv = 1.0f / (sqrtf(b5[4]) + 1.0e-6f);
  qn[tid] = qv * qnv;
  kn[tid] = kv * knv;
  named_bar_sync(3, 128);
  const float4 k4 = *(const float4*)&kn[lane * 4];
  const float4 q4 = *(const float4*)&qn[lane * 4];
#pragma unroll
  for (int r = 0; r < 4; ++r) {
    const int rr = warp + 4 * r, i = FG_ROWS * j + rr;
    float4 s = srow[r];
    s.x *= dec; s.y *= dec; s.z *= dec; s.w *= dec;
    const float sk = warp_sum(s.x * k4.x + s.y * k4.y + s.z * k4.z + s.w * k4.w);
    const float d = bg * (vrow[rr] - sk);
    s.x += d * k4.x; s.y += d * k4.y; s.z += d * k4.z; s.w += d * k4.w;
    const float yv = warp_sum(s.x * q4.x + s.y * q4.y + s.z * q4.z + s.w * q4.w);
    *((float4*)(g.S + ((long long)h * g.dv + i) * FG_DK) + lane) = s;
    if (lane == 0) g.y[h * g.dv + i] = yv;
  }
  // the layer's step counter: the last CTA of the grid advances it
  named_bar_sync(3, 128);
  if (tid == 0) {
    __threadfence();
    const int prev = atomicAdd(g.done, 1);
    if (prev == (int)gridDim.x - 1) {
      *g.done = 0;
      *g.step = t + 1;
      __threadfence();
    }
  }
}

size_t fused_gdn_smem(int H) {
  const int nsb = H / 256;
  size_t b = 16 * GEMV_MAX_STAGES + (2 * FG_NW + 4 + 16) * 4 + FG_NW * 16 * 4 + (size_t)nsb * 16 * 4 + (size_t)H * 4 +
             (size_t)nsb * 8 * MMA_KS_BYTES + 512 * 4 + 304 * 4 + 2 * (size_t)H * 4 + 128;
  return b + ((size_t)64 * nsb * 144 + 48 + 127) / 128 * 128;     // one 64-row Q4_K tile (stage_bytes)
}

int launch_fused_inproj_gdn(const void* Wperm, int H, const float* x, const float* attn_norm, float eps,
                            const GdnParams& g, float* z, int* err, cudaStream_t st, bool pdl) {
  if (g.nk != g.nv || g.dv != FG_DK || g.K < 1 || g.K > FG_MAXK || H % 256 || H > 8192)
    return set_error(INFERNO_EINVAL, "fused in_proj + GDN: unsupported shape");
  GemvParams p{};
  const int nsb = H / 256;
  p.seg[0].W = (const uint8_t*)Wperm;
  p.seg[0].rows = g.nv * 512;
  p.seg[0].tile0 = 0;
  p.nseg = 1;
  p.ntiles = g.nv * FG_CLUSTER;
  p.inner = H;
  p.row_bytes = nsb * 144;
  p.nkc = (H + GEMV_CHUNK - 1) / GEMV_CHUNK;
  p.TR = 64;
  p.nkg = 4;
  p.nb = 1;
  p.x = x;
  p.x_stride = H;
  p.pro = PRO_RMSNORM;
  p.pro_w = attn_norm;
  p.eps = eps;
  p.epi = EPI_STORE;
  p.err = err;
  p.l2_evict_first = 1;
  p.stages = 1;
  p.contig = 1;
  p.stage_bytes = (int)(((size_t)64 * p.row_bytes + 48 + 127) / 128 * 128);
  p.nxv = 1;
  p.xch_wk = p.xch_rk = -1;
  const size_t smem = fused_gdn_smem(H);
  static DeviceOnce once;
  cudaError_t ea = once.run([] {
    return cudaFuncSetAttribute(fused_inproj_gdn_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
  });
  if (ea != cudaSuccess) return set_error(INFERNO_ECUDA, "fused in_proj + GDN attribute: %s", cudaGetErrorString(ea));
  FusedGdnArgs fa{z};
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(g.nv * FG_CLUSTER);
  cfg.blockDim = dim3(FG_THREADS);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute at[2];
  at[0].id = cudaLaunchAttributeClusterDimension;
  at[0].val.clusterDim.x = FG_CLUSTER;
  at[0].val.clusterDim.y = 1;
  at[0].val.clusterDim.z = 1;
  at[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = pdl ? 2 : 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, fused_inproj_gdn_kernel, p, g, fa);
  return e == cudaSuccess ? 0 : set_error(INFERNO_ECUDA, "fused in_proj + GDN launch: %s", cudaGetErrorString(e));
}

}  // namespace inf
