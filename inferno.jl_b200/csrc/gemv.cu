// GEMV launch planner + template instantiations (see gemv.cuh for the kernel).
#include <algorithm>
#include <climits>
#include <cstdlib>
#include "internal.h"
#include "gemv.cuh"
#include "gemv_mma.cuh"
#include "gemv_mma_batch.cuh"

namespace inf {

namespace {

template <int TYPE, int NB, int R, int NW>
cudaError_t launch_one(const GemvParams& p, int grid, size_t smem, cudaStream_t st, bool pdl) {
  // one carve-out for every kernel of the engine: no L1 / shared-memory
  // reconfiguration between back-to-back launches
  static DeviceOnce once;
  cudaError_t ea = once.run([] {
    cudaError_t e = cudaFuncSetAttribute(gemv_kernel<TYPE, NB, R, NW>, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
    if (e != cudaSuccess) return e;
    return cudaFuncSetAttribute(gemv_kernel<TYPE, NB, R, NW>, cudaFuncAttributePreferredSharedMemoryCarveout,
                                cudaSharedmemCarveoutMaxShared);
  });
  if (ea != cudaSuccess) return ea;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3((NW + 1) * 32);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, gemv_kernel<TYPE, NB, R, NW>, p);
}

template <int TYPE, int NW>
cudaError_t launch_r(const GemvParams& p, int R, int grid, size_t smem, cudaStream_t st, bool pdl) {
  switch (R) {
    case 1: return launch_one<TYPE, 1, 1, NW>(p, grid, smem, st, pdl);
    case 2: return launch_one<TYPE, 1, 2, NW>(p, grid, smem, st, pdl);
    default: return launch_one<TYPE, 1, 4, NW>(p, grid, smem, st, pdl);
  }
}

template <int TYPE>
cudaError_t launch_nb(const GemvParams& p, int NB, int R, int NW, int grid, size_t smem, cudaStream_t st,
                      bool pdl) {
  switch (NB) {
    case 1: return NW == 8 ? launch_r<TYPE, 8>(p, R, grid, smem, st, pdl) : launch_r<TYPE, 16>(p, R, grid, smem, st, pdl);
    // batched columns use at most two rows per warp (the x fragments of all
    // columns are live at once; more rows would spill)
    case 4: return R == 1 ? launch_one<TYPE, 4, 1, 16>(p, grid, smem, st, pdl)
                          : launch_one<TYPE, 4, 2, 16>(p, grid, smem, st, pdl);
    default: return R == 1 ? launch_one<TYPE, 8, 1, 16>(p, grid, smem, st, pdl)
                           : launch_one<TYPE, 8, 2, 16>(p, grid, smem, st, pdl);
  }
}

template <int TYPE, int MODE, int NW>
cudaError_t launch_mma_mode(const GemvParams& p, int grid, size_t smem, cudaStream_t st, bool pdl) {
  // one carve-out for every kernel of the engine: no L1 / shared-memory
  // reconfiguration between back-to-back launches
  static DeviceOnce once;
  cudaError_t ea = once.run([] {
    cudaError_t e = cudaFuncSetAttribute(gemv_mma_kernel<TYPE, NW, MODE>, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
    if (e != cudaSuccess) return e;
    return cudaFuncSetAttribute(gemv_mma_kernel<TYPE, NW, MODE>, cudaFuncAttributePreferredSharedMemoryCarveout,
                                cudaSharedmemCarveoutMaxShared);
  });
  if (ea != cudaSuccess) return ea;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3((NW + 1) * 32);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, gemv_mma_kernel<TYPE, NW, MODE>, p);
}

template <int TYPE, int NW>
cudaError_t launch_mma_nw(const GemvParams& p, int grid, size_t smem, cudaStream_t st, bool pdl) {
  if (p.xch_wk >= 0 || p.xch_rk >= 0) return launch_mma_mode<TYPE, MMA_XCH, NW>(p, grid, smem, st, pdl);
  bool moe = p.nxv > 1;
  for (int i = 0; i < p.nseg; ++i) moe |= p.seg[i].indirect != 0;
  if (moe) return launch_mma_mode<TYPE, MMA_MOE, NW>(p, grid, smem, st, pdl);
  if (p.pro != PRO_RMSNORM && p.pro != PRO_NONE) return launch_mma_mode<TYPE, MMA_GATE, NW>(p, grid, smem, st, pdl);
  if (p.epi == EPI_SWIGLU) return launch_mma_mode<TYPE, MMA_SWIGLU, NW>(p, grid, smem, st, pdl);
  return launch_mma_mode<TYPE, MMA_PLAIN, NW>(p, grid, smem, st, pdl);
}

template <int TYPE>
cudaError_t launch_mma(const GemvParams& p, int nw, int grid, size_t smem, cudaStream_t st, bool pdl) {
  return nw == 8 ? launch_mma_nw<TYPE, 8>(p, grid, smem, st, pdl) : launch_mma_nw<TYPE, 16>(p, grid, smem, st, pdl);
}

// Integer tensor-core path (gemv_mma.cuh) for single-column Q4_K / Q6_K.
// Returns 1 when the shape does not fit it (the caller falls back).
int plan_launch_mma(const GemvCall& c, int dev, int sms, cudaStream_t st, bool pdl) {
  const int bb = bb_of(c.type);
  const bool paired = c.epi == EPI_SWIGLU;
  const int nsb = c.inner / 256;
  const long long row_bytes = (long long)nsb * bb;
  long long wbytes = 0;
  for (int i = 0; i < c.nmats; ++i) wbytes += (long long)c.mats[i].rows * row_bytes;
  // Per-layer matrices (<= 64 MB): lean CTAs (8 consumer warps, <= 110 KB of
  // shared memory), so that this kernel's CTA and the next kernel's fit on
  // one SM together; with the early trigger the next kernel's weights then
  // stream in while this one computes.  The lm_head keeps 16 warps and the
  // whole shared memory (it is throughput-bound).
  static const int env_lean = getenv("INFERNO_MMA_LEAN") ? atoi(getenv("INFERNO_MMA_LEAN")) : 0;
  static const int env_early = getenv("INFERNO_PDL_EARLY") ? atoi(getenv("INFERNO_PDL_EARLY")) : 0;
  const int nxv = c.nxv;
  auto fixed_of = [&](int nw) -> size_t {
    return 16 * GEMV_MAX_STAGES + (2 * nw + 4 + 16) * 4 + nw * 16 * 4 +
           (size_t)nxv * ((size_t)nsb * 16 * 4 + (size_t)c.inner * 4 + (size_t)nsb * 8 * MMA_KS_BYTES) + 128;
  };
  auto stage_of = [&](int TR) -> size_t {
    if (paired) return 2 * (((size_t)(TR / 2) * row_bytes + 32 + 15) / 16 * 16) + 128;
    return ((size_t)TR * row_bytes + 48 + 127) / 128 * 128;
  };
  // lean only when two stages of the smallest tile fit next to the staged
  // activations (long rows, e.g. 12288 inputs, keep the full CTA)
  const int NW = (env_lean && wbytes <= (64ll << 20) && fixed_of(8) + 2 * stage_of(16) <= 110 * 1024) ? 8 : 16;
  const size_t smem_cap = NW == 8 ? 110 * 1024 : 220 * 1024;
  const size_t fixed = fixed_of(NW);
  bool any_indirect = false;
  for (int i = 0; i < c.nmats; ++i) any_indirect |= c.mats[i].indirect != 0;
  // cost: tile steps of the busiest CTA (each warp walks ceil(nsb / nkg)
  // super-blocks per tile) plus the bytes it streams
  int best_tr = 0;
  double best = 1e300;
  // tuning knobs (measurement only): a fixed tile height, a cap on the grid
  static const int env_tr = getenv("INFERNO_MMA_TR") ? atoi(getenv("INFERNO_MMA_TR")) : 0;
  static const int env_cap = getenv("INFERNO_MMA_GRID_CAP") ? atoi(getenv("INFERNO_MMA_GRID_CAP")) : 0;
  static const int env_tr_big = getenv("INFERNO_MMA_TR_BIG") ? atoi(getenv("INFERNO_MMA_TR_BIG")) : 0;
  if (env_cap > 0 && wbytes <= (64ll << 20)) sms = std::min(sms, env_cap);
  for (int TR : {16, 32, 64, 128}) {
    if (env_tr && TR != env_tr && wbytes <= (64ll << 20)) continue;
    if (env_tr_big && TR != env_tr_big && wbytes > (64ll << 20)) continue;
    const int nrg = TR / 16, nkg = NW / nrg;
    // a ring of one stage (no weight prefetch past the current tile) only
    // when two do not fit next to the staged activations of a long row
    const int nstg = (int)std::min<size_t>(2, (smem_cap - std::min(smem_cap, fixed)) / stage_of(TR));
    if (nstg < 1) continue;
    const int eff = paired ? TR / 2 : TR;
    if ((any_indirect || nxv > 1) && c.erows % eff) continue;   // a tile stays inside one expert / slot
    long long tiles = 0;
    for (int i = 0; i < (paired ? 1 : c.nmats); ++i) tiles += (c.mats[i].rows + eff - 1) / eff;
    const long long waves = (tiles + sms - 1) / sms;
    const double cost = (double)waves * ((nsb + nkg - 1) / nkg) + (double)waves * TR * row_bytes / 65536.0 +
                        (nstg < 2 ? 2.0 * waves : 0.0);
    if (cost < best) { best = cost; best_tr = TR; }
  }
  if (!best_tr) return 1;
  const int TR = best_tr, eff = paired ? TR / 2 : TR;
  GemvParams p = {};
  int ntiles = 0;
  for (int i = 0; i < c.nmats; ++i) {
    p.seg[i].W = (const uint8_t*)c.mats[i].W;
    p.seg[i].y = c.mats[i].y;
    p.seg[i].rows = c.mats[i].rows;
    p.seg[i].indirect = c.mats[i].indirect;
    p.seg[i].xslot0 = c.mats[i].xslot0;
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
  p.eidx = c.eidx;
  p.estride = c.estride;
  p.erows = c.erows;
  p.n_experts = c.n_experts;
  p.nxv = nxv;
  p.xch_n = c.xch_n;
  p.xch_rank = c.xch_rank;
  p.xch_wk = c.xch_wk;
  p.xch_rk = c.xch_rk;
  p.xch_spin = c.xch_spin ? c.xch_spin : (1u << 22);
  p.xch_seq = c.xch_seq;
  for (int q = 0; q < 8; ++q) p.xch_parts[q] = c.xch_parts[q];
  p.x_next = c.x_next;
  p.nkc = (c.inner + GEMV_CHUNK - 1) / GEMV_CHUNK;
  p.TR = TR;
  p.nkg = NW / (TR / 16);
  p.nb = 1;
  p.x = c.x;
  p.x_stride = c.x_stride;
  p.y_stride = c.y_stride;
  p.pro = c.pro;
  p.pro_w = c.pro_w;
  p.pro_z = c.pro_z;
  p.eps = c.eps;
  p.pro_group = c.pro_group;
  p.epi = c.epi;
  p.argmax = c.argmax;
  p.argmax_row0 = c.argmax_row0;
  p.err = c.err ? c.err : device_error_word(dev);
  p.trace = c.trace;
  static const bool no_hint = getenv("INFERNO_GEMV_NO_L2HINT") != nullptr;
  p.l2_evict_first = no_hint ? 0 : 1;
  p.early_trigger = env_early;
  static const bool env_dbg = getenv("INFERNO_GEMV_DBG") != nullptr;
  p.dbg = env_dbg ? atoi(getenv("INFERNO_GEMV_DBG")) : 0;
  if (ntiles == 0) return 0;
  const size_t stage_bytes = stage_of(TR);
  p.stages = (int)std::min<size_t>(GEMV_MAX_STAGES, (smem_cap - fixed) / stage_bytes);
  p.contig = 1;
  p.stage_bytes = (int)stage_bytes;
  p.part1_off = (int)((((size_t)(TR / 2) * row_bytes + 32 + 15) / 16) * 16);
  const size_t smem = fixed + (size_t)p.stages * stage_bytes;
  const int grid = std::min(ntiles, sms);
  cudaError_t e = c.type == T_Q4_K   ? launch_mma<T_Q4_K>(p, NW, grid, smem, st, pdl)
                  : c.type == T_Q6_KR ? launch_mma<T_Q6_KR>(p, NW, grid, smem, st, pdl)
                                      : launch_mma<T_Q6_K>(p, NW, grid, smem, st, pdl);
  if (e != cudaSuccess) return set_error(-2, "gemv launch failed: %s", cudaGetErrorString(e));
  return 0;
}

template <int TYPE>
cudaError_t launch_mma_batch(const GemvParams& p, int grid, size_t smem, cudaStream_t st, bool pdl) {
  // one carve-out for every kernel of the engine: no L1 / shared-memory
  // reconfiguration between back-to-back launches
  static DeviceOnce once;
  cudaError_t ea = once.run([] {
    cudaError_t e = cudaFuncSetAttribute(gemv_mma_batch_kernel<TYPE, MMA_NBT>, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
    if (e != cudaSuccess) return e;
    return cudaFuncSetAttribute(gemv_mma_batch_kernel<TYPE, MMA_NBT>, cudaFuncAttributePreferredSharedMemoryCarveout,
                                cudaSharedmemCarveoutMaxShared);
  });
  if (ea != cudaSuccess) return ea;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3((MMA_NBT + 1) * 32);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, gemv_mma_batch_kernel<TYPE, MMA_NBT>, p);
}

// Batched (several columns) Q4_K / Q6_K calls on the tensor-core path
// (gemv_mma_batch.cuh), MMA_NBT columns per launch.  Returns 1 when the call
// does not fit it (the caller falls back to the CUDA-core kernel).
int plan_launch_mma_batch(const GemvCall& c, int dev, int sms, cudaStream_t st, bool pdl) {
  constexpr int NW = MMA_NBT;
  const int bb = bb_of(c.type);
  const bool paired = c.epi == EPI_SWIGLU;
  const int nsb = c.inner / 256;
  const long long row_bytes = (long long)nsb * bb;
  const size_t smem_cap = 220 * 1024;
  if (c.epi == EPI_ARGMAX || c.x_stride % 4 || (c.pro_z && c.x_stride % 4)) return 1;
  if (c.pro == PRO_HEADNORM_GATE && c.inner / c.pro_group > MMA_MAX_HEADS) return 1;
  for (int i = 0; i < c.nmats; ++i)
    if (c.mats[i].indirect) return 1;
  const size_t xq_col = (size_t)nsb * 8 * MMA_KSC_BYTES;
  const size_t fixed = mma_batch_fixed_bytes<NW>() + (size_t)MMA_NBT * nsb * 16 * 4 + MMA_NBT * xq_col + 128;
  auto stage_of = [&](int TR) -> size_t {
    if (paired) return 2 * (((size_t)(TR / 2) * row_bytes + 32 + 15) / 16 * 16) + 128;
    return ((size_t)TR * row_bytes + 48 + 127) / 128 * 128;
  };
  int best_tr = 0;
  double best = 1e300;
  for (int TR : {16, 32, 64, 128}) {
    const int nrg = TR / 16;
    if (nrg > NW) continue;
    const int nkg = NW / nrg;
    if (fixed > smem_cap || (smem_cap - fixed) / stage_of(TR) < 2) continue;
    const int eff = paired ? TR / 2 : TR;
    long long tiles = 0;
    for (int i = 0; i < (paired ? 1 : c.nmats); ++i) tiles += (c.mats[i].rows + eff - 1) / eff;
    const long long waves = (tiles + sms - 1) / sms;
    const double cost = (double)waves * ((nsb + nkg - 1) / nkg) + (double)waves * TR * row_bytes / 65536.0;
    if (cost < best) { best = cost; best_tr = TR; }
  }
  if (!best_tr) return 1;
  const int TR = best_tr, eff = paired ? TR / 2 : TR;
  GemvParams p = {};
  int ntiles = 0;
  for (int i = 0; i < c.nmats; ++i) {
    p.seg[i].W = (const uint8_t*)c.mats[i].W;
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
  p.nxv = 1;
  p.xch_wk = p.xch_rk = -1;
  p.nkc = (c.inner + GEMV_CHUNK - 1) / GEMV_CHUNK;
  p.TR = TR;
  p.nkg = NW / (TR / 16);
  p.x_stride = c.x_stride;
  p.y_stride = c.y_stride;
  p.pro = c.pro;
  p.pro_w = c.pro_w;
  p.eps = c.eps;
  p.pro_group = c.pro_group;
  p.epi = c.epi;
  p.err = c.err ? c.err : device_error_word(dev);
  static const bool no_hint = getenv("INFERNO_GEMV_NO_L2HINT") != nullptr;
  p.l2_evict_first = no_hint ? 0 : 1;
  if (ntiles == 0) return 0;
  const size_t stage_bytes = stage_of(TR);
  p.stages = (int)std::min<size_t>(GEMV_MAX_STAGES, (smem_cap - fixed) / stage_bytes);
  p.contig = 1;
  p.stage_bytes = (int)stage_bytes;
  p.part1_off = (int)((((size_t)(TR / 2) * row_bytes + 32 + 15) / 16) * 16);
  const size_t smem = fixed + (size_t)p.stages * stage_bytes;
  const int grid = std::min(ntiles, sms);
  for (int done = 0; done < c.nb; done += MMA_NBT) {
    p.nb = std::min(MMA_NBT, c.nb - done);
    p.x = c.x + (long long)done * c.x_stride;
    p.pro_z = c.pro_z ? c.pro_z + (long long)done * c.x_stride : nullptr;
    for (int i = 0; i < c.nmats; ++i) p.seg[i].y = c.mats[i].y ? c.mats[i].y + (long long)done * c.y_stride : nullptr;
    cudaError_t e = c.type == T_Q4_K ? launch_mma_batch<T_Q4_K>(p, grid, smem, st, pdl)
                                     : launch_mma_batch<T_Q6_K>(p, grid, smem, st, pdl);
    if (e != cudaSuccess) return set_error(-2, "batched gemv launch failed: %s", cudaGetErrorString(e));
  }
  return 0;
}

}  // namespace

// Regroup a Q6_K matrix (rows % 16 == 0) into the T_Q6_KR layout: one CTA of
// 32 threads per (16-row group, super-block).
__global__ void __launch_bounds__(32) repack_q6k_kernel(const uint8_t* __restrict__ src, uint8_t* __restrict__ dst,
                                                        int nsb) {
  const int G = blockIdx.x, sb = blockIdx.y, L = threadIdx.x;
  const int g = L >> 2, c = L & 3;
  const size_t rb = (size_t)nsb * 210;
  uint8_t* out = dst + ((size_t)G * nsb + sb) * Q6R_BLOCK;
  auto word = [&](int row, int w) -> uint32_t {
    const uint8_t* b = src + (size_t)row * rb + (size_t)sb * 210;
    const int off = w < 8 ? 64 * (w >> 2) + 32 * ((w >> 1) & 1) + 16 * (w & 1) + 4 * c
                          : 128 + 32 * ((w - 8) >> 1) + 16 * ((w - 8) & 1) + 4 * c;
    return (uint32_t)b[off] | ((uint32_t)b[off + 1] << 8) | ((uint32_t)b[off + 2] << 16) | ((uint32_t)b[off + 3] << 24);
  };
  const int ra = 16 * G + g, rbw = ra + 8;
#pragma unroll
  for (int i = 0; i < 6; ++i) {
    uint32_t v[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int w = 4 * i + j;
      v[j] = w < 12 ? word(ra, w) : word(rbw, w - 12);
    }
    *(uint4*)(out + (i * 32 + L) * 16) = make_uint4(v[0], v[1], v[2], v[3]);
  }
  if (L < 16) {
    const uint8_t* b = src + (size_t)(16 * G + L) * rb + (size_t)sb * 210;
    for (int j = 0; j < 16; ++j) out[3072 + L * 16 + j] = b[192 + j];
    out[3328 + L * 2] = b[208];
    out[3328 + L * 2 + 1] = b[209];
  }
}

int launch_repack_q6k(const void* src, void* dst, int rows, int inner, cudaStream_t st) {
  if (rows <= 0 || rows % 16 || inner <= 0 || inner % 256)
    return set_error(-1, "repack: Q6_K %d x %d is not a multiple of 16 rows x 256 columns", rows, inner);
  repack_q6k_kernel<<<dim3(rows / 16, inner / 256), 32, 0, st>>>((const uint8_t*)src, (uint8_t*)dst, inner / 256);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? 0 : set_error(-2, "repack launch: %s", cudaGetErrorString(e));
}

int launch_gemv(const GemvCall& c, cudaStream_t st, bool pdl) {
  if (c.type == T_Q6_KR) {
    // regrouped Q6_K exists only for the single-column tensor-core path
    if (c.nb != 1 || c.epi == EPI_SWIGLU || c.inner % 256 || c.nxv != 1)
      return set_error(-1, "gemv: regrouped Q6_K needs a single-column, non-paired call");
    for (int i = 0; i < c.nmats; ++i)
      if (c.mats[i].rows % 16 || c.mats[i].indirect) return set_error(-1, "gemv: regrouped Q6_K rows");
    int dev = 0;
    cudaGetDevice(&dev);
    const int rc = plan_launch_mma(c, dev, num_sms(dev), st, pdl);
    return rc > 0 ? set_error(-1, "gemv: regrouped Q6_K %d-column rows do not fit shared memory", c.inner) : rc;
  }
  if (!type_supported(c.type) || c.nmats < 1 || c.nmats > GEMV_MAX_SEG || c.nb < 1)
    return set_error(-1, "gemv: bad type/mats/batch (type=%d nmats=%d nb=%d)", c.type, c.nmats, c.nb);
  const int qk = qk_of(c.type), bb = bb_of(c.type);
  if (c.inner <= 0 || c.inner % (c.type == T_F32 ? 32 : qk) != 0 || (qk == 256 && c.inner % 256))
    return set_error(-1, "gemv: inner dim %d not a multiple of the block size", c.inner);
  const bool paired = c.epi == EPI_SWIGLU;
  if (paired && (c.nmats != 2 || c.mats[0].rows != c.mats[1].rows))
    return set_error(-1, "gemv: SwiGLU needs two matrices with equal rows");
  for (int i = 0; i < c.nmats; ++i) {
    if (((uintptr_t)c.mats[i].W & 15) != 0) return set_error(-1, "gemv: weight pointer not 16-byte aligned");
    if (c.mats[i].rows < 0) return set_error(-1, "gemv: negative rows");
  }
  if (c.pro == PRO_HEADNORM_GATE &&
      (c.pro_group <= 0 || c.pro_group % 32 || c.pro_group > 256 || c.inner % c.pro_group))
    return set_error(-1, "gemv: bad head group %d", c.pro_group);
  int dev = 0;
  cudaGetDevice(&dev);
  const int sms = num_sms(dev);
  bool any_indirect = false;
  for (int i = 0; i < c.nmats; ++i) any_indirect |= c.mats[i].indirect != 0;
  if (c.nxv < 1 || (c.nxv > 1 && (c.pro != PRO_NONE || c.erows <= 0 || c.nxv > 16)) ||
      (any_indirect && (!c.eidx || c.erows <= 0 || c.n_experts <= 0 || c.estride <= 0)))
    return set_error(-1, "gemv: bad expert / multi-vector arguments");
  static const bool no_mma = getenv("INFERNO_GEMV_NO_MMA") != nullptr;
  const bool mma_ok = !c.force_r && c.nb == 1 && (c.type == T_Q4_K || c.type == T_Q6_K) && c.inner % 256 == 0;
  if (mma_ok && (!no_mma || c.nxv > 1 || c.xch_wk >= 0 || c.xch_rk >= 0)) {
    const int rc = plan_launch_mma(c, dev, sms, st, pdl);
    if (rc <= 0) return rc;
  }
  if (c.nb >= 16) {   // many columns: the tensor-core GEMM (qgemm_tc.cu)
    const int rc = qgemm_from_gemv(c, st);
    if (rc <= 0) return rc;
  }
  static const bool no_mma_batch = getenv("INFERNO_GEMV_NO_MMA_BATCH") != nullptr;
  if (!no_mma && !no_mma_batch && !c.force_r && c.nb > 1 && c.nxv == 1 && (c.type == T_Q4_K || c.type == T_Q6_K) &&
      c.inner % 256 == 0) {
    const int rc = plan_launch_mma_batch(c, dev, sms, st, pdl);
    if (rc <= 0) return rc;
  }
  if (c.nxv > 1) return set_error(-1, "gemv: several input vectors need single-column Q4_K/Q6_K");
  if (c.xch_wk >= 0 || c.xch_rk >= 0)
    return set_error(-1, "gemv: the tensor-parallel exchange needs single-column Q4_K/Q6_K rows");
  const long long row_bytes = (long long)c.inner / qk * bb;
  const int nkc = (c.inner + GEMV_CHUNK - 1) / GEMV_CHUNK;
  long long wbytes = 0;
  for (int i = 0; i < c.nmats; ++i) wbytes += (long long)c.mats[i].rows * row_bytes;
  // small matrices: lean CTAs (8 consumer warps, <= ~110 KB smem) so that
  // two CTAs -- this kernel's and the next one's -- fit on an SM
  static const int env_nw = getenv("INFERNO_GEMV_FORCE_NW") ? atoi(getenv("INFERNO_GEMV_FORCE_NW")) : 0;
  // 16 consumer warps: per-tile parallelism matters more on the latency-bound
  // per-layer matrices than letting the next kernel's CTA co-reside (measured)
  const int NW = env_nw ? env_nw : 16;
  const size_t fixed = 16 * GEMV_MAX_STAGES + 128 * 4 + 256 * 8 + 128;
  const size_t smem_cap = NW == 8 ? 110 * 1024 : 220 * 1024;
  const size_t ring_budget = NW == 8 ? 64 * 1024 : 96 * 1024;
  auto stage_of = [&](int TR) -> size_t {
    if (paired) return 2 * (((size_t)(TR / 2) * row_bytes + 32 + 15) / 16 * 16) + 128;
    return ((size_t)TR * row_bytes + 48 + 127) / 128 * 128;
  };
  // activations + K-group partials for nbv columns
  auto xbytes = [&](int nbv) {
    return (size_t)nbv * nkc * GEMV_CHUNK * 4 + (size_t)nbv * 8 * 64 * 4;
  };
  const int nb_tmpl = c.nb >= 8 ? 8 : (c.nb >= 2 ? 4 : 1);

  // Tile shape: R rows per warp, nkg K groups (warps splitting the chunks of
  // a tile), TR = R * NW / nkg rows per tile, one bulk copy per tile.  Cost =
  // bytes the slowest CTA streams, with small penalties for fewer rows per
  // warp (activation reuse) and for K groups (cross-warp reduction).
  int best_r = 0, best_g = 1;
  static const int env_force_r = getenv("INFERNO_GEMV_FORCE_R") ? atoi(getenv("INFERNO_GEMV_FORCE_R")) : 0;
  // single-column calls use 2 rows per warp: one GEMV instantiation per type
  // keeps the engine's instruction working set small (the per-layer kernels
  // are latency-bound and cold code costs microseconds per launch)
  const int pref_r = c.force_r ? c.force_r : (env_force_r ? env_force_r : (c.nb == 1 ? (wbytes > (16ll << 20) ? 4 : 2) : 0));
  double best_cost = 1e300;
  for (int attempt = 0; attempt < 2 && !best_r; ++attempt) {
  // the preferred R is dropped (planner's choice) if its tiles do not fit
  const int force_r = (attempt == 0 || c.force_r) ? pref_r : 0;
  for (int R : {4, 2, 1}) {
    if (paired && R < 2) continue;
    if (force_r && R != force_r) continue;
    if (c.nb > 1 && R != (paired ? 2 : 1)) continue;
    for (int g : {1, 2, 4, 8}) {
      if (g > nkc) continue;
      const int TR = R * NW / g;
      if (TR > 64 || (paired && TR % 2)) continue;
      const size_t stg = stage_of(TR);
      if (fixed + xbytes(1) + 2 * stg > smem_cap) continue;
      const int eff = paired ? TR / 2 : TR;
      if (any_indirect && c.erows % eff) continue;   // a tile stays inside one expert
      long long tiles = 0;
      for (int i = 0; i < (paired ? 1 : c.nmats); ++i) tiles += (c.mats[i].rows + eff - 1) / eff;
      const long long waves = (tiles + sms - 1) / sms;
      const double cost = (double)waves * TR * row_bytes * (R == 4 ? 1.0 : R == 2 ? 1.1 : 1.22) * (1.0 + 0.04 * (g - 1));
      if (cost < best_cost) { best_cost = cost; best_r = R; best_g = g; }
    }
  }
  }
  if (!best_r) return set_error(-1, "gemv: rows of %lld bytes do not fit shared memory", row_bytes);
  const int R = best_r, TR = R * NW / best_g, eff = paired ? TR / 2 : TR;

  GemvParams p = {};
  int ntiles = 0;
  for (int i = 0; i < c.nmats; ++i) {
    p.seg[i].W = (const uint8_t*)c.mats[i].W;
    p.seg[i].y = c.mats[i].y;
    p.seg[i].rows = c.mats[i].rows;
    p.seg[i].indirect = c.mats[i].indirect;
    p.seg[i].xslot0 = 0;
    if (paired && i == 1) {
      p.seg[i].tile0 = INT_MAX;
    } else {
      p.seg[i].tile0 = ntiles;
      ntiles += (c.mats[i].rows + eff - 1) / eff;
    }
  }
  p.nseg = c.nmats;
  p.ntiles = ntiles;
  p.inner = c.inner;
  p.row_bytes = (int)row_bytes;
  p.eidx = c.eidx;
  p.estride = c.estride;
  p.erows = c.erows;
  p.n_experts = c.n_experts;
  p.nxv = 1;
  p.xch_wk = p.xch_rk = -1;
  p.nkc = nkc;
  p.TR = TR;
  p.nkg = best_g;
  p.pro = c.pro;
  p.pro_w = c.pro_w;
  p.eps = c.eps;
  p.pro_group = c.pro_group;
  p.epi = c.epi;
  p.err = c.err ? c.err : device_error_word(dev);
  p.trace = c.trace;
  static const bool no_hint = getenv("INFERNO_GEMV_NO_L2HINT") != nullptr;
  p.l2_evict_first = no_hint ? 0 : 1;
  if (ntiles == 0) return 0;
  const size_t stage_bytes = stage_of(TR);
  int stages = (int)std::min<size_t>(GEMV_MAX_STAGES, std::max<size_t>(2, ring_budget / stage_bytes));
  p.contig = 1;
  p.stage_bytes = (int)stage_bytes;
  p.part1_off = (int)((((size_t)(TR / 2) * row_bytes + 32 + 15) / 16) * 16);
  // batch groups that fit the activation staging area
  int done = 0;
  while (done < c.nb) {
    const int left = c.nb - done;
    int NB = std::min(nb_tmpl, left >= 8 ? 8 : (left >= 2 ? 4 : 1));
    auto need = [&](int nbv) { return fixed + xbytes(nbv) + stages * stage_bytes; };
    while (NB > 1 && need(NB) > smem_cap) NB = NB == 8 ? 4 : 1;
    while (need(NB) > smem_cap && stages > 2) --stages;
    if (need(NB) > smem_cap) return set_error(-1, "gemv: inner dim %d too large for shared memory", c.inner);
    p.stages = stages;
    p.nb = std::min(NB, left);
    p.x = c.x + (long long)done * c.x_stride;
    p.x_stride = c.x_stride;
    p.y_stride = c.y_stride;
    p.pro_z = c.pro_z ? c.pro_z + (long long)done * c.x_stride : nullptr;
    for (int i = 0; i < c.nmats; ++i) p.seg[i].y = c.mats[i].y ? c.mats[i].y + (long long)done * c.y_stride : nullptr;
    p.argmax = c.argmax ? c.argmax + done : nullptr;
    p.argmax_row0 = c.argmax_row0;
    const int grid = std::min(ntiles, sms);
    const size_t smem = need(NB);
    cudaError_t e;
    switch (c.type) {
      case T_Q4_K: e = launch_nb<T_Q4_K>(p, NB, R, NW, grid, smem, st, pdl); break;
      case T_Q5_K: e = launch_nb<T_Q5_K>(p, NB, R, NW, grid, smem, st, pdl); break;
      case T_Q6_K: e = launch_nb<T_Q6_K>(p, NB, R, NW, grid, smem, st, pdl); break;
      case T_Q8_0: e = launch_nb<T_Q8_0>(p, NB, R, NW, grid, smem, st, pdl); break;
      case T_IQ2_XXS: e = launch_nb<T_IQ2_XXS>(p, NB, R, NW, grid, smem, st, pdl); break;
      default: e = launch_nb<T_F32>(p, NB, R, NW, grid, smem, st, pdl); break;
    }
    if (e != cudaSuccess) return set_error(-2, "gemv launch failed: %s", cudaGetErrorString(e));
    done += p.nb;
  }
  return 0;
}

}  // namespace inf

namespace inf {
// debug: the tensor-core GEMV timeline stamps (INFERNO_GEMV_DBG=1)
int gemv_dbg_read(unsigned long long* out32) {
  return cudaMemcpyFromSymbol(out32, gemv_dbg, 32 * sizeof(unsigned long long)) == cudaSuccess ? 0 : -1;
}
}  // namespace inf
