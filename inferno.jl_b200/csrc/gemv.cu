// GEMV launch planner + template instantiations (see gemv.cuh for the kernel).
#include <algorithm>
#include <climits>
#include <cstdlib>
#include "internal.h"
#include "gemv.cuh"

namespace inf {

namespace {

template <int TYPE, int NB, int R>
cudaError_t launch_one(const GemvParams& p, int grid, size_t smem, cudaStream_t st, bool pdl) {
  static bool attr_done[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (!attr_done[dev & 63]) {
    cudaError_t e = cudaFuncSetAttribute(gemv_kernel<TYPE, NB, R>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         227 * 1024);
    if (e != cudaSuccess) return e;
    attr_done[dev & 63] = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(GEMV_THREADS);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, gemv_kernel<TYPE, NB, R>, p);
}

template <int TYPE, int NB>
cudaError_t launch_r(const GemvParams& p, int R, int grid, size_t smem, cudaStream_t st, bool pdl) {
  switch (R) {
    case 1: return launch_one<TYPE, NB, 1>(p, grid, smem, st, pdl);
    case 2: return launch_one<TYPE, NB, 2>(p, grid, smem, st, pdl);
    default: return launch_one<TYPE, NB, 4>(p, grid, smem, st, pdl);
  }
}

template <int TYPE>
cudaError_t launch_nb(const GemvParams& p, int NB, int R, int grid, size_t smem, cudaStream_t st, bool pdl) {
  switch (NB) {
    case 1: return launch_r<TYPE, 1>(p, R, grid, smem, st, pdl);
    // batched columns use one row per warp (the x fragments of all columns
    // are live at once; more rows would spill)
    case 4: return R == 1 ? launch_one<TYPE, 4, 1>(p, grid, smem, st, pdl) : launch_one<TYPE, 4, 2>(p, grid, smem, st, pdl);
    default: return R == 1 ? launch_one<TYPE, 8, 1>(p, grid, smem, st, pdl) : launch_one<TYPE, 8, 2>(p, grid, smem, st, pdl);
  }
}

}  // namespace

int launch_gemv(const GemvCall& c, cudaStream_t st, bool pdl) {
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
  int dev = 0;
  cudaGetDevice(&dev);
  const int sms = num_sms(dev);
  const long long row_bytes = (long long)c.inner / qk * bb;
  const int ce_bytes = GEMV_CHUNK / qk * bb;
  const int slot = ((std::min<long long>(ce_bytes, row_bytes) + 15) / 16) * 16 + 32;
  const int nkc = (c.inner + GEMV_CHUNK - 1) / GEMV_CHUNK;

  const bool sums = (c.type == T_Q4_K || c.type == T_Q5_K);
  static const bool force_rowcopy = getenv("INFERNO_GEMV_ROWCOPY") != nullptr;
  const bool contig = (nkc == 1) && !force_rowcopy;
  const size_t fixed = 16 * GEMV_MAX_STAGES + 32 * 4 + 256 * 8 + 128;
  const size_t smem_cap = 220 * 1024, ring_budget = 96 * 1024;
  auto stage_of = [&](int R) -> size_t {
    int TR = GEMV_NW * R;
    if (!contig) return (size_t)TR * slot;
    if (paired) return 2 * (((size_t)(TR / 2) * row_bytes + 32 + 15) / 16 * 16) + 128;
    return ((size_t)TR * row_bytes + 48 + 127) / 128 * 128;
  };
  auto xbytes = [&](int nbv) {
    return (size_t)nbv * nkc * GEMV_CHUNK * 4 + (sums ? (size_t)nbv * nkc * 64 * 4 : 0);
  };

  // R choice: minimise rows per CTA for the slowest CTA (waves x tile rows),
  // preferring larger R (activation reuse) on ties; R must leave room for
  // two stages next to the activations.
  int best_r = 0;
  long long best_cost = LLONG_MAX;
  for (int R : {4, 2, 1}) {
    if (paired && R < 2) continue;
    if (c.force_r && R != c.force_r) continue;
    if (c.nb > 1 && R != (paired ? 2 : 1)) continue;
    if (fixed + xbytes(1) + 2 * stage_of(R) > smem_cap) continue;
    int TR = GEMV_NW * R, eff = paired ? TR / 2 : TR;
    long long tiles = 0;
    for (int i = 0; i < (paired ? 1 : c.nmats); ++i) tiles += (c.mats[i].rows + eff - 1) / eff;
    long long waves = (tiles + sms - 1) / sms;
    // rows the slowest CTA handles; fewer rows per warp cost ~25% more per
    // row (activation reuse, per-tile overhead)
    long long cost = waves * TR * (R == 4 ? 100 : R == 2 ? 112 : 125);
    if (cost < best_cost) { best_cost = cost; best_r = R; }
  }
  if (!best_r) return set_error(-1, "gemv: inner dim %d too large for shared memory", c.inner);
  const int R = best_r, TR = GEMV_NW * R, eff = paired ? TR / 2 : TR;

  GemvParams p = {};
  int ntiles = 0;
  for (int i = 0; i < c.nmats; ++i) {
    p.seg[i].W = (const uint8_t*)c.mats[i].W;
    p.seg[i].y = c.mats[i].y;
    p.seg[i].rows = c.mats[i].rows;
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
  p.nkc = nkc;
  p.TR = TR;
  p.slot = slot;
  p.pro = c.pro;
  p.pro_w = c.pro_w;
  p.pro_z = c.pro_z;
  p.eps = c.eps;
  p.pro_group = c.pro_group;
  p.epi = c.epi;
  p.argmax = c.argmax;
  p.err = c.err ? c.err : device_error_word(dev);
  if (ntiles == 0) return 0;
  if (c.pro == PRO_HEADNORM_GATE && (c.pro_group <= 0 || c.inner % c.pro_group))
    return set_error(-1, "gemv: bad head group %d", c.pro_group);

  const size_t stage_bytes = stage_of(R);
  int stages = (int)std::min<size_t>(GEMV_MAX_STAGES, std::max<size_t>(2, ring_budget / stage_bytes));
  p.contig = contig ? 1 : 0;
  p.stage_bytes = (int)stage_bytes;
  p.part1_off = (int)((((size_t)(TR / 2) * row_bytes + 32 + 15) / 16) * 16);
  // batch groups that fit the x staging area
  int done = 0;
  while (done < c.nb) {
    int left = c.nb - done;
    int NB = left >= 8 ? 8 : (left >= 2 ? 4 : 1);
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
    int grid = std::min(ntiles, sms);
    size_t smem = need(NB);
    cudaError_t e;
    switch (c.type) {
      case T_Q4_K: e = launch_nb<T_Q4_K>(p, NB, R, grid, smem, st, pdl); break;
      case T_Q5_K: e = launch_nb<T_Q5_K>(p, NB, R, grid, smem, st, pdl); break;
      case T_Q6_K: e = launch_nb<T_Q6_K>(p, NB, R, grid, smem, st, pdl); break;
      case T_Q8_0: e = launch_nb<T_Q8_0>(p, NB, R, grid, smem, st, pdl); break;
      case T_IQ2_XXS: e = launch_nb<T_IQ2_XXS>(p, NB, R, grid, smem, st, pdl); break;
      default: e = launch_nb<T_F32>(p, NB, R, grid, smem, st, pdl); break;
    }
    if (e != cudaSuccess) return set_error(-2, "gemv launch failed: %s", cudaGetErrorString(e));
    done += p.nb;
  }
  return 0;
}

}  // namespace inf
