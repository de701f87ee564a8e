// Mixture-of-experts FFN pieces around the expert GEMVs (config 5).
//
// Restates the routing of Inferno.jl src/Model.jl:497-526 for batch-1 decode:
//   p = softmax(W_r * x)                (router logits from an F32 GEMV)
//   top = sortperm(p, rev=true)[1:k]    (stable: ties go to the lower index)
//   w_i = p_top[i] / sum(p_top)
//   out = sum_i w_i * expert_top[i](x)  (+ the always-on shared expert)
// The expert GEMVs themselves (gate/up SwiGLU over device-selected experts,
// one down GEMV over all selected experts with per-expert inputs) are the
// row-indirect GEMV paths of gemv.cuh / gemv_mma.cuh.
#include "internal.h"
#include "common.cuh"
#include "../../include/inferno_b200.h"

namespace inf {

constexpr int MOE_MAX_E = 1024;
constexpr int MOE_MAX_K = 16;

// One warp: softmax over E logits, stable top-k, renormalised weights.
__global__ void __launch_bounds__(32) moe_topk_kernel(const float* logits, int E, int K, int* idx, float* wts,
                                                      int* err, int ebase, int eloc) {
  __shared__ float p[MOE_MAX_E];
  __shared__ float sum_s;
  const int lane = threadIdx.x;
  pdl_wait();
  pdl_trigger();
  float mx = -INFINITY;
  for (int e = lane; e < E; e += 32) {
    const float v = logits[e];
    p[e] = v;
    mx = fmaxf(mx, v);
  }
  mx = warp_max(mx);
  for (int e = lane; e < E; e += 32) p[e] = expf(p[e] - mx);
  __syncwarp();
  if (lane == 0) {
    float s = 0.0f;                 // sequential, in expert order
    for (int e = 0; e < E; ++e) s += p[e];
    sum_s = s;
  }
  __syncwarp();
  const float sum = sum_s;
  for (int e = lane; e < E; e += 32) p[e] = p[e] / sum;
  __syncwarp();
  // k rounds of first-max selection (value descending, index ascending)
  int chosen[MOE_MAX_K];
  float pv[MOE_MAX_K];
  for (int r = 0; r < K; ++r) {
    float bv = -INFINITY;
    int bi = 0x7fffffff;
    for (int e = lane; e < E; e += 32) {
      const float v = p[e];
      if (v > bv || (v == bv && e < bi)) { bv = v; bi = e; }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
    }
    if (bi < 0 || bi >= E) {       // NaN logits: no valid maximum
      if (lane == 0) atomicExch(err, DERR_BAD_ARG);
      bi = 0;
      bv = 0.0f;
    }
    chosen[r] = bi;
    pv[r] = bv;
    __syncwarp();
    if (lane == 0) p[bi] = -INFINITY;
    __syncwarp();
  }
  if (lane == 0) {
    float ts = 0.0f;
    for (int r = 0; r < K; ++r) ts += pv[r];
    // expert parallelism: ids local to this rank's experts [ebase, ebase +
    // eloc), -1 for experts held by another rank
    for (int r = 0; r < K; ++r) {
      const int id = chosen[r] - ebase;
      idx[r] = (id >= 0 && id < eloc) ? id : -1;
      wts[r] = pv[r] / ts;
    }
  }
}

// x[j] += sum_i w_i * y[i][j] (+ y[K][j] for the shared expert), expert order
// fixed (deterministic).
// Expert parallelism (partial = 1): only this rank's experts contribute and
// rank 0 (add_x = 1) adds the residual and the shared expert; the caller then
// sums x over the ranks.
__global__ void moe_combine_kernel(float* x, const float* y, const float* wts, const int* idx, int K, int H, int shared,
                                   int add_x) {
  pdl_wait();
  pdl_trigger();
  const int j = blockIdx.x * blockDim.x + threadIdx.x;
  if (j >= H) return;
  float acc = 0.0f;
  for (int i = 0; i < K; ++i)
    if (idx[i] >= 0) acc = __fadd_rn(acc, __fmul_rn(wts[i], y[(long long)i * H + j]));
  if (shared) acc = __fadd_rn(acc, y[(long long)K * H + j]);
  x[j] = add_x ? __fadd_rn(x[j], acc) : acc;
}

// Expert parallelism over the fused residual exchange: this rank's partial
// sum_i w_i y_i (+ the shared expert on rank 0), without x, goes to every
// rank's exchange buffer as 64-bit {value, tag} words (sync point k, tag
// *seq + k + 1); the next RMSNorm GEMV of every rank polls the tags and adds
// x + sum over ranks in rank order (bit-identical on all ranks).
__global__ void moe_combine_xch_kernel(const float* y, const float* wts, const int* idx, int K, int H, int shared,
                                       MoeXch xc) {
  pdl_wait();
  pdl_trigger();
  const int j = blockIdx.x * blockDim.x + threadIdx.x;
  if (j >= H) return;
  float acc = 0.0f;
  for (int i = 0; i < K; ++i)
    if (idx[i] >= 0) acc = __fadd_rn(acc, __fmul_rn(wts[i], y[(long long)i * H + j]));
  if (shared) acc = __fadd_rn(acc, y[(long long)K * H + j]);
  const uint32_t tag = (uint32_t)(*xc.seq + (unsigned long long)xc.k + 1ull);
  const unsigned long long w = ((unsigned long long)tag << 32) | __float_as_uint(acc);
  const size_t off = ((size_t)(xc.k & 1) * xc.n + xc.rank) * H + j;
  for (int q = 0; q < xc.n; ++q)
    asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(xc.parts[q] + off), "l"(w) : "memory");
}

namespace {
template <class F, class... A>
int launch_pdl(F kern, dim3 grid, dim3 block, cudaStream_t st, bool pdl, A... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.stream = st;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = pdl ? 1 : 0;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kern, args...);
  return e == cudaSuccess ? 0 : set_error(INFERNO_ECUDA, "moe launch: %s", cudaGetErrorString(e));
}
}  // namespace

int launch_moe_topk(const float* logits, int E, int K, int* idx, float* wts, int* err, int ebase, int eloc,
                    cudaStream_t st, bool pdl) {
  if (E <= 0 || E > MOE_MAX_E || K <= 0 || K > MOE_MAX_K || K > E)
    return set_error(INFERNO_EINVAL, "moe: %d experts / top-%d unsupported (max %d / %d)", E, K, MOE_MAX_E, MOE_MAX_K);
  return launch_pdl(moe_topk_kernel, dim3(1), dim3(32), st, pdl, logits, E, K, idx, wts, err, ebase, eloc);
}

int launch_moe_combine(float* x, const float* y, const float* wts, const int* idx, int K, int H, int shared,
                       int add_x, cudaStream_t st, bool pdl) {
  return launch_pdl(moe_combine_kernel, dim3((H + 255) / 256), dim3(256), st, pdl, x, y, wts, idx, K, H, shared,
                    add_x);
}

int launch_moe_combine_xch(const float* y, const float* wts, const int* idx, int K, int H, int shared,
                           const MoeXch& xc, cudaStream_t st, bool pdl) {
  return launch_pdl(moe_combine_xch_kernel, dim3((H + 255) / 256), dim3(256), st, pdl, y, wts, idx, K, H, shared, xc);
}

}  // namespace inf
