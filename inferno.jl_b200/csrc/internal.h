// Host-side internal declarations shared by the engine's translation units.
#pragma once
#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <stdint.h>
#include <mutex>
#include <string>
#include <vector>

namespace inf {

// ---- error channel (thread-local last error, int status codes) ------------
int set_error(int code, const char* fmt, ...);
const char* last_error();

#define INF_CUDA_TRY(expr)                                                            \
  do {                                                                                \
    cudaError_t e_ = (expr);                                                          \
    if (e_ != cudaSuccess)                                                            \
      return ::inf::set_error(-2, "%s failed: %s (%s:%d)", #expr, cudaGetErrorString(e_), \
                              __FILE__, __LINE__);                                    \
  } while (0)

int num_sms(int device);

// One-time kernel set-up per device (cudaFuncSetAttribute and the like): the
// function attributes belong to the current device's context, so a second
// engine on another device needs its own call.  run(f) calls f() on the
// current device the first time, under a lock, and remembers success; a
// failure is returned and retried on the next call.
struct DeviceOnce {
  std::mutex mu;
  bool done[64] = {};
  template <class F>
  cudaError_t run(F&& f) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    std::lock_guard<std::mutex> g(mu);
    if (done[dev]) return cudaSuccess;
    e = f();
    if (e == cudaSuccess) done[dev] = true;
    return e;
  }
};

// ---- kernel launchers (return 0 or a negative status) ---------------------
struct GemvMat {
  const void* W;   // device, 16-byte aligned
  float* y;        // device output rows
  int rows;
  int indirect = 0;   // rows gathered through GemvCall::eidx (MoE experts)
  int xslot0 = 0;     // input-vector slot of the first row (GemvCall::nxv > 1)
};

struct GemvCall {
  int type = 0;
  int inner = 0;
  GemvMat mats[4];
  int nmats = 0;
  int nb = 1;
  const float* x = nullptr;
  long long x_stride = 0;     // elements between batch columns of x
  long long y_stride = 0;     // elements between batch columns of y
  int pro = 0;
  const float* pro_w = nullptr;
  const float* pro_z = nullptr;
  float eps = 1e-6f;
  int pro_group = 0;
  int epi = 0;
  unsigned long long* argmax = nullptr;
  int argmax_row0 = 0;        // global index of row 0 of mats[0] (vocab-split lm_head)
  int* err = nullptr;
  int force_r = 0;            // 0 = planner's choice
  // MoE: for an `indirect` matrix, row r is row (r % erows) of expert
  // eidx[r / erows] (device ids), experts `estride` bytes apart
  const int* eidx = nullptr;
  long long estride = 0;
  int erows = 0;
  int n_experts = 0;
  // several input vectors (x + v * x_stride, v < nxv): rows use vector
  // xslot0 + r / erows (single-column tensor-core path, PRO_NONE only)
  int nxv = 1;
  // tensor-parallel residual exchange (see GemvParams::xch_*); -1 = off
  int xch_n = 0, xch_rank = 0, xch_wk = -1, xch_rk = -1;
  unsigned xch_spin = 0;      // reader poll limit per word (0 = 2^22)
  const unsigned long long* xch_seq = nullptr;
  unsigned long long* xch_parts[8] = {};
  float* x_next = nullptr;
  unsigned long long* trace = nullptr;   // debug phase timestamps (32 slots)
};

int launch_gemv(const GemvCall& c, cudaStream_t st, bool pdl);

// Tensor-core quantized GEMM (qgemm_tc.cu) for T >= 16 token columns:
// y[t][r] = sum_k W[r][k] x[t][k].  The activations come as fp16 hi / lo rows
// [T][K] with a per-token power-of-two exponent (launch_qgemm_act), the
// weight scale from a bound of |w| (launch_qgemm_wbound).
struct QgemmCall {
  int type = 0;
  int K = 0;
  GemvMat mats[4];
  int nmats = 0;
  int T = 0;
  const void* xhi = nullptr;   // __half [T][K]
  const void* xlo = nullptr;   // __half [T][K] (split)
  const float* xexp = nullptr; // [T]
  long long y_stride = 0;
  int epi = 0;                 // 0 store, 1 add, 2 SwiGLU (mats[0] gate, mats[1] up -> mats[0].y)
  const float* wbound = nullptr;
  int* err = nullptr;
  bool split = true;           // hi/lo fp16 operand pairs (three MMAs) for fp32-level results
  float* ws = nullptr;         // split-K workspace (qgemm_ws_bytes(); null: no split K)
  int* tickets = nullptr;      // split-K tickets (QGEMM_TICKETS ints, zeroed once)
};
constexpr int QGEMM_TICKETS = 256;
size_t qgemm_ws_bytes();
bool qgemm_supported(int type);
// token tile of the GEMM for T columns, and T rounded up to whole tiles (the
// activation buffers hold that many rows)
int qgemm_bn(int T);
int qgemm_rows_padded(int T);
int launch_qgemm(const QgemmCall& c, cudaStream_t st, bool pdl);
int launch_qgemm_act(const float* x, long long x_stride, int K, int T, int pro, const float* pro_w,
                     const float* pro_z, int group, float eps, __half* xhi, __half* xlo, float* xexp,
                     cudaStream_t st, bool pdl);
// bound of |w| over a matrix into *out (reset: start from 0, else fold in with max)
int launch_qgemm_wbound(int type, const void* W, long long rows, int K, float* out, cudaStream_t st, bool reset);
// a batched GemvCall (nb >= 16, store / add epilogue, plain or RMSNorm input)
// on the tensor-core GEMM with stream-ordered scratch; returns 1 when the
// call does not fit that path
int qgemm_from_gemv(const GemvCall& c, cudaStream_t st);
// Q6_K -> the engine-internal 16-row-group layout T_Q6_KR (same byte count)
int launch_repack_q6k(const void* src, void* dst, int rows, int inner, cudaStream_t st);
int launch_dequant(int type, const void* src, long long n, float* dst, cudaStream_t st);
// Q8_K helpers of the compatibility tier (q8k.cu)
int launch_quantize_q8k(const float* x, void* y, long long nblocks, cudaStream_t st);
int launch_vec_dot_q8k(int type, const void* x, const void* y, int nb, float* out, cudaStream_t st);
// q*_gemv with the reference C kernels' numerics (Q8_K activations for the
// K-quants, AVX2 lane order); y8 holds inner / 256 block_q8_K of scratch
int launch_ref_gemv(int type, const void* W, const float* x, void* y8, int inner, int rows, float* out,
                    cudaStream_t st);
struct GdnParams;
struct AttnParams;
// fused [in_proj | attn_gate] GEMV + GDN step (fused_gdn.cu); Wperm holds the
// head-regrouped rows [q_h | k_h | v_h | z_h] x nv
int launch_fused_inproj_gdn(const void* Wperm, int H, const float* x, const float* attn_norm, float eps,
                            const GdnParams& g, float* z, int* err, cudaStream_t st, bool pdl);

// chunked prefill (prefill.cu): tokens per chunk = the batched GEMV's columns
constexpr int PF_MAX_T = 128;
// chunks of at least this many tokens run their products on the tensor-core
// GEMM (qgemm_tc.cu) and the GDN as token-parallel prep + recurrence;
// shorter chunks use the batched GEMV and the chunk-sequential GDN kernel
constexpr int PF_TC_MIN_T = 16;
constexpr int GEMM_TC_MIN_T = 4;     // batched products on the tcgen05 GEMM from this many columns
struct GdnParams;
struct AttnParams;
int launch_gdn_chunk(const GdnParams& p, int T, cudaStream_t st);
// the delta-rule recurrence of T steps (gdn_seq.cu): q, k [T][H][128], v, y
// [T][H][dv], beta, g [T][H], S [H][dv][128]
int launch_gdn_seq(int T, int n_heads, int dv, const float* q, const float* k, const float* v, const float* beta,
                   const float* g, float* S, float* y, cudaStream_t st);
// Prefill form of the GDN step for T tokens: per-token projections' conv,
// gates and norms in parallel over (token, head) into the scratch rows
// (qn, kn [T][nv][128], vv [T][nv][dv], beta, g [T][nv]), the conv ring and
// step counter update, then the sequential recurrence (launch_gdn_seq)
struct GdnScratch {
  float *qn, *kn, *vv, *beta, *g;
};
int launch_gdn_prefill(const GdnParams& p, int T, const GdnScratch& s, cudaStream_t st);
int launch_attn_chunk(const AttnParams& p, int pos0, int T, cudaStream_t st);

// sampler parameters (sample.cu; InfernoSampling without the ABI padding)
struct SampleArgs {
  float temperature, top_p, min_p, presence, repetition;
  int top_k;
  unsigned long long seed;
};
int launch_sample(const float* logits, int V, const SampleArgs& a, const uint8_t* seen, float u, const int* step,
                  int* out_tok, unsigned long long* out_key, uint8_t* mark_seen, cudaStream_t st, bool pdl);
int launch_moe_topk(const float* logits, int E, int K, int* idx, float* wts, int* err, int ebase, int eloc,
                    cudaStream_t st, bool pdl);
int launch_moe_combine(float* x, const float* y, const float* wts, const int* idx, int K, int H, int shared,
                       int add_x, cudaStream_t st, bool pdl);
// expert-parallel combine into the residual exchange (sync point k)
struct MoeXch {
  unsigned long long* parts[8];
  const unsigned long long* seq;
  int n, rank, k;
};
int launch_moe_combine_xch(const float* y, const float* wts, const int* idx, int K, int H, int shared,
                           const MoeXch& xc, cudaStream_t st, bool pdl);
// RoPE tables cos / sin [ctx][rd/2] (src/ModelCPU.jl:134-153: inv_freq in
// Float64 rounded to Float32, angle in Float32, correctly rounded cos / sin)
void build_rope(int ctx, int rd, float theta, std::vector<float>& cs, std::vector<float>& sn);
// positions per split-K attention CTA for a cache of max_ctx positions (a
// multiple of 32 giving at most 128 splits)
int attn_split_len(int max_ctx);
int launch_embed_row(int type, const void* W, long long row_bytes, int inner, const int* row_ptr, float* dst,
                     int vocab, cudaStream_t st, bool pdl, int nrows = 1);

// device error word of the library (per device)
int* device_error_word(int device);

}  // namespace inf
