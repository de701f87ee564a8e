// C ABI: error channel, device-pointer tier and the QuantizedKernels.jl
// compatibility tier (same symbols and signatures as the reference's
// src/kernels/quant_kernels.c, so the .so can stand in for
// libquant_kernels.so at QuantizedKernels.LIBQUANT_PATH).
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <unordered_map>
#include <vector>
#include "internal.h"
#include "gemv.cuh"
#include "../../include/inferno_b200.h"

namespace inf {

namespace {
thread_local std::string g_last_error;
std::mutex g_mu;
int g_sms[64] = {};
int* g_err_word[64] = {};
}  // namespace

int set_error(int code, const char* fmt, ...) {
  char buf[1024];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof buf, fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}
const char* last_error() { return g_last_error.c_str(); }

int num_sms(int device) {
  if (device < 0 || device >= 64) return 148;
  if (!g_sms[device]) {
    int v = 0;
    cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, device);
    g_sms[device] = v > 0 ? v : 148;
  }
  return g_sms[device];
}

int* device_error_word(int device) {
  std::lock_guard<std::mutex> lk(g_mu);
  if (device < 0 || device >= 64) return nullptr;
  if (!g_err_word[device]) {
    int* p = nullptr;
    if (cudaMalloc(&p, sizeof(int)) != cudaSuccess) return nullptr;
    cudaMemset(p, 0, sizeof(int));
    g_err_word[device] = p;
  }
  return g_err_word[device];
}

// ---------------------------------------------------------------------------
// compatibility tier state: device copies of host weight arrays, keyed by the
// host pointer and size (Julia keeps its weight arrays alive and immutable),
// plus staging for x / y.  One mutex: the reference's C kernels are also not
// meant to be called concurrently on one scratch pool.
// ---------------------------------------------------------------------------
struct CompatState {
  bool init = false;
  int device = 0;
  cudaStream_t stream = nullptr;
  struct W { void* dev; size_t bytes; uint64_t sig; };
  std::unordered_map<const void*, W> weights;
  float* dx = nullptr; size_t dx_cap = 0;
  float* dy = nullptr; size_t dy_cap = 0;
  uint8_t* db = nullptr; size_t db_cap = 0;   // block bytes of the Q8_K helpers
};
CompatState g_compat;
std::mutex g_compat_mu;

static uint64_t sig_of(const uint8_t* p, size_t n) {
  // cheap content signature: size + first/last 64 bytes (FNV-1a)
  uint64_t h = 1469598103934665603ull ^ n;
  size_t k = n < 64 ? n : 64;
  for (size_t i = 0; i < k; ++i) h = (h ^ p[i]) * 1099511628211ull;
  for (size_t i = n - k; i < n; ++i) h = (h ^ p[i]) * 1099511628211ull;
  return h;
}

static int compat_init() {
  if (g_compat.init) return 0;
  int dev = 0;
  const char* e = getenv("INFERNO_B200_DEVICE");
  if (e) dev = atoi(e);
  INF_CUDA_TRY(cudaSetDevice(dev));
  INF_CUDA_TRY(cudaStreamCreateWithFlags(&g_compat.stream, cudaStreamNonBlocking));
  g_compat.device = dev;
  g_compat.init = true;
  return 0;
}

static int compat_weight(const uint8_t* host, size_t bytes, const void** dev) {
  uint64_t s = sig_of(host, bytes);
  auto it = g_compat.weights.find(host);
  if (it != g_compat.weights.end() && it->second.bytes == bytes && it->second.sig == s) {
    *dev = it->second.dev;
    return 0;
  }
  if (it != g_compat.weights.end()) {
    cudaFree(it->second.dev);
    g_compat.weights.erase(it);
  }
  void* d = nullptr;
  INF_CUDA_TRY(cudaMalloc(&d, (bytes + 15) / 16 * 16));
  INF_CUDA_TRY(cudaMemcpyAsync(d, host, bytes, cudaMemcpyHostToDevice, g_compat.stream));
  g_compat.weights[host] = {d, bytes, s};
  *dev = d;
  return 0;
}

static int grow(float** p, size_t* cap, size_t n) {
  if (*cap >= n) return 0;
  if (*p) cudaFree(*p);
  *p = nullptr;
  INF_CUDA_TRY(cudaMalloc(p, n * sizeof(float)));
  *cap = n;
  return 0;
}

static int grow_bytes(uint8_t** p, size_t* cap, size_t n) {
  if (*cap >= n) return 0;
  if (*p) cudaFree(*p);
  *p = nullptr;
  INF_CUDA_TRY(cudaMalloc(p, n));
  *cap = n;
  return 0;
}

static int compat_gemv(int type, const uint8_t* W, const float* x, float* out, int inner, int outer) {
  std::lock_guard<std::mutex> lk(g_compat_mu);
  int rc;
  if ((rc = compat_init())) return rc;
  INF_CUDA_TRY(cudaSetDevice(g_compat.device));
  if (inner <= 0 || outer <= 0) return set_error(-1, "compat gemv: bad dims %d x %d", outer, inner);
  const size_t bytes = (size_t)outer * (inner / qk_of(type)) * bb_of(type);
  const void* dW;
  if ((rc = compat_weight(W, bytes, &dW))) return rc;
  if ((rc = grow(&g_compat.dx, &g_compat.dx_cap, inner))) return rc;
  if ((rc = grow(&g_compat.dy, &g_compat.dy_cap, outer))) return rc;
  INF_CUDA_TRY(cudaMemcpyAsync(g_compat.dx, x, (size_t)inner * 4, cudaMemcpyHostToDevice, g_compat.stream));
  const char* fp32 = getenv("INFERNO_COMPAT_FP32");
  if (!(fp32 && fp32[0] == '1') && type != T_IQ2_XXS && type != T_F32) {
    // default: the replaced library's numerics, bit for bit
    if (type != T_Q8_0 && (rc = grow_bytes(&g_compat.db, &g_compat.db_cap, (size_t)(inner / 256) * 292)))
      return rc;
    if ((rc = launch_ref_gemv(type, dW, g_compat.dx, g_compat.db, inner, outer, g_compat.dy, g_compat.stream)))
      return rc;
    INF_CUDA_TRY(cudaMemcpyAsync(out, g_compat.dy, (size_t)outer * 4, cudaMemcpyDeviceToHost, g_compat.stream));
    INF_CUDA_TRY(cudaStreamSynchronize(g_compat.stream));
    return 0;
  }
  GemvCall c;
  c.type = type;
  c.inner = inner;
  c.mats[0] = {dW, g_compat.dy, outer};
  c.nmats = 1;
  c.x = g_compat.dx;
  if ((rc = launch_gemv(c, g_compat.stream, false))) return rc;
  INF_CUDA_TRY(cudaMemcpyAsync(out, g_compat.dy, (size_t)outer * 4, cudaMemcpyDeviceToHost, g_compat.stream));
  INF_CUDA_TRY(cudaStreamSynchronize(g_compat.stream));
  return 0;
}

// quantize_row_q8_K on the device: host x[k] -> host block_q8_K[k / 256]
static int compat_quantize_q8k(const float* x, void* y, int64_t k) {
  std::lock_guard<std::mutex> lk(g_compat_mu);
  int rc;
  // QuantizedKernels.jl:151-152 passes k as a Cint, so the upper half of the
  // 64-bit argument is not defined there: read the low 32 bits in that case
  if (k < 0 || k > 0x7fffffffLL) k = (int64_t)(uint32_t)k;
  if (!x || !y) return set_error(INFERNO_EINVAL, "quantize_row_q8_K: null pointer");
  if (k < 0 || k % 256) return set_error(INFERNO_EINVAL, "quantize_row_q8_K: k = %lld is not a multiple of 256",
                                         (long long)k);
  if (!k) return 0;
  if ((rc = compat_init())) return rc;
  INF_CUDA_TRY(cudaSetDevice(g_compat.device));
  const size_t ybytes = (size_t)(k / 256) * 292;
  if ((rc = grow(&g_compat.dx, &g_compat.dx_cap, (size_t)k))) return rc;
  if ((rc = grow_bytes(&g_compat.db, &g_compat.db_cap, ybytes))) return rc;
  INF_CUDA_TRY(cudaMemcpyAsync(g_compat.dx, x, (size_t)k * 4, cudaMemcpyHostToDevice, g_compat.stream));
  if ((rc = launch_quantize_q8k(g_compat.dx, g_compat.db, k / 256, g_compat.stream))) return rc;
  INF_CUDA_TRY(cudaMemcpyAsync(y, g_compat.db, ybytes, cudaMemcpyDeviceToHost, g_compat.stream));
  INF_CUDA_TRY(cudaStreamSynchronize(g_compat.stream));
  return 0;
}

// one block-row dot product x (weight blocks) . y (Q8_K or Q8_0 blocks), host pointers
static int compat_vec_dot(int type, const void* x, const void* y, int nb, float* out) {
  std::lock_guard<std::mutex> lk(g_compat_mu);
  int rc;
  *out = 0.0f;
  if (nb < 0 || (nb && (!x || !y))) return set_error(INFERNO_EINVAL, "vec_dot: bad arguments (nb = %d)", nb);
  if (!nb) return 0;
  if ((rc = compat_init())) return rc;
  INF_CUDA_TRY(cudaSetDevice(g_compat.device));
  const size_t xb = (size_t)nb * bb_of(type), yb = (size_t)nb * (type == T_Q8_0 ? 34 : 292);
  const size_t yoff = (xb + 15) / 16 * 16;
  if ((rc = grow_bytes(&g_compat.db, &g_compat.db_cap, yoff + yb))) return rc;
  if ((rc = grow(&g_compat.dy, &g_compat.dy_cap, 1))) return rc;
  INF_CUDA_TRY(cudaMemcpyAsync(g_compat.db, x, xb, cudaMemcpyHostToDevice, g_compat.stream));
  INF_CUDA_TRY(cudaMemcpyAsync(g_compat.db + yoff, y, yb, cudaMemcpyHostToDevice, g_compat.stream));
  if ((rc = launch_vec_dot_q8k(type, g_compat.db, g_compat.db + yoff, nb, g_compat.dy, g_compat.stream))) return rc;
  INF_CUDA_TRY(cudaMemcpyAsync(out, g_compat.dy, 4, cudaMemcpyDeviceToHost, g_compat.stream));
  INF_CUDA_TRY(cudaStreamSynchronize(g_compat.stream));
  return 0;
}

static float compat_dot_report(int type, const void* x, const void* y, int nb, const char* what) {
  float r = 0.0f;
  if (compat_vec_dot(type, x, y, nb, &r)) {
    fprintf(stderr, "libinferno_b200: %s: %s\n", what, last_error());
    return NAN;
  }
  return r;
}

}  // namespace inf

using namespace inf;

extern "C" {

const char* inferno_last_error(void) { return inf::last_error(); }
int inferno_version(void) { return INFERNO_B200_VERSION; }

int inferno_device_error(int device, int clear) {
  int* w = device_error_word(device);
  if (!w) return set_error(INFERNO_ECUDA, "no device error word");
  int v = 0;
  if (cudaMemcpy(&v, w, sizeof v, cudaMemcpyDeviceToHost) != cudaSuccess)
    return set_error(INFERNO_ECUDA, "reading device error word failed");
  if (clear) cudaMemset(w, 0, sizeof(int));
  return v;
}

int inferno_dequantize(int ggml_type, const void* src, int64_t n, float* dst, void* stream) {
  if (!src || !dst || n < 0) return set_error(INFERNO_EINVAL, "dequantize: null pointer or negative size");
  if (!type_supported(ggml_type)) return set_error(INFERNO_EINVAL, "dequantize: unsupported ggml type %d", ggml_type);
  if (n % (ggml_type == T_Q8_0 || ggml_type == T_F32 ? 32 : 256))
    return set_error(INFERNO_EINVAL, "dequantize: %lld elements not a whole number of blocks", (long long)n);
  int rc = launch_dequant(ggml_type, src, n, dst, (cudaStream_t)stream);
  return rc ? set_error(INFERNO_ECUDA, "dequantize launch failed") : 0;
}

int inferno_gemv(int ggml_type, const void* W, const float* x, float* y, int inner, int outer, int batch,
                 void* stream) {
  if (!W || !x || !y) return set_error(INFERNO_EINVAL, "gemv: null pointer");
  if (outer < 0 || batch < 1) return set_error(INFERNO_EINVAL, "gemv: bad outer/batch");
  GemvCall c;
  c.type = ggml_type;
  c.inner = inner;
  c.mats[0] = {W, y, outer};
  c.nmats = 1;
  c.nb = batch;
  c.x = x;
  c.x_stride = inner;
  c.y_stride = outer;
  return launch_gemv(c, (cudaStream_t)stream, false);
}

int inferno_gemv_ex(int ggml_type, const void* W, const float* x, float* y, int inner, int outer, int batch,
                    int prologue, const float* norm_w, float eps, int epilogue, unsigned long long* argmax,
                    int force_rows_per_warp, void* stream) {
  if (!W || !x) return set_error(INFERNO_EINVAL, "gemv_ex: null pointer");
  GemvCall c;
  c.type = ggml_type;
  c.inner = inner;
  c.mats[0] = {W, y, outer};
  c.nmats = 1;
  c.nb = batch;
  c.x = x;
  c.x_stride = inner;
  c.y_stride = outer;
  c.pro = prologue;
  c.pro_w = norm_w;
  c.eps = eps;
  c.epi = epilogue;
  c.argmax = argmax;
  c.force_r = force_rows_per_warp;
  if (prologue == PRO_RMSNORM && !norm_w) return set_error(INFERNO_EINVAL, "gemv_ex: RMSNorm needs a weight");
  if (epilogue == EPI_ARGMAX && !argmax) return set_error(INFERNO_EINVAL, "gemv_ex: argmax output missing");
  if (epilogue == EPI_SWIGLU) return set_error(INFERNO_EINVAL, "gemv_ex: use inferno_gemv_swiglu");
  return launch_gemv(c, (cudaStream_t)stream, false);
}

int inferno_gemv_swiglu(int ggml_type, const void* Wg, const void* Wu, const float* x, float* h, int inner,
                        int rows, int batch, const float* norm_w, float eps, void* stream) {
  GemvCall c;
  c.type = ggml_type;
  c.inner = inner;
  c.mats[0] = {Wg, h, rows};
  c.mats[1] = {Wu, nullptr, rows};
  c.nmats = 2;
  c.nb = batch;
  c.x = x;
  c.x_stride = inner;
  c.y_stride = rows;
  c.pro = norm_w ? PRO_RMSNORM : PRO_NONE;
  c.pro_w = norm_w;
  c.eps = eps;
  c.epi = EPI_SWIGLU;
  return launch_gemv(c, (cudaStream_t)stream, false);
}

// ---- compatibility tier (void returns, as in the reference) -----------------
// Numerics note: the reference quantizes x to Q8_K and does integer dots
// (quant_kernels.c:166-306); these run the engine's fp32-activation kernel.
// The q8 scratch argument is accepted and ignored.
static void compat_report(int rc, const char* fn) {
  if (rc) fprintf(stderr, "[inferno_b200] %s failed: %s\n", fn, inf::last_error());
}
void q4_k_gemv(const uint8_t* weight, const float* x, float* out, void* q8_buf, int inner_dim, int outer_dim) {
  (void)q8_buf;
  compat_report(compat_gemv(T_Q4_K, weight, x, out, inner_dim, outer_dim), "q4_k_gemv");
}
void q5_k_gemv(const uint8_t* weight, const float* x, float* out, void* q8_buf, int inner_dim, int outer_dim) {
  (void)q8_buf;
  compat_report(compat_gemv(T_Q5_K, weight, x, out, inner_dim, outer_dim), "q5_k_gemv");
}
void q6_k_gemv(const uint8_t* weight, const float* x, float* out, void* q8_buf, int inner_dim, int outer_dim) {
  (void)q8_buf;
  compat_report(compat_gemv(T_Q6_K, weight, x, out, inner_dim, outer_dim), "q6_k_gemv");
}
void q8_0_gemv(const uint8_t* weight, const float* x, float* out, int inner_dim, int outer_dim) {
  compat_report(compat_gemv(T_Q8_0, weight, x, out, inner_dim, outer_dim), "q8_0_gemv");
}

void quantize_row_q8_K(const float* x, void* y, int64_t k) {
  compat_report(compat_quantize_q8k(x, y, k), "quantize_row_q8_K");
}
float vec_dot_q4_K_q8_K(const void* x, const void* y, int nb) {
  return compat_dot_report(T_Q4_K, x, y, nb, "vec_dot_q4_K_q8_K");
}
float vec_dot_q5_K_q8_K(const void* x, const void* y, int nb) {
  return compat_dot_report(T_Q5_K, x, y, nb, "vec_dot_q5_K_q8_K");
}
float vec_dot_q6_K_q8_K(const void* x, const void* y, int nb) {
  return compat_dot_report(T_Q6_K, x, y, nb, "vec_dot_q6_K_q8_K");
}
float vec_dot_q8_0_q8_0(const void* x, const void* y, int nb) {
  return compat_dot_report(T_Q8_0, x, y, nb, "vec_dot_q8_0_q8_0");
}

int inferno_compat_release(void) {
  std::lock_guard<std::mutex> lk(g_compat_mu);
  if (!g_compat.init) return 0;
  cudaSetDevice(g_compat.device);
  for (auto& kv : g_compat.weights) cudaFree(kv.second.dev);
  g_compat.weights.clear();
  if (g_compat.dx) cudaFree(g_compat.dx);
  if (g_compat.dy) cudaFree(g_compat.dy);
  if (g_compat.db) cudaFree(g_compat.db);
  g_compat.dx = g_compat.dy = nullptr;
  g_compat.db = nullptr;
  g_compat.dx_cap = g_compat.dy_cap = g_compat.db_cap = 0;
  return 0;
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Failure-path check of the tensor-parallel exchange reader on one GPU: the
// tensor-core GEMV runs in reader mode (RMSNorm prologue that polls the
// ranks' tagged partials) against two "peer" partial buffers that nothing
// writes, so every tag stays stale; with a poll limit of spin_limit per word
// the kernel must record DERR_MBAR_TIMEOUT, skip the remaining waits and
// return.  No reference counterpart (the reference has no multi-GPU path).
// ---------------------------------------------------------------------------
extern "C" int inferno_debug_xch_timeout(int spin_limit, int* device_error_out) {
  if (spin_limit <= 0 || spin_limit > (1 << 22))
    return set_error(INFERNO_EINVAL, "debug_xch_timeout: spin_limit must be in [1, 2^22]");
  constexpr int H = 1024, ROWS = 64, NR = 2;
  const size_t wbytes = (size_t)ROWS * (H / 256) * 144;
  // [W][x][norm w][y][partials 2 x NR x H words][seq 8 words][x_next][error word]
  const size_t bytes = wbytes + 4 * H * 3 + 8 * (size_t)2 * NR * H + 8 * 8 + 4 * H + 256;
  uint8_t* buf = nullptr;
  INF_CUDA_TRY(cudaMalloc(&buf, bytes));
  cudaError_t e = cudaMemset(buf, 0, bytes);   // Q4_K blocks with d = dmin = 0, x = 0, tags 0
  int rc = 0;
  if (e != cudaSuccess) rc = set_error(INFERNO_ECUDA, "debug_xch_timeout: %s", cudaGetErrorString(e));
  uint8_t* q = buf + wbytes;
  float* x = (float*)q;
  float* normw = x + H;
  float* y = normw + H;
  unsigned long long* parts = (unsigned long long*)(y + H);
  unsigned long long* seq = parts + 2 * NR * H;   // sequence base 0: the expected tag is 1
  float* x_next = (float*)(seq + 8);
  int* err = (int*)(x_next + H);
  if (!rc) {
    GemvCall c;
    c.type = T_Q4_K;
    c.inner = H;
    c.mats[0] = {buf, y, ROWS};
    c.nmats = 1;
    c.x = x;
    c.x_stride = H;
    c.pro = PRO_RMSNORM;
    c.pro_w = normw;
    c.err = err;
    c.xch_n = NR;
    c.xch_rank = 0;
    c.xch_rk = 0;
    c.xch_spin = (unsigned)spin_limit;
    c.xch_seq = seq;
    c.xch_parts[0] = parts;
    c.xch_parts[1] = parts;
    c.x_next = x_next;
    rc = launch_gemv(c, (cudaStream_t)0, false);
  }
  int h = 0;
  if (!rc) {
    e = cudaDeviceSynchronize();
    if (e == cudaSuccess) e = cudaMemcpy(&h, err, 4, cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) rc = set_error(INFERNO_ECUDA, "debug_xch_timeout: %s", cudaGetErrorString(e));
  }
  cudaFree(buf);
  if (rc) return rc;
  if (device_error_out) *device_error_out = h;
  return h ? set_error(INFERNO_EDEVICE, "exchange reader timed out (device error %d)", h) : 0;
}
