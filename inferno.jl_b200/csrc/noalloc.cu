// Host-pointer GEMV that never allocates device memory.
//
// inferno_gemv_host_noalloc is the allocation-free sibling of the
// compatibility GEMVs (q4_k_gemv & co. in api.cu).  Those upload the weight
// matrix and stage x / y in device buffers they cudaMalloc on first use.  Some
// callers cannot allow that: a host runtime that owns the device allocator
// (or a pool with a hard budget) and forbids other libraries from calling
// cudaMalloc behind its back, or a plugin sandbox with no allocation rights.
// This entry point stages the weight, x and y in one file-scope device array
// instead, sized at compile time and held by every GPU that loads the library
// until the process exits.
//
// Numerics are those of q*_gemv: the replaced library's Q8_K path by
// default, fp32 activations with INFERNO_COMPAT_FP32=1 (and always for
// IQ2_XXS / F32).  It runs on the calling thread's current CUDA device (the
// compatibility entries pick INFERNO_B200_DEVICE instead).
//
// Limits and sharing rules (also in include/inferno_b200.h):
//  * weight + x + y (each rounded up to 256 bytes) must fit in
//    INFERNO_NOALLOC_SCRATCH_BYTES; larger requests fail with INFERNO_EINVAL;
//  * the array is shared by every call on a device and keeps the last call's
//    contents; calls are serialised by a host mutex and are synchronous, but
//    work that another thread or library enqueues on the same array would
//    race with it;
//  * the first call on a device looks up the array's device address
//    (cudaGetSymbolAddress); make that first call before any stream capture.
#include <mutex>
#include "internal.h"
#include "gemv.cuh"
#include "../../include/inferno_b200.h"

namespace inf {
namespace {

constexpr size_t kScratchBytes = INFERNO_NOALLOC_SCRATCH_BYTES;
static __device__ __align__(256) unsigned char g_noalloc_scratch[kScratchBytes];

std::mutex g_noalloc_mu;
void* g_noalloc_ptr[64] = {};   // device address of the array, per device

size_t up256(size_t n) { return (n + 255) / 256 * 256; }

}  // namespace
}  // namespace inf

using namespace inf;

extern "C" int inferno_gemv_host_noalloc(int ggml_type, const uint8_t* weight, const float* x, float* out,
                                         int inner_dim, int outer_dim) {
  if (!weight || !x || !out) return set_error(INFERNO_EINVAL, "gemv_host_noalloc: null pointer");
  if (!type_supported(ggml_type)) return set_error(INFERNO_EINVAL, "gemv_host_noalloc: unsupported type %d", ggml_type);
  if (inner_dim <= 0 || outer_dim <= 0 || inner_dim % qk_of(ggml_type) || (ggml_type == T_F32 && inner_dim % 32))
    return set_error(INFERNO_EINVAL, "gemv_host_noalloc: bad dims %d x %d", outer_dim, inner_dim);
  // the numerics of q*_gemv: the replaced library's Q8_K path unless
  // INFERNO_COMPAT_FP32=1 (IQ2_XXS and F32 have no q*_gemv and always take
  // the fp32-activation GEMV)
  const char* fp32 = getenv("INFERNO_COMPAT_FP32");
  const bool ref_numerics = !(fp32 && fp32[0] == '1') && ggml_type != T_IQ2_XXS && ggml_type != T_F32;
  const size_t wbytes = (size_t)outer_dim * (inner_dim / qk_of(ggml_type)) * bb_of(ggml_type);
  // layout in the array: [error word][x][y][Q8_K blocks of x][weight]
  const size_t off_x = 256, off_y = off_x + up256((size_t)inner_dim * 4);
  const size_t off_q = off_y + up256((size_t)outer_dim * 4);
  const size_t qbytes = (ref_numerics && ggml_type != T_Q8_0) ? (size_t)(inner_dim / 256) * 292 : 0;
  const size_t off_w = off_q + up256(qbytes);
  const size_t need = off_w + up256(wbytes);
  if (need > kScratchBytes)
    return set_error(INFERNO_EINVAL,
                     "gemv_host_noalloc: %zu bytes of weights and vectors exceed the %zu-byte static scratch; "
                     "use q*_gemv / inferno_gemv for larger matrices",
                     need, kScratchBytes);
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  int dev = 0;
  INF_CUDA_TRY(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64) return set_error(INFERNO_EINVAL, "gemv_host_noalloc: device %d out of range", dev);
  if (!g_noalloc_ptr[dev]) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || !p)
      return set_error(INFERNO_ECUDA, "gemv_host_noalloc: cudaGetSymbolAddress failed: %s", cudaGetErrorString(e));
    g_noalloc_ptr[dev] = p;
  }
  unsigned char* base = (unsigned char*)g_noalloc_ptr[dev];
  int* err = (int*)base;
  float* dx = (float*)(base + off_x);
  float* dy = (float*)(base + off_y);
  void* dq = base + off_q;
  void* dw = base + off_w;
  // the error word must start at zero; x, y, the Q8_K blocks and the weight
  // are fully rewritten by every call
  INF_CUDA_TRY(cudaMemset(err, 0, sizeof(int)));
  INF_CUDA_TRY(cudaMemcpy(dw, weight, wbytes, cudaMemcpyHostToDevice));
  INF_CUDA_TRY(cudaMemcpy(dx, x, (size_t)inner_dim * 4, cudaMemcpyHostToDevice));
  int rc;
  if (ref_numerics) {
    rc = launch_ref_gemv(ggml_type, dw, dx, dq, inner_dim, outer_dim, dy, (cudaStream_t)0);
  } else {
    GemvCall c;
    c.type = ggml_type;
    c.inner = inner_dim;
    c.mats[0] = {dw, dy, outer_dim};
    c.nmats = 1;
    c.x = dx;
    c.x_stride = inner_dim;
    c.err = err;
    rc = launch_gemv(c, (cudaStream_t)0, false);
  }
  if (rc) return rc;
  INF_CUDA_TRY(cudaMemcpy(out, dy, (size_t)outer_dim * 4, cudaMemcpyDeviceToHost));
  int h_err = 0;
  INF_CUDA_TRY(cudaMemcpy(&h_err, err, sizeof(int), cudaMemcpyDeviceToHost));
  if (h_err) return set_error(INFERNO_EDEVICE, "gemv_host_noalloc: kernel reported device error %d", h_err);
  return 0;
}
