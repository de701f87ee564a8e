/*
 * inferno_b200.h -- C ABI of libinferno_b200.so, the sm_100a decode engine
 * for Inferno.jl's Qwen3.5 hybrid models.
 *
 * Every entry is extern "C" with plain pointers and sizes.  Functions return
 * an int status (0 = OK, negative = error) unless noted; the message of the
 * last error on the calling thread is inferno_last_error().  Citations give
 * the reference interface (Inferno.jl source tree) each entry replaces.
 *
 * Three tiers:
 *   1. compatibility: the exact symbols of src/kernels/quant_kernels.c, so the
 *      library can be dropped in at QuantizedKernels.LIBQUANT_PATH;
 *   2. device kernels: dequantize / GEMV on device pointers;
 *   3. engine: the model lives on the GPU; the host calls per layer
 *      (`layer(x, pos, rope, cache)`) or per token / per decode loop.
 */
#ifndef INFERNO_B200_H
#define INFERNO_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define INFERNO_B200_VERSION 1

/* status codes */
#define INFERNO_OK 0
#define INFERNO_EINVAL (-1)  /* bad argument                               */
#define INFERNO_ECUDA (-2)   /* CUDA runtime / launch error                 */
#define INFERNO_ENOMEM (-3)  /* device allocation failed                    */
#define INFERNO_ESTATE (-4)  /* call not valid in the engine's state        */
#define INFERNO_EDEVICE (-5) /* a kernel reported an error (timeout, ...)   */
#define INFERNO_ENCCL (-6)   /* NCCL error                                  */
#define INFERNO_ENOTFOUND (-7) /* metadata key not present                   */
#define INFERNO_EFORMAT (-8) /* malformed GGUF file                         */

/* ggml type ids accepted (GGUF spec; src/GGUF.jl:25-60) */
#define INFERNO_F32 0
#define INFERNO_Q8_0 8
#define INFERNO_Q4_K 12
#define INFERNO_Q5_K 13
#define INFERNO_Q6_K 14
#define INFERNO_IQ2_XXS 16

/* thread-local message of the last failing call on this thread */
const char* inferno_last_error(void);
int inferno_version(void);
/* device-side error word (1 = a bounded wait timed out); clear != 0 resets it */
int inferno_device_error(int device, int clear);

/* ======================= 1. compatibility tier ===========================
 * Same names and signatures as src/kernels/quant_kernels.c:602-697, bound by
 * the ccalls at src/QuantizedKernels.jl:88-90, 106-108, 125-127, 141-143.
 * Host pointers in, host results out (each call copies x in and y out; a
 * weight array is uploaded on first sight and cached by host pointer, size
 * and a content signature).  Numerics: by default those of the replaced
 * library, bit for bit (x quantized to Q8_K on the device, the AVX2 build's
 * lane and fma order; Q8_0 with fp32 x); with INFERNO_COMPAT_FP32=1 in the
 * environment, fp32 activations through the engine's GEMV.  q8_buf is
 * accepted and not written.  void returns as in
 * the reference; failures are printed to stderr and kept in
 * inferno_last_error(). */
void q4_k_gemv(const uint8_t* weight, const float* x, float* out, void* q8_buf, int inner_dim, int outer_dim);
void q5_k_gemv(const uint8_t* weight, const float* x, float* out, void* q8_buf, int inner_dim, int outer_dim);
void q6_k_gemv(const uint8_t* weight, const float* x, float* out, void* q8_buf, int inner_dim, int outer_dim);
void q8_0_gemv(const uint8_t* weight, const float* x, float* out, int inner_dim, int outer_dim);
/* The Q8_K helpers QuantizedKernels.jl also binds (QuantizedKernels.jl:148-175,
 * replacing quant_kernels.c:166-196, :204-519, :531-559), computed on the
 * device from host pointers and bit-identical to the reference's AVX2 + FMA
 * build.  y of quantize_row_q8_K receives k / 256 blocks of 292 bytes
 * {float d; int8 qs[256]; int16 bsums[16]}.  x of vec_dot_* are nb weight
 * blocks, y nb block_q8_K (block_q8_0 for vec_dot_q8_0_q8_0).  A failing
 * vec_dot returns NaN; the message is in inferno_last_error(). */
void quantize_row_q8_K(const float* x, void* y, int64_t k);
float vec_dot_q4_K_q8_K(const void* x, const void* y, int nb);
float vec_dot_q5_K_q8_K(const void* x, const void* y, int nb);
float vec_dot_q6_K_q8_K(const void* x, const void* y, int nb);
float vec_dot_q8_0_q8_0(const void* x, const void* y, int nb);
/* frees the cached device copies of compatibility-tier weights */
int inferno_compat_release(void);

/* Allocation-free host-pointer GEMV: out[r] = sum_i W[r,i] * x[i] with the
 * numerics of q*_gemv above (the replaced library's Q8_K path by default,
 * fp32 activations with INFERNO_COMPAT_FP32=1; IQ2_XXS and F32, which have no
 * q*_gemv, always use fp32 activations), but it never calls cudaMalloc (or
 * any allocating routine).  It is for callers that cannot let a library
 * allocate device memory -- a host runtime that owns the device allocator or
 * enforces a hard memory budget, or a sandboxed plugin without allocation
 * rights.  This entry has no counterpart in the reference.
 * It runs on the calling thread's current CUDA device (unlike q*_gemv, which
 * select INFERNO_B200_DEVICE).  Weight, x, y and x's Q8_K blocks are staged
 * in one static device array of INFERNO_NOALLOC_SCRATCH_BYTES that every GPU
 * loading the library keeps until exit; their sum (each rounded up to 256 B,
 * plus 256 B) must fit, else INFERNO_EINVAL.  The array is shared by all
 * calls and keeps the last call's contents; calls are synchronous and
 * serialised by a mutex, but overlapping GPU work on the array from elsewhere
 * would race.  The first call on a device looks up the array's address; make
 * it before any stream capture.  Returns 0 or a negative status. */
#define INFERNO_NOALLOC_SCRATCH_BYTES (32u << 20)
int inferno_gemv_host_noalloc(int ggml_type, const uint8_t* weight, const float* x, float* out, int inner_dim,
                              int outer_dim);

/* ======================= 2. device kernel tier ============================
 * All pointers are device pointers; `stream` is a cudaStream_t (NULL = legacy
 * default stream).  Weight buffers hold GGUF blocks in native row-major layout
 * (src/QuantsCPU.jl:37-115): row r at byte r*(inner/QK)*block_bytes; they must
 * be 16-byte aligned and readable up to the next 16-byte boundary (true of
 * every cudaMalloc allocation). */

/* Bit-exact dequantization to fp32: replaces Dequant.dequantize_{q4_k,q5_k,
 * q6_k,q8_0,iq2_xxs} (src/Dequant.jl:12-54, 304-441, 558-601). */
int inferno_dequantize(int ggml_type, const void* src, int64_t n_elements, float* dst, void* stream);

/* y[b*outer + r] = sum_i W[r,i] * x[b*inner + i] for b < batch: replaces
 * ModelCPU.mul! on quantized weights (src/ModelCPU.jl:284-444). */
int inferno_gemv(int ggml_type, const void* W, const float* x, float* y, int inner, int outer, int batch,
                 void* stream);

/* GEMV with a fused prologue / epilogue:
 *   prologue 0 = none, 1 = RMSNorm(x; norm_w, eps) (src/ModelCPU.jl:110-122)
 *   epilogue 0 = store, 1 = y += W x (residual, src/ModelCPU.jl:880-889),
 *            3 = first-max argmax into argmax[b] as a packed 64-bit key
 *                (ordered-float << 32 | 0xffffffff - row); y may be NULL.
 *                argmax[] must be zeroed first (src/ModelCPU.jl:1123-1127).
 * force_rows_per_warp: 0 = planner's choice, else 1, 2 or 4 (tuning). */
int inferno_gemv_ex(int ggml_type, const void* W, const float* x, float* y, int inner, int outer, int batch,
                    int prologue, const float* norm_w, float eps, int epilogue, unsigned long long* argmax,
                    int force_rows_per_warp, void* stream);

/* h = silu(Wg x') * (Wu x') with x' = RMSNorm(x; norm_w) if norm_w != NULL:
 * the fused gate/up half of mlp_forward (src/ModelCPU.jl:447-473). */
int inferno_gemv_swiglu(int ggml_type, const void* Wg, const void* Wu, const float* x, float* h, int inner,
                        int rows, int batch, const float* norm_w, float eps, void* stream);

/* Gated delta-rule recurrence over T steps (the state
 * update of GatedDeltaNetCPU, src/ModelCPU.jl:640-674, without projections):
 * S_h = S_h*exp(g); S_h += beta*(v - S_h k) k^T; y = S_h q, per head and step.
 * Device pointers: q, k [T][n_heads][dk]; v, y [T][n_heads][dv];
 * beta, g [T][n_heads]; S [n_heads][dv][dk] fp32, updated in place.
 * dk = 128, dv % 16 == 0; q, k, S 16-byte aligned. */
int inferno_gdn_recurrence(int T, int n_heads, int dk, int dv, const float* q, const float* k, const float* v,
                           const float* beta, const float* g, float* S, float* y, void* stream);

/* One gated full-attention decode step of one layer at position pos: the
 * part of FullAttentionCPU after its q/k/v projections
 * (src/ModelCPU.jl:766-851): rmsnorm_rotary! of q and k (:187-231, NeoX
 * half-split RoPE on the first rope_dim dims, tables as :134-153),
 * update_kv_cache! (:245-258), flash_attention_cpu! per query head
 * (src/FlashAttention.jl:16-74, blocked GQA kv = h / (n_heads/n_kv_heads))
 * and the sigmoid gate (:846-851).  Device pointers: qg [n_heads][2*head_dim]
 * (q then gate per head, as the wq projection lays it out), k, v
 * [n_kv_heads][head_dim] (pre-norm), q_norm, k_norm [head_dim], caches
 * [max_ctx][n_kv_heads][head_dim] (rows < pos hold earlier positions; row pos
 * is written), out [n_heads][head_dim].  head_dim 256; split_len = positions
 * per split-K CTA (a multiple of 32; 0 = the engine's choice for max_ctx).
 * The call is synchronous on `stream` (it stages the RoPE rows and the split
 * scratch with stream-ordered allocation). */
int inferno_attention_step(const float* qg, const float* k, const float* v, const float* q_norm, const float* k_norm,
                           float eps, int n_heads, int n_kv_heads, int head_dim, int rope_dim, float rope_theta,
                           float* k_cache, float* v_cache, int max_ctx, int pos, int split_len, float* out,
                           void* stream);

/* The same recurrence in its chunked (WY / UT-transform) form for prefill:
 * chunks of `chunk` = 64 tokens, within a chunk the products are dense
 * matrices (K K^T, the unit-triangular solve, W = T diag(e^G) K, U = T V,
 * Q K^T) and only the 16-row blocks of S walk the chunks in order.  Same
 * arguments and layouts as inferno_gdn_recurrence (dk = 128, dv a multiple of
 * 16 up to 128); results agree with the sequential form to fp32 reordering.
 * Stream-ordered scratch of about T * n_heads * 1.3 KB. */
int inferno_gdn_chunked(int T, int n_heads, int dk, int dv, const float* q, const float* k, const float* v,
                        const float* beta, const float* g, float* S, float* y, int chunk, void* stream);

/* Sampling parameters of generate_cpu / softmax_sample
 * (src/ModelCPU.jl:1123-1225): temperature 0 = greedy. */
typedef struct InfernoSampling {
  float temperature;
  float top_p;               /* 1 = off */
  int32_t top_k;             /* 0 = off (the nucleus is then searched within the 1024 most probable tokens) */
  float min_p;               /* 0 = off; relative to the largest probability */
  float repetition_penalty;  /* 1 = off */
  float presence_penalty;    /* 0 = off */
  uint64_t seed;             /* Philox-4x32-10 key; the counter is the step */
} InfernoSampling;

/* Samples one token from device logits[vocab] with softmax_sample's
 * semantics; seen (device, vocab bytes, may be NULL) marks the tokens the
 * penalties apply to; u in [0, 1) is the uniform draw (u < 0: Philox(seed, 0)).
 * out_token is a device pointer. */
int inferno_sample_logits(const float* logits, int vocab, const InfernoSampling* s, const uint8_t* seen, float u,
                          int32_t* out_token, void* stream);

/* ======================= 3. engine tier ==================================== */

/* Model hyper-parameters, filled by the host from GGUF metadata
 * (LoaderCPU.get_config, src/LoaderCPU.jl:393-418; ssm dims per
 * src/LoaderCPU.jl:498-516 with nk taken from ssm.group_count). */
typedef struct InfernoConfig {
  int32_t struct_size;           /* sizeof(InfernoConfig) */
  int32_t device;                /* CUDA device ordinal */
  int32_t hidden_size;
  int32_t intermediate_size;     /* dense FFN (0 for MoE models) */
  int32_t num_layers;
  int32_t vocab_size;
  int32_t n_heads;               /* full-attention query heads */
  int32_t n_kv_heads;
  int32_t head_dim;
  int32_t ssm_nv;                /* Gated DeltaNet value heads (time_step_rank) */
  int32_t ssm_nk;                /* Gated DeltaNet q/k heads (group_count) */
  int32_t ssm_dk;                /* state_size */
  int32_t ssm_dv;                /* inner_size / nv */
  int32_t ssm_conv_kernel;
  int32_t max_ctx;               /* KV-cache capacity in positions */
  int32_t n_experts;             /* 0 = dense FFN */
  int32_t n_experts_used;
  int32_t expert_ffn;
  int32_t shared_expert_ffn;
  int32_t max_batch;             /* state slices for batched decode (0 or 1: one sequence) */
  float rms_eps;
  float rope_theta;
  float partial_rotary_factor;
  int32_t use_graphs;            /* capture the decode step in a CUDA graph */
  int32_t use_pdl;               /* programmatic dependent launch between kernels */
  int32_t tp_rank, tp_size;      /* tensor parallel (tp_size 1 = off) */
  const void* nccl_unique_id;    /* 128-byte ncclUniqueId when tp_size > 1 */
} InfernoConfig;

typedef struct InfernoEngine InfernoEngine;

int inferno_engine_create(const InfernoConfig* cfg, InfernoEngine** out);

/* Raw GGUF tensor bytes in native layout (the keep_quantized branch of
 * LoaderCPU.extract_tensor_cpu, src/LoaderCPU.jl:131-155), by GGUF name;
 * ne[] in GGUF order (ne[0] fastest), unused dims = 1. */
int inferno_engine_upload_tensor(InfernoEngine* eng, const char* name, int ggml_type, const int64_t ne[4],
                                 const void* host_bytes, size_t nbytes);

/* Binds uploaded tensors to layers (a layer is Gated DeltaNet iff
 * blk.i.ssm_a exists, src/LoaderCPU.jl:431), allocates state and builds the
 * RoPE table (src/ModelCPU.jl:134-153). */
int inferno_engine_finalize(InfernoEngine* eng);

/* One decoder layer in place on x[hidden] (host pointer), at position pos:
 * replaces DecoderLayerCPU(x, pos, rope, cache) (src/ModelCPU.jl:870-891). */
int inferno_layer_forward(InfernoEngine* eng, int layer, float* x_host, int pos);

/* Runs tokens tok[0..n) (0-based ids) at positions pos0.. and returns the
 * logits of the last one (vocab floats, may be NULL) and its first-max argmax
 * (may be NULL): replaces forward_cpu! + argmax (src/ModelCPU.jl:945-989,
 * 1123-1127). */
int inferno_forward_tokens(InfernoEngine* eng, const int32_t* tok, int n, int pos0, float* logits_out,
                           int32_t* argmax_out);

/* Logits (vocab floats per position, may be NULL) and first-max argmax of
 * EVERY position of tok[0..n) at positions pos0..: the full_logits forward
 * that mtp_verify_step! runs over draft tokens (src/ModelCPU.jl:1914-1930;
 * the caller compares argmax_out[i] with tok[i+1]).  Like the reference, the
 * recurrent state and KV cache advance over all n tokens. */
int inferno_forward_tokens_all(InfernoEngine* eng, const int32_t* tok, int n, int pos0, float* logits_out,
                               int32_t* argmax_out);

/* Greedy decode on the device: feeds `tok` at `pos`, then each argmax at the
 * next position, n_steps times; out_tokens[i] = token produced at step i.
 * The generation loop of test/benchmark_e2e.jl:43-59 / Engine.generate
 * (src/Engine.jl:327-344) with temperature 0. */
int inferno_decode_greedy(InfernoEngine* eng, int32_t tok, int pos, int n_steps, int32_t* out_tokens);

/* Sampled decode on the device: like inferno_decode_greedy, but each token is
 * drawn by the sampler of generate_cpu (src/ModelCPU.jl:1236-1254) with the
 * penalties applied to seen_tokens (host, may be NULL) and every generated
 * token; the draws come from Philox(s->seed, step). */
int inferno_decode_sample(InfernoEngine* eng, int32_t tok, int pos, int n_steps, const InfernoSampling* s,
                          const int32_t* seen_tokens, int n_seen, int32_t* out_tokens);

/* Batched decode (InfernoConfig.max_batch = B_max > 1; dense models on one
 * GPU): the engine keeps B_max slices of recurrent state and KV cache, one
 * per sequence.  inferno_select_sequence(eng, b) points every single-sequence
 * call (forward_tokens, decode_greedy, layer_forward, ...) at slice b -- e.g.
 * to prefill each sequence's own prompt.  inferno_decode_batch then decodes
 * sequences 0..B-1 in lockstep, greedily: sequence b feeds toks[b] at pos[b],
 * then each step's first-max argmax at the next position; out_tokens[t*B + b]
 * is sequence b's token of step t.  Every GEMV runs once per step over the B
 * sequences (one weight read per step; B >= 16 on the tensor-core GEMM),
 * the GDN and attention kernels index each sequence's own slice.  The token
 * loop of the reference (src/ModelCPU.jl:945-989, MoE over tokens at
 * src/Model.jl:478-561) run for B independent sequences; no reference
 * counterpart for the batching itself. */
int inferno_select_sequence(InfernoEngine* eng, int seq);
int inferno_decode_batch(InfernoEngine* eng, const int32_t* toks, const int32_t* pos, int B, int n_steps,
                         int32_t* out_tokens);

/* Zero GDN conv + recurrent state and the KV cache (src/ModelCPU.jl:525-529). */
int inferno_reset_states(InfernoEngine* eng);

/* Hidden state after `layer` for the last token run (debug / parity). */
int inferno_dump_hidden(InfernoEngine* eng, int layer, float* out_host);

/* Serialise / restore the recurrent state + KV cache (host buffer). */
int64_t inferno_state_size(InfernoEngine* eng);
int inferno_state_export(InfernoEngine* eng, void* host_buf, int64_t nbytes);
int inferno_state_import(InfernoEngine* eng, const void* host_buf, int64_t nbytes);

/* Checkpoint / resume on the device: copy the recurrent state + KV cache to
 * an engine-owned device snapshot, and back (stream-ordered, no host copy). */
int inferno_state_save_device(InfernoEngine* eng);
int inferno_state_restore_device(InfernoEngine* eng);

/* Kernels launched per decode token by this engine (for launch accounting). */
int inferno_kernels_per_token(InfernoEngine* eng);

/* How a sharded engine (tp_size > 1) sums residuals across ranks: 0 = not
 * sharded, 1 = the fused peer-memory exchange in the GEMV epilogue/prologue,
 * 2 = NCCL all-reduce.  No counterpart in the reference (which runs on one
 * device); reporting only. */
int inferno_comm_mode(InfernoEngine* eng);

/* Profiling pass: runs n_tokens greedy steps eagerly (no graph, no PDL) with
 * CUDA events between kernels and accumulates device time per kernel class:
 * [0] embedding, [1] layer GEMVs, [2] GDN step, [3] attention, [4] lm_head
 * GEMV + argmax, [5] finalize.  Arrays hold 6 entries. */
int inferno_profile_tokens(InfernoEngine* eng, int32_t tok, int pos, int n_tokens, float* ms_by_class,
                           int32_t* launches_by_class);

/* Debug: with INFERNO_B200_TRACE set at engine creation and a library built
 * with -DINFERNO_KTRACE=1, every GEMV, GDN and attention launch of a token
 * folds the %globaltimer stamps of all its CTAs into 8 u64 slots (launch
 * order): [0] kind (1 CUDA-core GEMV, 2 tensor-core GEMV, 3 GDN step,
 * 4 attention), [1] ~first CTA entry, [2] ~first CTA past
 * griddepcontrol.wait, [3] last CTA past the wait, [4] last prologue done,
 * [5] last first weight tile, [6] last CTA exit ("~": stored complemented).
 * out == NULL clears the stamps (call before the token to record); else
 * copies n u64 out. */
int inferno_debug_trace(InfernoEngine* eng, unsigned long long* out, int n);

/* Device time of the last inferno_decode_greedy call in ms (CUDA events). */
float inferno_last_decode_ms(InfernoEngine* eng);

/* Tensor parallel: a fresh 128-byte NCCL unique id for InfernoConfig.
 * nccl_unique_id (made by rank 0 and shared by the host, e.g. through
 * torch.distributed).  Each rank then creates its engine with its rank and
 * uploads its shard of the GGUF tensors (inferno_b200/tp.py); the engine
 * all-reduces the residual stream after ssm_out / attn_output / ffn_down and
 * the lm_head argmax over NCCL (NVLink).  No reference counterpart: the
 * reference has no multi-GPU path for this model family. */
#define INFERNO_TP_UNIQUE_ID_BYTES 128
int inferno_tp_unique_id(void* out, int nbytes);

/* Failure-path check of the tensor-parallel residual exchange on one GPU
 * (debug / tests): runs the tensor-core GEMV as an exchange reader against
 * partial buffers that nothing writes, with a poll limit of spin_limit
 * (1 .. 2^22) per word.  Expected result: INFERNO_EDEVICE with
 * *device_error_out = 1 (bounded wait timed out), the kernel having returned
 * and the context still usable.  The engine's own limit is set with
 * INFERNO_XCH_SPIN at engine creation (default 2^22 polls).  No reference
 * counterpart. */
int inferno_debug_xch_timeout(int spin_limit, int* device_error_out);

int inferno_engine_destroy(InfernoEngine* eng);

/* ============================ GGUF files =================================
 * Replaces GGUF.read_gguf (src/GGUF.jl:119-165) and the keep_quantized tensor
 * view of LoaderCPU.extract_tensor_cpu (src/LoaderCPU.jl:131-155).  The file
 * is memory-mapped read-only and parsed in place (version 2 or 3, strings up
 * to 1 MiB as in the reference, data aligned to general.alignment, default
 * 32); every read is bounds-checked and a malformed file returns
 * INFERNO_EFORMAT.  Returned names / strings / data pointers stay valid until
 * inferno_gguf_close. */
typedef struct InfernoGguf InfernoGguf;
int inferno_gguf_open(const char* path, InfernoGguf** out);
int inferno_gguf_close(InfernoGguf* g);
int inferno_gguf_version(const InfernoGguf* g);
int64_t inferno_gguf_n_tensors(const InfernoGguf* g);
int64_t inferno_gguf_n_kv(const InfernoGguf* g);
int64_t inferno_gguf_data_offset(const InfernoGguf* g);
/* key i in file order (NULL when out of range) */
const char* inferno_gguf_key(const InfernoGguf* g, int64_t i);
/* tensor i in file order: name, ggml type, ne[4] (missing dims = 1), data
 * bytes (0 when the type's block size is unknown) and a pointer to the bytes
 * in the mapping; any output may be NULL */
int inferno_gguf_tensor_info(const InfernoGguf* g, int64_t i, const char** name, int* ggml_type, int64_t ne[4],
                             uint64_t* nbytes, const void** data);
/* metadata by key: integer (any integer or bool type; uint64 bit for bit),
 * number (float32/64 or an integer), string, array (element type, length,
 * pointer to the first element; NULL for string arrays).  A missing key
 * returns INFERNO_ENOTFOUND, a value of another kind INFERNO_EINVAL. */
int inferno_gguf_get_int(const InfernoGguf* g, const char* key, int64_t* out);
int inferno_gguf_get_float(const InfernoGguf* g, const char* key, double* out);
int inferno_gguf_get_string(const InfernoGguf* g, const char* key, const char** out);
int inferno_gguf_get_array(const InfernoGguf* g, const char* key, int* elem_type, int64_t* len, const void** data);
/* Uploads every tensor of the file to the engine by its GGUF name, from the
 * mapping through pinned double-buffered staging (the engine-tier
 * equivalent of calling inferno_engine_upload_tensor per tensor).  Every
 * tensor must have a type the engine takes (F32, Q8_0, Q4_K, Q5_K, Q6_K,
 * IQ2_XXS); call before inferno_engine_finalize. */
int inferno_engine_load_gguf(InfernoEngine* eng, const InfernoGguf* g);

#ifdef __cplusplus
}
#endif
#endif /* INFERNO_B200_H */
