// The decode engine: owns the model on one GPU and runs Inferno.jl's
// per-token loop (src/ModelCPU.jl:945-989 forward_cpu!, :870-891 decoder
// layer, :1014-1046 lm_head, :1123-1127 greedy argmax) as a chain of fused
// sm_100a kernels, captured once into CUDA graphs with programmatic dependent
// launch between kernels.
//
// Per token (batch 1):
//   embed row (Q6_K dequant of token_embd row `tok`)
//   per GDN layer:  [in_proj|attn_gate] GEMV (RMSNorm prologue)
//                   GDN step (conv, norms, gates, delta rule)
//                   ssm_out GEMV (head-norm x SiLU(z) prologue, residual add)
//                   ffn gate/up GEMV (RMSNorm prologue, SwiGLU epilogue)
//                   ffn_down GEMV (residual add)
//   per attn layer: [wq|wk|wv] GEMV (RMSNorm prologue)
//                   split-K attention (norms, RoPE, KV append, gate)
//                   wo GEMV (residual add), FFN as above
//   lm_head GEMV (final RMSNorm prologue, first-max argmax epilogue)
//   finalize (next token, position, output slot)
// All control state (token, position, step) lives in device memory so the
// same graph replays for prompt tokens and for greedy decode.
#include <algorithm>
#include <cmath>
#include <cstring>
#include <map>
#include <memory>
#include <string>
#include <vector>
#include <nccl.h>
#include "internal.h"
#include "gemv.cuh"
#include "params.h"
#include "persist.h"
#include "gguf_internal.h"
#include "../../include/inferno_b200.h"

namespace inf {

struct Ctl {                 // device-resident step control
  int tok;                   // token embedded by the next step
  int pos;                   // its position
  int step;                  // steps run in the current call
  int n_prompt;              // prompt tokens of the current call
  int last;                  // argmax of the last step
  int pad[3];
  unsigned long long argkey; // packed first-max of the running lm_head
};

__global__ void finalize_kernel(Ctl* c, const int* prompt, int* out, int max_out, unsigned long long* xch_seq,
                                int xch_nsync, int* steps, int nsteps) {
  pdl_wait();
  pdl_trigger();
  // the Gated DeltaNet layers' step counters (their kernels ran with
  // self_advance = 0 in this token)
  for (int i = threadIdx.x; i < nsteps; i += blockDim.x) steps[i] += 1;
  if (threadIdx.x) return;
  if (xch_seq) *xch_seq += (unsigned long long)xch_nsync;   // sequence base of the next token's sync points
  const unsigned long long key = c->argkey;
  const int am = (int)(0xffffffffu - (uint32_t)(key & 0xffffffffull));
  c->last = am;
  const int s = c->step;
  c->tok = (s + 1 < c->n_prompt) ? prompt[s + 1] : am;
  const int o = s - (c->n_prompt - 1);
  if (o >= 0 && o < max_out) out[o] = am;
  c->pos = c->pos + 1;
  c->step = s + 1;
  c->argkey = 0ull;
}

struct DevTensor {
  int type = -1;
  int64_t ne[4] = {1, 1, 1, 1};
  void* d = nullptr;
  size_t bytes = 0;
  float* wb = nullptr;   // bound of |w| shared by this tensor's tensor-core GEMM group (prefill)
  int64_t rows() const { return ne[1] * ne[2] * ne[3]; }
};

struct LayerBind {
  bool ssm = false;
  DevTensor *attn_norm = nullptr, *post_norm = nullptr;
  DevTensor *in_proj = nullptr, *gate = nullptr, *ssm_out = nullptr, *conv1d = nullptr, *alpha = nullptr,
            *beta = nullptr, *ssm_a = nullptr, *dt_bias = nullptr, *ssm_norm = nullptr;
  DevTensor *wq = nullptr, *wk = nullptr, *wv = nullptr, *wo = nullptr, *q_norm = nullptr, *k_norm = nullptr;
  DevTensor *ffn_gate = nullptr, *ffn_up = nullptr, *ffn_down = nullptr;
  DevTensor ffn_down_raw;      // GGUF-layout copy when ffn_down is regrouped (batched prefill GEMVs)
  void* wperm = nullptr;       // fused in_proj + GDN: head-regrouped [q|k|v|z] rows (Q4_K)
  // MoE FFN (config 5): router, routed experts, optional shared expert
  DevTensor *router = nullptr, *exp_gate = nullptr, *exp_up = nullptr, *exp_down = nullptr;
  DevTensor *sh_gate = nullptr, *sh_up = nullptr, *sh_down = nullptr;
  float* ring = nullptr;
  float* S = nullptr;
  int* step = nullptr;
  int* done = nullptr;
  float* kc = nullptr;
  float* vc = nullptr;
  // sequence 0's slices (batched decode keeps one slice per sequence)
  float *ring0 = nullptr, *S0 = nullptr, *kc0 = nullptr, *vc0 = nullptr;
};

}  // namespace inf

struct InfernoEngine {
  InfernoConfig cfg{};
  int dev = 0;
  cudaStream_t st = nullptr;
  std::map<std::string, inf::DevTensor> tensors;
  std::vector<inf::LayerBind> layers;
  inf::DevTensor *embd = nullptr, *out_norm = nullptr, *lm_head = nullptr;
  // tensor parallel: rank `tp_rank` of `tp_size` owns a slice of every layer
  // (sharded by the host) and rows [tp_rank*V/tp, ...) of the lm_head
  ncclComm_t comm = nullptr;
  inf::DevTensor lm_view;
  inf::DevTensor lm_packed;         // tied lm_head regrouped for the tensor-core GEMV (T_Q6_KR)
  inf::DevTensor* lm_raw = nullptr;  // the lm_head in GGUF layout
  float* logits_local = nullptr;
  // fused tensor-parallel exchange over NVLink peer memory (xch); when off
  // (INFERNO_TP_NCCL=1 or a GEMV outside the tensor-core path) the residual
  // is summed with ncclAllReduce
  bool ep = false;                  // expert parallel: ranks split the MoE experts, the rest is replicated
  bool tp = false;                  // tensor parallel: ranks hold shards of every layer
  bool xch = false;
  float* x2 = nullptr;              // second residual buffer (alternates per sync point)
  float* xcur = nullptr;            // buffer holding the current residual while enqueueing
  int xch_k = 0, xch_pending = -1;  // next sync index / sync whose partials are pending
  unsigned long long* xch_peer[8] = {};   // every rank's [2][N][H] exchange words (own + IPC-mapped)
  unsigned* xch_done = nullptr;           // setup barrier word
  unsigned long long* xch_seq = nullptr;
  unsigned xch_spin = 0;            // reader polls per word before a timeout (INFERNO_XCH_SPIN; 0 = 2^22)
  bool finalized = false;
  int C = 0, di = 0, rd = 0, split_len = 64, nsplit = 1;
  // activations
  float *x = nullptr, *qkv = nullptr, *z = nullptr, *y = nullptr, *qg = nullptr, *k = nullptr, *v = nullptr,
        *o = nullptr, *h = nullptr, *logits = nullptr;
  float *rope_cos = nullptr, *rope_sin = nullptr, *part_o = nullptr, *part_ml = nullptr, *hidden = nullptr;
  int* att_counters = nullptr;
  // chunked prefill: activations of up to PF_MAX_T tokens ([t][...] rows)
  bool prefill = false;
  // prefill graphs by (tokens, first position, logits): built on the second
  // call with the same key (the first runs eagerly)
  std::map<long long, cudaGraphExec_t> pf_graphs;
  std::map<long long, int> pf_seen;
  float *xb = nullptr, *qkvb = nullptr, *zb = nullptr, *yb = nullptr, *qgb = nullptr, *kb = nullptr,
        *vb = nullptr, *ob = nullptr, *hb = nullptr;
  // tensor-core prefill: fp16 hi / lo activation rows [PF_MAX_T][max inner],
  // token exponents, the GDN prep rows and the weight bounds
  __half *pf_xhi = nullptr, *pf_xlo = nullptr;
  float* qg_ws = nullptr;          // split-K workspace of the tensor-core GEMM
  int* qg_tickets = nullptr;
  float* pf_xexp = nullptr;
  inf::GdnScratch pf_gdn{};
  float* pf_wbounds = nullptr;
  // MoE scratch: router logits, selected ids / weights, expert hidden, expert outputs
  float *moe_logits = nullptr, *moe_w = nullptr, *moe_h = nullptr, *moe_y = nullptr;
  int* moe_idx = nullptr;
  inf::Ctl* ctl = nullptr;
  int *prompt = nullptr, *out_tokens = nullptr;
  int max_out = 0;
  int* err = nullptr;
  // state arena (for reset / export)
  std::vector<std::pair<void*, size_t>> state_bufs;
  std::vector<void*> allocs;
  cudaGraphExec_t g1 = nullptr, g1_logits = nullptr, g8 = nullptr;
  cudaEvent_t ev0 = nullptr, ev1 = nullptr;
  float last_ms = 0.f;
  bool dump = false;
  unsigned ablate = 0;           // debug: kernel classes left out (INFERNO_B200_ABLATE)
  // persistent decode kernel (decode.cu)
  bool persistent = false;
  bool repack = false;           // Q6_K GEMV matrices regrouped (T_Q6_KR)
  inf::PkStage* pk_stages = nullptr;
  int pk_nstages = 0;
  size_t pk_smem = 0;
  int pk_slot = 0, pk_hidden_pad = 0, pk_inner_pad = 0;
  unsigned* pk_barrier = nullptr;
  int* pk_abort = nullptr;
  // sampled decode: parameters of the graph being captured (null = greedy) and
  // the tokens the penalties apply to
  const inf::SampleArgs* sampling = nullptr;
  uint8_t* seen = nullptr;
  unsigned long long* trace = nullptr;   // debug: per-launch timeline slots (INFERNO_B200_TRACE)
  // Gated DeltaNet step counters of every layer, contiguous; while a decode
  // token is enqueued (in_token) the GDN kernels leave them to the token's
  // finalize kernel (token_steps; off when a fused in_proj + GDN layer
  // advances its own)
  int* gdn_steps = nullptr;
  bool in_token = false, token_steps = false;
  // whole-head GDN kernel in batch-1 decode tokens (INFERNO_GDN_HEAD=1); off by
  // default: 16 CTAs of 512 threads measured slower than 128 row-block CTAs
  // plus the head-norm prologue of ssm_out (0.70 vs 0.66 ms/token, config 1).
  // Batched decode always uses it (one CTA per head and sequence).
  bool gdn_head = false;
  // batched decode: nseq = max_batch state slices; `cur_seq` is the slice the
  // single-sequence calls use; per batch size B one captured step graph
  int nseq = 1, cur_seq = 0;
  int *bt_tok = nullptr, *bt_pos = nullptr, *bt_out = nullptr, *bt_step = nullptr;
  unsigned long long* bt_keys = nullptr;
  int bt_out_cap = 0;
  std::map<int, cudaGraphExec_t> bt_graphs;
  int trace_idx = 0;
  int launches = 0;              // kernels enqueued since the last enqueue_token began
  int token_launches = 0;        // kernels of one decode token (set by enqueue_token)
  void* snapshot = nullptr;      // device copy of the state arena
  size_t state_bytes = 0;
  // profiling: events between the kernels of one eager token
  bool profiling = false;
  std::vector<cudaEvent_t> prof_ev;
  std::vector<int> prof_kind;     // kernel class per interval
};

namespace inf {

namespace {

int build_persistent(InfernoEngine* e);
int run_persistent(InfernoEngine* e, int tok0, int pos0, int n_prompt, int n_steps);

template <class T>
int dalloc(InfernoEngine* e, T** p, size_t count, bool state = false) {
  void* d = nullptr;
  size_t bytes = (count * sizeof(T) + 255) / 256 * 256;
  cudaError_t r = cudaMalloc(&d, bytes);
  if (r != cudaSuccess)
    return set_error(INFERNO_ENOMEM, "cudaMalloc(%zu) failed: %s", bytes, cudaGetErrorString(r));
  cudaMemset(d, 0, bytes);
  e->allocs.push_back(d);
  if (state) e->state_bufs.push_back({d, bytes});
  *p = (T*)d;
  return 0;
}

DevTensor* find(InfernoEngine* e, const std::string& n) {
  auto it = e->tensors.find(n);
  return it == e->tensors.end() ? nullptr : &it->second;
}

int require(InfernoEngine* e, const std::string& n, DevTensor** out, int type = -2) {
  DevTensor* t = find(e, n);
  if (!t) return set_error(INFERNO_EINVAL, "missing tensor %s", n.c_str());
  if (type != -2 && t->type != type) return set_error(INFERNO_EINVAL, "tensor %s: type %d, expected %d", n.c_str(), t->type, type);
  *out = t;
  return 0;
}

// kernel classes reported by the profiling pass
enum KClass { K_EMBED = 0, K_GEMV = 1, K_GDN = 2, K_ATTN = 3, K_LMHEAD = 4, K_FINAL = 5, K_NCLASS = 6 };

void mark(InfernoEngine* e, int kind) {
  ++e->launches;
  if (!e->profiling) return;
  cudaEvent_t ev;
  cudaEventCreate(&ev);
  cudaEventRecord(ev, e->st);
  e->prof_ev.push_back(ev);
  e->prof_kind.push_back(kind);
}

// debug timeline: 8 slots per launch of a token (INFERNO_B200_TRACE)
constexpr int TRACE_SLOTS = 8, TRACE_LAUNCHES = 1024;
unsigned long long* trace_slot(InfernoEngine* e) {
  if (!e->trace || e->trace_idx >= TRACE_LAUNCHES) return nullptr;
  return e->trace + TRACE_SLOTS * (e->trace_idx++);
}

constexpr int EPI_XCH_WRITE = 100;   // engine-level: residual partial to the TP exchange

int gemv(InfernoEngine* e, int type, int inner, std::initializer_list<GemvMat> mats, const float* x, int pro,
         const float* pro_w, const float* pro_z, int group, int epi, unsigned long long* argmax, bool pdl) {
  GemvCall c;
  c.type = type;
  c.inner = inner;
  for (auto& m : mats) c.mats[c.nmats++] = m;
  c.x = x;
  c.x_stride = inner;
  c.pro = pro;
  c.pro_w = pro_w;
  c.pro_z = pro_z;
  c.pro_group = group;
  c.eps = e->cfg.rms_eps;
  c.epi = epi;
  c.argmax = argmax;
  c.err = e->err;
  if (e->xch) {
    const int n = e->cfg.tp_size;
    c.xch_n = n;
    c.xch_rank = e->cfg.tp_rank;
    c.xch_seq = e->xch_seq;
    c.xch_spin = e->xch_spin;
    for (int q = 0; q < n; ++q) c.xch_parts[q] = e->xch_peer[q];
    if (epi == EPI_XCH_WRITE) {
      c.epi = EPI_STORE;
      c.xch_wk = e->xch_k;
      e->xch_pending = e->xch_k++;
    } else if (pro == PRO_RMSNORM && x == e->xcur && e->xch_pending >= 0) {
      c.xch_rk = e->xch_pending;
      c.x_next = e->xcur == e->x ? e->x2 : e->x;
    }
  }
  c.trace = trace_slot(e);
  int rc = launch_gemv(c, e->st, pdl);
  if (!rc) mark(e, epi == EPI_ARGMAX ? K_LMHEAD : K_GEMV);
  return rc;
}

GemvMat M(DevTensor* t, float* y) { return GemvMat{t->d, y, (int)t->rows()}; }

// Residual epilogue of a sublayer's last GEMV.  Tensor parallel: rank 0 adds
// its partial to x, the other ranks store theirs, and one all-reduce (sum) of
// x completes x + sum_r partial_r on every rank.
int residual_epi(InfernoEngine* e) {
  // expert parallel: the attention / GDN sublayers are replicated (local
  // residual add); only the expert FFN's partial sums are exchanged
  if (e->xch && e->tp) return EPI_XCH_WRITE;
  return (e->tp && e->cfg.tp_rank != 0) ? EPI_STORE : EPI_ADD;
}

// After the GEMVs that consumed a pending exchange: the completed residual now
// lives in the other buffer.
void xch_commit(InfernoEngine* e) {
  if (e->xch_pending < 0) return;
  e->xcur = e->xcur == e->x ? e->x2 : e->x;
  e->xch_pending = -1;
}

int tp_sum_x(InfernoEngine* e) {
  if (!e->tp || e->xch) return 0;
  ncclResult_t r = ncclAllReduce(e->x, e->x, (size_t)e->cfg.hidden_size, ncclFloat, ncclSum, e->comm, e->st);
  if (r != ncclSuccess) return set_error(INFERNO_ENCCL, "all-reduce of the residual: %s", ncclGetErrorString(r));
  return 0;
}

// MoE FFN of one layer (src/Model.jl:478-561 routing, SwiGLU experts):
// router GEMV -> softmax/top-k -> routed gate/up (experts gathered through the
// device ids) -> shared gate/up -> one down GEMV over every selected expert,
// each with its own input slice -> weighted combine into x.
int enqueue_moe(InfernoEngine* e, LayerBind& L, bool pdl) {
  const InfernoConfig& c = e->cfg;
  const int H = c.hidden_size, E = c.n_experts, K = c.n_experts_used, Ie = c.expert_ffn;
  // expert parallel: this rank holds experts [ebase, ebase + El)
  const int El = e->ep ? E / c.tp_size : E, ebase = e->ep ? c.tp_rank * El : 0;
  const bool lead = !e->ep || c.tp_rank == 0;
  const bool shared = L.sh_gate != nullptr;
  const float* pn = (const float*)L.post_norm->d;
  int rc;
  if ((rc = gemv(e, L.router->type, H, {M(L.router, e->moe_logits)}, e->xcur, PRO_RMSNORM, pn, nullptr, 0, EPI_STORE,
                 nullptr, pdl)))
    return rc;
  if ((rc = launch_moe_topk(e->moe_logits, E, K, e->moe_idx, e->moe_w, e->err, ebase, El, e->st, pdl))) return rc;
  mark(e, K_GEMV);
  {
    GemvCall g;
    g.type = L.exp_gate->type;
    g.inner = H;
    g.mats[0] = GemvMat{L.exp_gate->d, e->moe_h, K * Ie, 1, 0};
    g.mats[1] = GemvMat{L.exp_up->d, nullptr, K * Ie, 1, 0};
    g.nmats = 2;
    g.x = e->xcur;
    g.x_stride = H;
    g.pro = PRO_RMSNORM;
    g.pro_w = pn;
    g.eps = c.rms_eps;
    g.epi = EPI_SWIGLU;
    g.err = e->err;
    g.eidx = e->moe_idx;
    g.estride = (long long)(L.exp_gate->bytes / El);
    g.erows = Ie;
    g.n_experts = El;
    if ((rc = launch_gemv(g, e->st, pdl))) return rc;
    mark(e, K_GEMV);
  }
  if (shared && (rc = gemv(e, L.sh_gate->type, H, {M(L.sh_gate, e->moe_h + (size_t)K * Ie), M(L.sh_up, nullptr)}, e->xcur,
                           PRO_RMSNORM, pn, nullptr, 0, EPI_SWIGLU, nullptr, pdl)))
    return rc;
  {
    GemvCall g;
    g.type = L.exp_down->type;
    g.inner = Ie;
    g.mats[0] = GemvMat{L.exp_down->d, e->moe_y, K * H, 1, 0};
    g.nmats = 1;
    if (shared) g.mats[g.nmats++] = GemvMat{L.sh_down->d, e->moe_y + (size_t)K * H, H, 0, K};
    g.x = e->moe_h;
    g.x_stride = Ie;
    g.nxv = K + (shared ? 1 : 0);
    g.pro = PRO_NONE;
    g.eps = c.rms_eps;
    g.epi = EPI_STORE;
    g.err = e->err;
    g.eidx = e->moe_idx;
    g.estride = (long long)(L.exp_down->bytes / El);
    g.erows = H;
    g.n_experts = El;
    if ((rc = launch_gemv(g, e->st, pdl))) return rc;
    mark(e, K_GEMV);
  }
  if (e->ep && e->xch) {
    // partial sums to every rank's exchange buffer; the next RMSNorm GEMV adds them
    MoeXch xc{};
    for (int q = 0; q < c.tp_size; ++q) xc.parts[q] = e->xch_peer[q];
    xc.seq = e->xch_seq;
    xc.n = c.tp_size;
    xc.rank = c.tp_rank;
    xc.k = e->xch_k;
    if ((rc = launch_moe_combine_xch(e->moe_y, e->moe_w, e->moe_idx, K, H, (shared && lead) ? 1 : 0, xc, e->st,
                                     pdl)))
      return rc;
    mark(e, K_GEMV);
    e->xch_pending = e->xch_k++;
    return 0;
  }
  if ((rc = launch_moe_combine(e->xcur, e->moe_y, e->moe_w, e->moe_idx, K, H, (shared && lead) ? 1 : 0, lead ? 1 : 0,
                                e->st, pdl)))
    return rc;
  mark(e, K_GEMV);
  if (e->ep) {
    // x = x + sum over ranks of their experts' partials
    ncclResult_t r = ncclAllReduce(e->x, e->x, (size_t)H, ncclFloat, ncclSum, e->comm, e->st);
    if (r != ncclSuccess) return set_error(INFERNO_ENCCL, "expert-parallel all-reduce: %s", ncclGetErrorString(r));
  }
  return 0;
}

int enqueue_layer(InfernoEngine* e, int li, bool pdl) {
  LayerBind& L = e->layers[li];
  const InfernoConfig& c = e->cfg;
  const int H = c.hidden_size;
  int rc;
  const unsigned ab = e->ablate;   // timing experiments only: results are wrong when set
  if (L.ssm && L.wperm) {
    // [in_proj | attn_gate] GEMV and the GDN step as one cluster kernel
    GdnParams g{};
    g.in_norm = (const float*)L.attn_norm->d;
    g.eps = c.rms_eps;
    g.H = H;
    g.nv = c.ssm_nv;
    g.nk = c.ssm_nk;
    g.dv = c.ssm_dv;
    g.K = c.ssm_conv_kernel;
    g.C = e->C;
    g.conv_w = (const float*)L.conv1d->d;
    g.ring = L.ring;
    g.w_alpha = (const float*)L.alpha->d;
    g.w_beta = (const float*)L.beta->d;
    g.ssm_a = (const float*)L.ssm_a->d;
    g.dt_bias = (const float*)L.dt_bias->d;
    g.S = L.S;
    g.y = e->y;
    g.step = L.step;
    g.done = L.done;
    if ((rc = launch_fused_inproj_gdn(L.wperm, H, e->xcur, (const float*)L.attn_norm->d, c.rms_eps, g, e->z, e->err,
                                      e->st, pdl)))
      return rc;
    mark(e, K_GDN);
    xch_commit(e);
    if (!(ab & 8) && (rc = gemv(e, L.ssm_out->type, e->di, {M(L.ssm_out, e->xcur)}, e->y, (ab & 128) ? PRO_NONE : PRO_HEADNORM_GATE,
                   (const float*)L.ssm_norm->d, e->z, c.ssm_dv, residual_epi(e), nullptr, pdl)))
      return rc;
    if ((rc = tp_sum_x(e))) return rc;
  } else if (L.ssm) {
    // [in_proj | attn_gate] on RMSNorm(x)
    if (ab & 1) {
    } else if (L.in_proj->type == L.gate->type) {
      if ((rc = gemv(e, L.in_proj->type, H, {M(L.in_proj, e->qkv), M(L.gate, e->z)}, e->xcur, PRO_RMSNORM,
                     (const float*)L.attn_norm->d, nullptr, 0, EPI_STORE, nullptr, pdl)))
        return rc;
    } else {
      if ((rc = gemv(e, L.in_proj->type, H, {M(L.in_proj, e->qkv)}, e->xcur, PRO_RMSNORM, (const float*)L.attn_norm->d,
                     nullptr, 0, EPI_STORE, nullptr, pdl)))
        return rc;
      if ((rc = gemv(e, L.gate->type, H, {M(L.gate, e->z)}, e->xcur, PRO_RMSNORM, (const float*)L.attn_norm->d,
                     nullptr, 0, EPI_STORE, nullptr, pdl)))
        return rc;
    }
    xch_commit(e);
    GdnParams g{};
    g.x = e->xcur;
    g.in_norm = (const float*)L.attn_norm->d;
    g.eps = c.rms_eps;
    g.H = H;
    g.nv = c.ssm_nv;
    g.nk = c.ssm_nk;
    g.dv = c.ssm_dv;
    g.K = c.ssm_conv_kernel;
    g.C = e->C;
    g.qkv = e->qkv;
    g.conv_w = (const float*)L.conv1d->d;
    g.ring = L.ring;
    g.w_alpha = (const float*)L.alpha->d;
    g.w_beta = (const float*)L.beta->d;
    g.ssm_a = (const float*)L.ssm_a->d;
    g.dt_bias = (const float*)L.dt_bias->d;
    g.S = L.S;
    g.y = e->y;
    g.step = L.step;
    g.done = L.done;
    g.trace = trace_slot(e);
    g.self_advance = (e->in_token && e->token_steps) ? 0 : 1;
    // whole-head step (output norm + gate fused, ssm_out reads a plain input)
    // inside decode tokens, where the finalize kernel advances the counters
    const bool head = e->gdn_head && !g.self_advance;
    if (head) {
      g.z = e->z;
      g.out_norm = (const float*)L.ssm_norm->d;
    }
    if (!(ab & 2) && (rc = head ? launch_gdn_head(g, e->st, pdl) : launch_gdn_step(g, e->st, pdl))) return rc;
    mark(e, K_GDN);
    const int sp = (head || (ab & 128)) ? PRO_NONE : PRO_HEADNORM_GATE;
    if (!(ab & 8) && (rc = gemv(e, L.ssm_out->type, e->di, {M(L.ssm_out, e->xcur)}, e->y, sp,
                   (const float*)L.ssm_norm->d, e->z, c.ssm_dv, residual_epi(e), nullptr, pdl)))
      return rc;
    if ((rc = tp_sum_x(e))) return rc;
  } else {
    const int qrows = (int)L.wq->rows();
    (void)qrows;
    if (ab & 1) {
    } else if (L.wq->type == L.wk->type && L.wk->type == L.wv->type) {
      if ((rc = gemv(e, L.wq->type, H, {M(L.wq, e->qg), M(L.wk, e->k), M(L.wv, e->v)}, e->xcur, PRO_RMSNORM,
                     (const float*)L.attn_norm->d, nullptr, 0, EPI_STORE, nullptr, pdl)))
        return rc;
    } else {
      if ((rc = gemv(e, L.wq->type, H, {M(L.wq, e->qg), M(L.wk, e->k)}, e->xcur, PRO_RMSNORM,
                     (const float*)L.attn_norm->d, nullptr, 0, EPI_STORE, nullptr, pdl)))
        return rc;
      if ((rc = gemv(e, L.wv->type, H, {M(L.wv, e->v)}, e->xcur, PRO_RMSNORM, (const float*)L.attn_norm->d, nullptr,
                     0, EPI_STORE, nullptr, pdl)))
        return rc;
    }
    xch_commit(e);
    AttnParams a{};
    a.qg = e->qg;
    a.k = e->k;
    a.v = e->v;
    a.q_norm = (const float*)L.q_norm->d;
    a.k_norm = (const float*)L.k_norm->d;
    a.eps = c.rms_eps;
    a.rope_cos = e->rope_cos;
    a.rope_sin = e->rope_sin;
    a.rd = e->rd;
    a.kc = L.kc;
    a.vc = L.vc;
    a.nh = c.n_heads;
    a.nkv = c.n_kv_heads;
    a.ctx = c.max_ctx;
    a.split_len = e->split_len;
    a.nsplit = e->nsplit;
    a.pos = &e->ctl->pos;
    a.part_o = e->part_o;
    a.part_ml = e->part_ml;
    a.counters = e->att_counters;
    a.out = e->o;
    a.err = e->err;
    a.trace = trace_slot(e);
    if (!(ab & 4) && (rc = launch_attn_decode(a, e->st, pdl))) return rc;
    mark(e, K_ATTN);
    if (!(ab & 8) && (rc = gemv(e, L.wo->type, c.n_heads * c.head_dim, {M(L.wo, e->xcur)}, e->o, PRO_NONE, nullptr, nullptr, 0,
                   residual_epi(e), nullptr, pdl)))
      return rc;
    if ((rc = tp_sum_x(e))) return rc;
  }
  if (c.n_experts) {
    if ((rc = enqueue_moe(e, L, pdl))) return rc;
    if (e->dump)
      INF_CUDA_TRY(cudaMemcpyAsync(e->hidden + (size_t)li * H, e->xcur, (size_t)H * 4, cudaMemcpyDeviceToDevice, e->st));
    return 0;
  }
  // FFN: SwiGLU(gate, up) on RMSNorm(x), then down with residual add
  if (L.ffn_gate->type == L.ffn_up->type) {
    if (!(ab & 16) && (rc = gemv(e, L.ffn_gate->type, H, {M(L.ffn_gate, e->h), M(L.ffn_up, nullptr)}, e->xcur, PRO_RMSNORM,
                   (const float*)L.post_norm->d, nullptr, 0, EPI_SWIGLU, nullptr, pdl)))
      return rc;
    xch_commit(e);
  } else {
    return set_error(INFERNO_EINVAL, "layer %d: ffn_gate and ffn_up must share a type", li);
  }
  if (!(ab & 32) && (rc = gemv(e, L.ffn_down->type, c.intermediate_size, {M(L.ffn_down, e->xcur)}, e->h, PRO_NONE, nullptr, nullptr,
                 0, residual_epi(e), nullptr, pdl)))
    return rc;
  if ((rc = tp_sum_x(e))) return rc;
  if (e->dump)
    INF_CUDA_TRY(cudaMemcpyAsync(e->hidden + (size_t)li * H, e->xcur, (size_t)H * 4, cudaMemcpyDeviceToDevice, e->st));
  return 0;
}

// batched GEMV over T token columns (x rows x_stride apart, y rows y_stride apart)
// (reuse_act: the previous bgemv converted the same input with the same
// prologue; its fp16 activation rows are used again)
int bgemv(InfernoEngine* e, const DevTensor* W, int inner, std::initializer_list<GemvMat> mats, const float* x,
          int T, long long x_stride, long long y_stride, int pro, const float* pro_w, const float* pro_z, int group,
          int epi, bool reuse_act = false) {
  GemvCall c;
  c.type = W->type;
  c.inner = inner;
  for (auto& m : mats) c.mats[c.nmats++] = m;
  c.nb = T;
  c.x = x;
  c.x_stride = x_stride;
  c.y_stride = y_stride;
  c.pro = pro;
  c.pro_w = pro_w;
  c.pro_z = pro_z;
  c.pro_group = group;
  c.eps = e->cfg.rms_eps;
  c.epi = epi;
  c.err = e->err;
  // the tcgen05 GEMM from 4 token columns on (measured: batched decode of 8
  // sequences 2561 -> 2700 tokens/s at config 1, 399 -> 458 at config 4
  // against the integer mma.sync batch GEMV)
  static const int tc_min = getenv("INFERNO_TC_MIN_T") ? std::max(1, atoi(getenv("INFERNO_TC_MIN_T"))) : GEMM_TC_MIN_T;
  if (T >= tc_min && e->pf_xhi && W->wb && qgemm_supported(W->type) && epi != EPI_ARGMAX && inner % 256 == 0) {
    // fp16 hi / lo activations with the prologue applied, then the tcgen05 GEMM
    int rc = 0;
    if (!reuse_act) {
      // programmatic dependent launch: the conversion waits for its inputs,
      // the GEMM stages its (constant) weights while the conversion runs
      rc = launch_qgemm_act(x, x_stride, inner, T, pro, pro_w, pro_z, group, e->cfg.rms_eps, e->pf_xhi, e->pf_xlo,
                            e->pf_xexp, e->st, true);
      if (rc) return rc;
      mark(e, K_GEMV);
    }
    QgemmCall q;
    q.type = W->type;
    q.K = inner;
    for (auto& m : mats) q.mats[q.nmats++] = m;
    q.T = T;
    q.xhi = e->pf_xhi;
    q.xlo = e->pf_xlo;
    q.xexp = e->pf_xexp;
    q.y_stride = y_stride;
    q.epi = epi == EPI_ADD ? 1 : epi == EPI_SWIGLU ? 2 : 0;
    q.wbound = W->wb;
    q.err = e->err;
    q.ws = e->qg_ws;
    q.tickets = e->qg_tickets;
    rc = launch_qgemm(q, e->st, true);
    if (!rc) mark(e, K_GEMV);
    return rc;
  }
  const int rc = launch_gemv(c, e->st, false);
  if (!rc) mark(e, K_GEMV);
  return rc;
}

// One prefill chunk: T <= PF_MAX_T prompt tokens (device ids) at positions
// pos0.. through every layer with batched GEMVs and the chunk kernels of
// prefill.cu; the last chunk also runs the lm_head on its last token.
// Tensor-parallel prefill: the row-parallel products (ssm_out, attn_output,
// ffn_down) leave each rank a partial of the residual update; rank 0 adds its
// partial to the residual rows, the others store theirs over them, and one
// NCCL all-reduce of the [T][H] rows makes every rank's residual
// x + sum_r partial_r.
int pf_residual_epi(InfernoEngine* e) { return (!e->tp || e->cfg.tp_rank == 0) ? EPI_ADD : EPI_STORE; }
int pf_tp_sum(InfernoEngine* e, int T) {
  if (!e->tp) return 0;
  ncclResult_t r = ncclAllReduce(e->xb, e->xb, (size_t)T * e->cfg.hidden_size, ncclFloat, ncclSum, e->comm, e->st);
  return r == ncclSuccess ? 0 : set_error(INFERNO_ENCCL, "prefill residual all-reduce: %s", ncclGetErrorString(r));
}

int enqueue_prefill_chunk(InfernoEngine* e, const int* toks, int T, int pos0, bool last, bool logits) {
  const InfernoConfig& c = e->cfg;
  const int H = c.hidden_size, I = c.intermediate_size, hdq = c.n_heads * c.head_dim;
  int rc;
  if ((rc = launch_embed_row(e->embd->type, e->embd->d, (long long)e->embd->bytes / e->embd->rows(), H, toks, e->xb,
                             c.vocab_size, e->st, false, T)))
    return set_error(INFERNO_ECUDA, "prefill embedding launch failed (%d)", rc);
  for (int li = 0; li < c.num_layers; ++li) {
    LayerBind& L = e->layers[li];
    const float* an = (const float*)L.attn_norm->d;
    if (L.ssm) {
      if ((rc = bgemv(e, L.in_proj, H, {M(L.in_proj, e->qkvb)}, e->xb, T, H, e->C, PRO_RMSNORM, an, nullptr, 0,
                      EPI_STORE)) ||
          (rc = bgemv(e, L.gate, H, {M(L.gate, e->zb)}, e->xb, T, H, e->di, PRO_RMSNORM, an, nullptr, 0, EPI_STORE,
                      L.in_proj->wb && L.gate->wb)))
        return rc;
      GdnParams g{};
      g.x = e->xb;
      g.in_norm = an;
      g.eps = c.rms_eps;
      g.H = H;
      g.nv = c.ssm_nv;
      g.nk = c.ssm_nk;
      g.dv = c.ssm_dv;
      g.K = c.ssm_conv_kernel;
      g.C = e->C;
      g.qkv = e->qkvb;
      g.conv_w = (const float*)L.conv1d->d;
      g.ring = L.ring;
      g.w_alpha = (const float*)L.alpha->d;
      g.w_beta = (const float*)L.beta->d;
      g.ssm_a = (const float*)L.ssm_a->d;
      g.dt_bias = (const float*)L.dt_bias->d;
      g.S = L.S;
      g.y = e->yb;
      g.step = L.step;
      g.done = L.done;
      if (T >= PF_TC_MIN_T && e->pf_gdn.qn) {
        if ((rc = launch_gdn_prefill(g, T, e->pf_gdn, e->st))) return rc;
      } else if ((rc = launch_gdn_chunk(g, T, e->st))) {
        return rc;
      }
      mark(e, K_GDN);
      if ((rc = bgemv(e, L.ssm_out, e->di, {M(L.ssm_out, e->xb)}, e->yb, T, e->di, H, PRO_HEADNORM_GATE,
                      (const float*)L.ssm_norm->d, e->zb, c.ssm_dv, pf_residual_epi(e))) ||
          (rc = pf_tp_sum(e, T)))
        return rc;
    } else {
      const int kvd = c.n_kv_heads * c.head_dim;
      if ((rc = bgemv(e, L.wq, H, {M(L.wq, e->qgb)}, e->xb, T, H, 2 * hdq, PRO_RMSNORM, an, nullptr, 0, EPI_STORE)))
        return rc;
      if (L.wk->type == L.wv->type) {
        if ((rc = bgemv(e, L.wk, H, {M(L.wk, e->kb), M(L.wv, e->vb)}, e->xb, T, H, kvd, PRO_RMSNORM, an, nullptr, 0,
                        EPI_STORE, L.wq->wb && L.wk->wb)))
          return rc;
      } else if ((rc = bgemv(e, L.wk, H, {M(L.wk, e->kb)}, e->xb, T, H, kvd, PRO_RMSNORM, an, nullptr, 0, EPI_STORE)) ||
                 (rc = bgemv(e, L.wv, H, {M(L.wv, e->vb)}, e->xb, T, H, kvd, PRO_RMSNORM, an, nullptr, 0, EPI_STORE))) {
        return rc;
      }
      AttnParams a{};
      a.qg = e->qgb;
      a.k = e->kb;
      a.v = e->vb;
      a.q_norm = (const float*)L.q_norm->d;
      a.k_norm = (const float*)L.k_norm->d;
      a.eps = c.rms_eps;
      a.rope_cos = e->rope_cos;
      a.rope_sin = e->rope_sin;
      a.rd = e->rd;
      a.kc = L.kc;
      a.vc = L.vc;
      a.nh = c.n_heads;
      a.nkv = c.n_kv_heads;
      a.ctx = c.max_ctx;
      a.split_len = e->split_len;
      a.nsplit = e->nsplit;
      a.part_o = e->part_o;
      a.part_ml = e->part_ml;
      a.counters = e->att_counters;
      a.out = e->ob;
      a.err = e->err;
      if ((rc = launch_attn_chunk(a, pos0, T, e->st))) return rc;
      mark(e, K_ATTN);
      if ((rc = bgemv(e, L.wo, hdq, {M(L.wo, e->xb)}, e->ob, T, hdq, H, PRO_NONE, nullptr, nullptr, 0,
                      pf_residual_epi(e))) ||
          (rc = pf_tp_sum(e, T)))
        return rc;
    }
    DevTensor* down = L.ffn_down->type == T_Q6_KR ? &L.ffn_down_raw : L.ffn_down;
    if ((rc = bgemv(e, L.ffn_gate, H, {M(L.ffn_gate, e->hb), M(L.ffn_up, nullptr)}, e->xb, T, H, I, PRO_RMSNORM,
                    (const float*)L.post_norm->d, nullptr, 0, EPI_SWIGLU)) ||
        (rc = bgemv(e, down, I, {M(down, e->xb)}, e->hb, T, I, H, PRO_NONE, nullptr, nullptr, 0,
                    pf_residual_epi(e))) ||
        (rc = pf_tp_sum(e, T)))
      return rc;
  }
  if (!last) return 0;
  e->xch_pending = -1;
  return gemv(e, e->lm_head->type, H, {M(e->lm_head, logits ? e->logits : nullptr)}, e->xb + (size_t)(T - 1) * H,
              PRO_RMSNORM, (const float*)e->out_norm->d, nullptr, 0, EPI_ARGMAX, &e->ctl->argkey, false);
}

int launch_finalize(InfernoEngine* e, bool pdl) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(1);
  cfg.blockDim = dim3(32);
  cfg.stream = e->st;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = pdl ? 1 : 0;
  cudaError_t r = cudaLaunchKernelEx(&cfg, finalize_kernel, e->ctl, (const int*)e->prompt, e->out_tokens, e->max_out,
                                     e->xch ? e->xch_seq : (unsigned long long*)nullptr, e->xch_k,
                                     e->token_steps ? e->gdn_steps + (size_t)e->cur_seq * e->cfg.num_layers : (int*)nullptr,
                                     e->token_steps ? e->cfg.num_layers : 0);
  if (r != cudaSuccess) return set_error(INFERNO_ECUDA, "finalize launch: %s", cudaGetErrorString(r));
  mark(e, K_FINAL);
  return 0;
}

int enqueue_token(InfernoEngine* e, bool write_logits, bool pdl) {
  const InfernoConfig& c = e->cfg;
  int rc;
  e->xcur = e->x;          // the embedding row lands in x
  e->xch_k = 0;
  e->xch_pending = -1;
  e->launches = 0;
  e->trace_idx = 0;
  e->in_token = true;
  struct InTokenReset {
    InfernoEngine* e;
    ~InTokenReset() { e->in_token = false; }
  } in_token_reset{e};
  if (e->profiling) mark(e, -1), --e->launches;
  if ((rc = launch_embed_row(e->embd->type, e->embd->d, (long long)e->embd->bytes / e->embd->rows(), c.hidden_size,
                             &e->ctl->tok, e->x, c.vocab_size, e->st, pdl)))
    return set_error(INFERNO_ECUDA, "embedding launch failed (%d)", rc);
  mark(e, K_EMBED);
  for (int i = 0; i < c.num_layers; ++i)
    if ((rc = enqueue_layer(e, i, pdl))) return rc;
  if (e->sampling) write_logits = true;
  if (e->tp) {
    // vocab-split lm_head: local rows, global first-max through a u64 max
    // all-reduce of the packed (ordered value, ~index) keys
    GemvCall g;
    g.type = e->lm_head->type;
    g.inner = c.hidden_size;
    g.mats[0] = M(e->lm_head, write_logits ? e->logits_local : nullptr);
    g.nmats = 1;
    g.x = e->xcur;
    g.x_stride = c.hidden_size;
    g.pro = PRO_RMSNORM;
    g.pro_w = (const float*)e->out_norm->d;
    g.eps = c.rms_eps;
    g.epi = EPI_ARGMAX;
    g.argmax = &e->ctl->argkey;
    g.argmax_row0 = c.tp_rank * (int)e->lm_head->rows();
    g.err = e->err;
    if (e->xch) {
      g.xch_n = c.tp_size;
      g.xch_rank = c.tp_rank;
      g.xch_seq = e->xch_seq;
      g.xch_spin = e->xch_spin;
      for (int q = 0; q < c.tp_size; ++q) g.xch_parts[q] = e->xch_peer[q];
      g.xch_rk = e->xch_pending;
      g.x_next = e->xcur == e->x ? e->x2 : e->x;
    }
    if ((rc = launch_gemv(g, e->st, pdl))) return rc;
    xch_commit(e);
    mark(e, K_LMHEAD);
    ncclResult_t r = ncclAllReduce(&e->ctl->argkey, &e->ctl->argkey, 1, ncclUint64, ncclMax, e->comm, e->st);
    if (r == ncclSuccess && write_logits)
      r = ncclAllGather(e->logits_local, e->logits, (size_t)e->lm_head->rows(), ncclFloat, e->comm, e->st);
    if (r != ncclSuccess) return set_error(INFERNO_ENCCL, "lm_head collectives: %s", ncclGetErrorString(r));
    if (e->sampling && (rc = launch_sample(e->logits, c.vocab_size, *e->sampling, e->seen, -1.0f, &e->ctl->step,
                                           nullptr, &e->ctl->argkey, e->seen, e->st, pdl)))
      return rc;
    rc = launch_finalize(e, pdl);
    e->token_launches = e->launches;
    return rc;
  }
  if (!(e->ablate & 64) && (rc = gemv(e, e->lm_head->type, c.hidden_size, {M(e->lm_head, write_logits ? e->logits : nullptr)}, e->xcur,
                 PRO_RMSNORM, (const float*)e->out_norm->d, nullptr, 0, EPI_ARGMAX, &e->ctl->argkey, pdl)))
    return rc;
  // sampled decode: the drawn token replaces the argmax key (finalize reads it)
  if (e->sampling && (rc = launch_sample(e->logits, c.vocab_size, *e->sampling, e->seen, -1.0f, &e->ctl->step, nullptr,
                                         &e->ctl->argkey, e->seen, e->st, pdl)))
    return rc;
  rc = launch_finalize(e, pdl);
  e->token_launches = e->launches;
  return rc;
}

int capture(InfernoEngine* e, int ntok, bool logits, cudaGraphExec_t* out) {
  cudaGraph_t g = nullptr;
  INF_CUDA_TRY(cudaStreamBeginCapture(e->st, cudaStreamCaptureModeThreadLocal));
  int rc = 0;
  for (int t = 0; t < ntok && !rc; ++t) rc = enqueue_token(e, logits && t == ntok - 1, e->cfg.use_pdl != 0);
  cudaError_t r = cudaStreamEndCapture(e->st, &g);
  if (rc) {
    if (g) cudaGraphDestroy(g);
    return rc;
  }
  if (r != cudaSuccess) return set_error(INFERNO_ECUDA, "graph capture failed: %s", cudaGetErrorString(r));
  r = cudaGraphInstantiate(out, g, 0);
  cudaGraphDestroy(g);
  if (r != cudaSuccess) return set_error(INFERNO_ECUDA, "graph instantiate failed: %s", cudaGetErrorString(r));
  return 0;
}

int check_device_error(InfernoEngine* e) {
  int v = 0;
  INF_CUDA_TRY(cudaMemcpy(&v, e->err, sizeof v, cudaMemcpyDeviceToHost));
  if (v) {
    cudaMemset(e->err, 0, sizeof(int));
    return set_error(INFERNO_EDEVICE, "a kernel reported device error %d (1 = bounded wait timed out, 2 = bad "
                                      "argument such as a position beyond max_ctx)", v);
  }
  return 0;
}

// run `n` steps: graph replays (8-token graph for bulk) or eager launches
int capture_token_graphs(InfernoEngine* e);

int run_steps(InfernoEngine* e, int n, bool logits_last) {
  int rc;
  if (e->cfg.use_graphs && !e->dump && !e->g1 && (rc = capture_token_graphs(e))) return rc;
  if (e->cfg.use_graphs && !e->dump) {
    int left = n;
    while (left >= 8 + (logits_last ? 1 : 0)) {
      INF_CUDA_TRY(cudaGraphLaunch(e->g8, e->st));
      left -= 8;
    }
    while (left > 0) {
      INF_CUDA_TRY(cudaGraphLaunch((left == 1 && logits_last) ? e->g1_logits : e->g1, e->st));
      --left;
    }
  } else {
    for (int t = 0; t < n; ++t)
      if ((rc = enqueue_token(e, logits_last && t == n - 1, e->cfg.use_pdl != 0))) return rc;
  }
  return 0;
}

}  // namespace
}  // namespace inf

using namespace inf;

namespace inf {
namespace {

// Fused tensor-parallel exchange: every rank allocates [2 slots][N][H] 64-bit
// {value, tag} words, the CUDA IPC handles are all-gathered over the engine's
// NCCL communicator and every peer buffer is mapped.  Used when every
// residual GEMV and every RMSNorm consumer runs on the tensor-core path.
int setup_xch(InfernoEngine* e) {
  const InfernoConfig& c = e->cfg;
  const int n = c.tp_size, H = c.hidden_size;
  const char* nc = getenv("INFERNO_TP_NCCL");
  if ((nc && atoi(nc) != 0) || e->dump || n > 8 || H > 8192) return 0;
  auto ok = [](const DevTensor* t, int64_t inner) {
    return t && (t->type == T_Q4_K || t->type == T_Q6_K || t->type == T_Q6_KR) && inner % 256 == 0;
  };
  // every GEMV that reads the exchanged residual (RMSNorm inputs) and, under
  // tensor parallelism, every one that writes a partial runs on the
  // tensor-core path; expert parallelism exchanges after the expert FFN,
  // whose next reader is the next layer's first GEMV (or the lm_head)
  bool eligible = ok(e->lm_head, H);
  for (auto& L : e->layers) {
    if (L.ssm)
      eligible = eligible && ok(L.in_proj, H) && ok(L.gate, H) && (e->ep || ok(L.ssm_out, e->di));
    else
      eligible = eligible && ok(L.wq, H) && ok(L.wk, H) && ok(L.wv, H) &&
                 (e->ep || ok(L.wo, (int64_t)c.n_heads * c.head_dim));
    if (!e->ep) eligible = eligible && ok(L.ffn_gate, H) && ok(L.ffn_up, H) && ok(L.ffn_down, c.intermediate_size);
  }
  if (!eligible) return 0;
  int rc;
  unsigned long long* mine = nullptr;
  if ((rc = dalloc(e, &mine, (size_t)2 * n * H)) || (rc = dalloc(e, &e->x2, H)) ||
      (rc = dalloc(e, &e->xch_done, 1)) || (rc = dalloc(e, &e->xch_seq, 1)))
    return rc;
  cudaIpcMemHandle_t h;
  INF_CUDA_TRY(cudaIpcGetMemHandle(&h, mine));
  uint8_t* dh = nullptr;
  INF_CUDA_TRY(cudaMalloc(&dh, (size_t)n * sizeof h));
  INF_CUDA_TRY(cudaMemcpy(dh + (size_t)c.tp_rank * sizeof h, &h, sizeof h, cudaMemcpyHostToDevice));
  ncclResult_t r = ncclAllGather(dh + (size_t)c.tp_rank * sizeof h, dh, sizeof h, ncclUint8, e->comm, e->st);
  std::vector<cudaIpcMemHandle_t> all(n);
  cudaError_t ce = cudaStreamSynchronize(e->st);
  if (ce == cudaSuccess) ce = cudaMemcpy(all.data(), dh, (size_t)n * sizeof h, cudaMemcpyDeviceToHost);
  cudaFree(dh);
  if (r != ncclSuccess) return set_error(INFERNO_ENCCL, "exchange of IPC handles: %s", ncclGetErrorString(r));
  if (ce != cudaSuccess) return set_error(INFERNO_ECUDA, "exchange of IPC handles: %s", cudaGetErrorString(ce));
  for (int q = 0; q < n; ++q) {
    if (q == c.tp_rank) {
      e->xch_peer[q] = mine;
      continue;
    }
    void* ptr = nullptr;
    ce = cudaIpcOpenMemHandle(&ptr, all[q], cudaIpcMemLazyEnablePeerAccess);
    if (ce != cudaSuccess)
      return set_error(INFERNO_ECUDA, "cudaIpcOpenMemHandle(rank %d): %s", q, cudaGetErrorString(ce));
    e->xch_peer[q] = (unsigned long long*)ptr;
  }
  // every rank mapped every buffer before anyone writes into a peer
  r = ncclAllReduce(e->xch_done, e->xch_done, 1, ncclUint32, ncclSum, e->comm, e->st);
  if (r != ncclSuccess) return set_error(INFERNO_ENCCL, "exchange setup barrier: %s", ncclGetErrorString(r));
  INF_CUDA_TRY(cudaStreamSynchronize(e->st));
  e->xch = true;
  return 0;
}

}  // namespace
}  // namespace inf

extern "C" {

namespace inf {
namespace {

// Tensor-core prefill: activation staging and, per GEMM group of a prefill
// chunk, one bound of |w| (the GEMM's power-of-two weight scale).
int setup_tc_prefill(InfernoEngine* e) {
  const char* off = getenv("INFERNO_NO_TC_GEMM");
  if (off && atoi(off) != 0) return 0;
  const InfernoConfig& c = e->cfg;
  const int H = c.hidden_size;
  const size_t kmax = std::max<size_t>({(size_t)H, (size_t)e->di, (size_t)c.intermediate_size,
                                        (size_t)c.n_heads * c.head_dim});
  const size_t rows = (size_t)qgemm_rows_padded(PF_MAX_T);
  int rc;
  if ((rc = dalloc(e, (uint16_t**)&e->pf_xhi, rows * kmax)) || (rc = dalloc(e, (uint16_t**)&e->pf_xlo, rows * kmax)) ||
      (rc = dalloc(e, &e->pf_xexp, rows)) || (rc = dalloc(e, &e->qg_ws, qgemm_ws_bytes() / 4)) ||
      (rc = dalloc(e, &e->qg_tickets, QGEMM_TICKETS)))
    return rc;
  if (e->C) {
    const size_t n = (size_t)PF_MAX_T * c.ssm_nv;
    if ((rc = dalloc(e, &e->pf_gdn.qn, n * 128)) || (rc = dalloc(e, &e->pf_gdn.kn, n * 128)) ||
        (rc = dalloc(e, &e->pf_gdn.vv, n * c.ssm_dv)) || (rc = dalloc(e, &e->pf_gdn.beta, n)) ||
        (rc = dalloc(e, &e->pf_gdn.g, n)))
      return rc;
  }
  std::vector<std::vector<DevTensor*>> groups;
  for (auto& L : e->layers) {
    if (L.ssm) {
      groups.push_back({L.in_proj});
      groups.push_back({L.gate});
      groups.push_back({L.ssm_out});
    } else {
      groups.push_back({L.wq});
      if (L.wk->type == L.wv->type) groups.push_back({L.wk, L.wv});
      else groups.push_back({L.wk}), groups.push_back({L.wv});
      groups.push_back({L.wo});
    }
    if (L.ffn_gate) groups.push_back({L.ffn_gate, L.ffn_up});
    if (L.ffn_down) groups.push_back({L.ffn_down->type == T_Q6_KR ? &L.ffn_down_raw : L.ffn_down});
  }
  if ((rc = dalloc(e, &e->pf_wbounds, groups.size()))) return rc;
  for (size_t gi = 0; gi < groups.size(); ++gi) {
    float* wb = e->pf_wbounds + gi;
    bool first = true;
    for (DevTensor* t : groups[gi]) {
      if (!t || !qgemm_supported(t->type)) continue;
      if ((rc = launch_qgemm_wbound(t->type, t->d, t->rows(), (int)t->ne[0], wb, e->st, first))) return rc;
      first = false;
      t->wb = wb;
    }
  }
  return 0;
}

}  // namespace
}  // namespace inf

int inferno_engine_create(const InfernoConfig* cfg, InfernoEngine** out) {
  if (!cfg || !out) return set_error(INFERNO_EINVAL, "engine_create: null argument");
  if (cfg->struct_size != (int)sizeof(InfernoConfig))
    return set_error(INFERNO_EINVAL, "engine_create: struct_size %d != %d (header mismatch)", cfg->struct_size,
                     (int)sizeof(InfernoConfig));
  const InfernoConfig& c = *cfg;
  if (c.hidden_size <= 0 || c.hidden_size % 256 || c.num_layers <= 0 || c.vocab_size <= 0)
    return set_error(INFERNO_EINVAL, "engine_create: hidden_size must be a positive multiple of 256");
  if (c.head_dim != 256) return set_error(INFERNO_EINVAL, "engine_create: head_dim %d unsupported (256)", c.head_dim);
  if (c.ssm_dk != 128) return set_error(INFERNO_EINVAL, "engine_create: ssm state size %d unsupported (128)", c.ssm_dk);
  if (c.ssm_nk <= 0 || c.ssm_nv % c.ssm_nk) return set_error(INFERNO_EINVAL, "engine_create: nv %% nk != 0");
  if (c.max_ctx <= 0) return set_error(INFERNO_EINVAL, "engine_create: max_ctx must be positive");
  if (c.max_batch < 0 || c.max_batch > PF_MAX_T)
    return set_error(INFERNO_EINVAL, "engine_create: max_batch %d outside [1, %d]", c.max_batch, PF_MAX_T);
  if (c.max_batch > 1 && c.tp_size > 1)
    return set_error(INFERNO_EINVAL, "engine_create: batched decode runs on one GPU (tp_size 1)");
  if (c.tp_size < 1 || c.tp_rank < 0 || c.tp_rank >= c.tp_size)
    return set_error(INFERNO_EINVAL, "engine_create: tp_rank %d / tp_size %d", c.tp_rank, c.tp_size);
  if (c.tp_size > 1 && !c.nccl_unique_id)
    return set_error(INFERNO_EINVAL, "engine_create: tensor / expert parallel needs an NCCL unique id");
  if (c.tp_size > 1 && c.n_experts && c.n_experts % c.tp_size)
    return set_error(INFERNO_EINVAL, "engine_create: %d experts not divisible by %d ranks", c.n_experts, c.tp_size);
  if (c.n_experts && (c.n_experts > 1024 || c.n_experts_used <= 0 || c.n_experts_used > 16 ||
                      c.n_experts_used > c.n_experts || c.expert_ffn <= 0 || c.expert_ffn % 256 ||
                      c.n_experts_used + 1 > 16))
    return set_error(INFERNO_EINVAL, "engine_create: MoE needs <= 1024 experts, top-k in [1, 15] and an expert "
                                     "width that is a multiple of 256");
  auto* e = new InfernoEngine();
  e->cfg = c;
  e->nseq = c.max_batch > 1 ? c.max_batch : 1;
  e->ep = c.tp_size > 1 && c.n_experts > 0;
  e->tp = c.tp_size > 1 && !e->ep;
  e->dev = c.device;
  if (cudaSetDevice(e->dev) != cudaSuccess) {
    delete e;
    return set_error(INFERNO_ECUDA, "cudaSetDevice(%d) failed", c.device);
  }
  if (cudaStreamCreateWithFlags(&e->st, cudaStreamNonBlocking) != cudaSuccess) {
    delete e;
    return set_error(INFERNO_ECUDA, "stream creation failed");
  }
  cudaEventCreate(&e->ev0);
  cudaEventCreate(&e->ev1);
  if (c.tp_size > 1) {
    ncclUniqueId id;
    memcpy(&id, c.nccl_unique_id, sizeof id);
    ncclResult_t r = ncclCommInitRank(&e->comm, c.tp_size, id, c.tp_rank);
    if (r != ncclSuccess) {
      cudaStreamDestroy(e->st);
      delete e;
      return set_error(INFERNO_ENCCL, "ncclCommInitRank(rank %d of %d): %s", c.tp_rank, c.tp_size,
                       ncclGetErrorString(r));
    }
  }
  if (const char* sp = getenv("INFERNO_XCH_SPIN")) e->xch_spin = (unsigned)strtoul(sp, nullptr, 0);
  if (const char* gh = getenv("INFERNO_GDN_HEAD")) e->gdn_head = atoi(gh) != 0;
  const char* d = getenv("INFERNO_B200_DUMP");
  e->dump = d && atoi(d) != 0;
  if (const char* ab = getenv("INFERNO_B200_ABLATE")) e->ablate = (unsigned)strtoul(ab, nullptr, 0);
  if (getenv("INFERNO_B200_TRACE")) {
    if (cudaMalloc(&e->trace, 8 * 8192) != cudaSuccess) e->trace = nullptr;
    else cudaMemset(e->trace, 0, 8 * 8192);
  }
  *out = e;
  return 0;
}

int inferno_engine_upload_tensor(InfernoEngine* e, const char* name, int ggml_type, const int64_t ne[4],
                                 const void* host, size_t nbytes) {
  if (!e || !name || !ne || !host) return set_error(INFERNO_EINVAL, "upload: null argument");
  if (e->finalized) return set_error(INFERNO_ESTATE, "upload after finalize");
  if (!type_supported(ggml_type)) return set_error(INFERNO_EINVAL, "upload %s: unsupported ggml type %d", name, ggml_type);
  int64_t n = ne[0] * ne[1] * ne[2] * ne[3];
  if (ne[0] <= 0 || n <= 0 || ne[0] % qk_of(ggml_type))
    return set_error(INFERNO_EINVAL, "upload %s: bad dims", name);
  size_t want = (size_t)(n / qk_of(ggml_type)) * bb_of(ggml_type);
  if (want != nbytes)
    return set_error(INFERNO_EINVAL, "upload %s: %zu bytes given, %zu expected for its type and dims", name, nbytes,
                     want);
  INF_CUDA_TRY(cudaSetDevice(e->dev));
  DevTensor t;
  t.type = ggml_type;
  for (int i = 0; i < 4; ++i) t.ne[i] = ne[i];
  t.bytes = nbytes;
  if (cudaMalloc(&t.d, (nbytes + 255) / 256 * 256) != cudaSuccess)
    return set_error(INFERNO_ENOMEM, "upload %s: cudaMalloc(%zu) failed", name, nbytes);
  INF_CUDA_TRY(cudaMemcpy(t.d, host, nbytes, cudaMemcpyHostToDevice));
  auto it = e->tensors.find(name);
  if (it != e->tensors.end()) cudaFree(it->second.d);
  e->tensors[name] = t;
  return 0;
}

// Every tensor of a parsed GGUF file to the device, straight from the file
// mapping (the raw-bytes view of LoaderCPU.extract_tensor_cpu with
// keep_quantized, src/LoaderCPU.jl:131-155): the bytes go through two pinned
// staging buffers, so reading the mapping (page faults included) overlaps
// the DMA of the previous chunk.
int inferno_engine_load_gguf(InfernoEngine* e, const InfernoGguf* g) {
  if (!e || !g) return set_error(INFERNO_EINVAL, "load_gguf: null argument");
  if (e->finalized) return set_error(INFERNO_ESTATE, "load_gguf after finalize");
  for (const GgufTensor& t : g->tensors) {
    if (!type_supported(t.type) || !t.nbytes || t.ne[0] % qk_of(t.type))
      return set_error(INFERNO_EINVAL, "load_gguf: tensor %s has type %d / dims the engine does not take",
                       t.name.c_str(), t.type);
  }
  INF_CUDA_TRY(cudaSetDevice(e->dev));
  constexpr size_t CHUNK = 32u << 20;
  struct Staging {
    void* buf[2] = {nullptr, nullptr};
    cudaEvent_t ev[2] = {nullptr, nullptr};
    bool used[2] = {false, false};
    ~Staging() {
      for (int k = 0; k < 2; ++k) {
        if (ev[k]) { cudaEventSynchronize(ev[k]); cudaEventDestroy(ev[k]); }
        if (buf[k]) cudaFreeHost(buf[k]);
      }
    }
  } stg;
  for (int k = 0; k < 2; ++k) {
    if (cudaHostAlloc(&stg.buf[k], CHUNK, cudaHostAllocDefault) != cudaSuccess)
      return set_error(INFERNO_ENOMEM, "load_gguf: pinned staging allocation failed");
    INF_CUDA_TRY(cudaEventCreateWithFlags(&stg.ev[k], cudaEventDisableTiming));
  }
  int k = 0;
  for (const GgufTensor& t : g->tensors) {
    DevTensor dt;
    dt.type = t.type;
    for (int d = 0; d < 4; ++d) dt.ne[d] = t.ne[d];
    dt.bytes = t.nbytes;
    if (cudaMalloc(&dt.d, (t.nbytes + 255) / 256 * 256) != cudaSuccess)
      return set_error(INFERNO_ENOMEM, "load_gguf %s: cudaMalloc(%llu) failed", t.name.c_str(),
                       (unsigned long long)t.nbytes);
    const uint8_t* src = g->map + g->data_offset + t.offset;
    for (size_t off = 0; off < t.nbytes; off += CHUNK) {
      const size_t n = std::min<size_t>(CHUNK, t.nbytes - off);
      if (stg.used[k] && cudaEventSynchronize(stg.ev[k]) != cudaSuccess) {
        cudaFree(dt.d);
        return set_error(INFERNO_ECUDA, "load_gguf %s: staging copy failed", t.name.c_str());
      }
      memcpy(stg.buf[k], src + off, n);
      if (cudaMemcpyAsync((uint8_t*)dt.d + off, stg.buf[k], n, cudaMemcpyHostToDevice, e->st) != cudaSuccess ||
          cudaEventRecord(stg.ev[k], e->st) != cudaSuccess) {
        cudaStreamSynchronize(e->st);
        cudaFree(dt.d);
        return set_error(INFERNO_ECUDA, "load_gguf %s: host-to-device copy failed", t.name.c_str());
      }
      stg.used[k] = true;
      k ^= 1;
    }
    auto it = e->tensors.find(t.name);
    if (it != e->tensors.end()) {
      cudaStreamSynchronize(e->st);
      cudaFree(it->second.d);
    }
    e->tensors[t.name] = dt;
  }
  INF_CUDA_TRY(cudaStreamSynchronize(e->st));
  return 0;
}

int inferno_engine_finalize(InfernoEngine* e) {
  if (!e) return set_error(INFERNO_EINVAL, "finalize: null engine");
  if (e->finalized) return 0;
  INF_CUDA_TRY(cudaSetDevice(e->dev));
  InfernoConfig& c = e->cfg;
  int rc;
  if ((rc = require(e, "token_embd.weight", &e->embd))) return rc;
  if ((rc = require(e, "output_norm.weight", &e->out_norm, T_F32))) return rc;
  e->lm_head = find(e, "output.weight");
  if (!e->lm_head) e->lm_head = e->embd;   // tied (src/LoaderCPU.jl:358-371)
  e->lm_raw = e->lm_head;                  // GGUF layout (batched lm_head)
  // Q6_K matrices of the single-column GEMVs are regrouped per 16 rows for
  // the tensor-core path (aligned 16-byte loads; the same bytes and results).
  // The persistent kernel reads GGUF rows: no regrouping there.
  {
    const char* nr = getenv("INFERNO_NO_REPACK");
    const char* pe = getenv("INFERNO_B200_PERSISTENT");
    e->repack = !(nr && atoi(nr) != 0) && !(pe && atoi(pe) != 0);
  }
  if (e->repack && e->lm_head->type == T_Q6_K && e->lm_head->rows() % 16 == 0 && c.hidden_size % 256 == 0 &&
      (!e->tp || (c.vocab_size / c.tp_size) % 16 == 0)) {
    e->lm_packed = *e->lm_head;
    void* d = nullptr;
    if (cudaMalloc(&d, (e->lm_head->bytes + 255) / 256 * 256) != cudaSuccess)
      return set_error(INFERNO_ENOMEM, "lm_head regrouping: cudaMalloc(%zu) failed", e->lm_head->bytes);
    e->allocs.push_back(d);
    if ((rc = launch_repack_q6k(e->lm_head->d, d, (int)e->lm_head->rows(), c.hidden_size, e->st))) return rc;
    e->lm_packed.d = d;
    e->lm_packed.type = T_Q6_KR;
    e->lm_head = &e->lm_packed;
  }
  if (e->tp) {
    if (c.vocab_size % c.tp_size || e->lm_head->rows() != c.vocab_size)
      return set_error(INFERNO_EINVAL, "tensor parallel: vocab %d not divisible by %d", c.vocab_size, c.tp_size);
    const int vl = c.vocab_size / c.tp_size;
    const size_t rb = e->lm_head->bytes / (size_t)c.vocab_size;
    e->lm_view = *e->lm_head;
    e->lm_view.d = (uint8_t*)e->lm_head->d + (size_t)c.tp_rank * vl * rb;
    e->lm_view.ne[1] = vl;
    e->lm_view.bytes = (size_t)vl * rb;
    e->lm_head = &e->lm_view;
    if ((rc = dalloc(e, &e->logits_local, vl))) return rc;
  }
  if (e->embd->ne[0] != c.hidden_size || e->embd->rows() != c.vocab_size)
    return set_error(INFERNO_EINVAL, "token_embd dims do not match hidden/vocab");
  e->di = c.ssm_nv * c.ssm_dv;
  e->C = 2 * c.ssm_nk * c.ssm_dk + e->di;
  e->layers.resize(c.num_layers);
  bool any_attn = false;
  for (int i = 0; i < c.num_layers; ++i) {
    const std::string p = "blk." + std::to_string(i) + ".";
    LayerBind& L = e->layers[i];
    if ((rc = require(e, p + "attn_norm.weight", &L.attn_norm, T_F32)) ||
        (rc = require(e, p + "post_attention_norm.weight", &L.post_norm, T_F32)))
      return rc;
    L.ssm = find(e, p + "ssm_a") != nullptr;   // src/LoaderCPU.jl:431
    if (L.ssm) {
      if ((rc = require(e, p + "attn_qkv.weight", &L.in_proj)) || (rc = require(e, p + "attn_gate.weight", &L.gate)) ||
          (rc = require(e, p + "ssm_out.weight", &L.ssm_out)) ||
          (rc = require(e, p + "ssm_conv1d.weight", &L.conv1d, T_F32)) ||
          (rc = require(e, p + "ssm_alpha.weight", &L.alpha, T_F32)) ||
          (rc = require(e, p + "ssm_beta.weight", &L.beta, T_F32)) || (rc = require(e, p + "ssm_a", &L.ssm_a, T_F32)) ||
          (rc = require(e, p + "ssm_dt.bias", &L.dt_bias, T_F32)) ||
          (rc = require(e, p + "ssm_norm.weight", &L.ssm_norm, T_F32)))
        return rc;
      if (L.in_proj->rows() != e->C || L.gate->rows() != e->di || L.ssm_out->ne[0] != e->di ||
          L.conv1d->ne[0] != c.ssm_conv_kernel || L.conv1d->ne[1] != e->C || L.alpha->rows() != c.ssm_nv ||
          L.ssm_norm->ne[0] != c.ssm_dv)
        return set_error(INFERNO_EINVAL, "layer %d: GDN tensor dims do not match the config", i);
      // one slice of state per sequence of a batched decode (max_batch);
      // the single-sequence paths use the selected slice (sequence 0 by default)
      if ((rc = dalloc(e, &L.ring, (size_t)e->nseq * c.ssm_conv_kernel * e->C, true)) ||
          (rc = dalloc(e, &L.S, (size_t)e->nseq * c.ssm_nv * c.ssm_dv * c.ssm_dk, true)) ||
          (rc = dalloc(e, &L.done, 4)))
        return rc;
      if (!e->gdn_steps && (rc = dalloc(e, &e->gdn_steps, (size_t)e->nseq * c.num_layers, true))) return rc;
      L.step = e->gdn_steps + i;
      L.ring0 = L.ring;
      L.S0 = L.S;
    } else {
      any_attn = true;
      if ((rc = require(e, p + "attn_q.weight", &L.wq)) || (rc = require(e, p + "attn_k.weight", &L.wk)) ||
          (rc = require(e, p + "attn_v.weight", &L.wv)) || (rc = require(e, p + "attn_output.weight", &L.wo)) ||
          (rc = require(e, p + "attn_q_norm.weight", &L.q_norm, T_F32)) ||
          (rc = require(e, p + "attn_k_norm.weight", &L.k_norm, T_F32)))
        return rc;
      if (L.wq->rows() != 2LL * c.n_heads * c.head_dim || L.wk->rows() != (int64_t)c.n_kv_heads * c.head_dim ||
          L.wo->ne[0] != (int64_t)c.n_heads * c.head_dim)
        return set_error(INFERNO_EINVAL, "layer %d: attention tensor dims do not match the config", i);
      size_t kv = (size_t)c.max_ctx * c.n_kv_heads * c.head_dim;
      if ((rc = dalloc(e, &L.kc, kv * e->nseq, true)) || (rc = dalloc(e, &L.vc, kv * e->nseq, true))) return rc;
      L.kc0 = L.kc;
      L.vc0 = L.vc;
    }
    if (c.n_experts) {
      const int E = c.n_experts, Ie = c.expert_ffn;
      const int El = e->ep ? E / c.tp_size : E;   // experts held by this rank
      if ((rc = require(e, p + "ffn_gate_inp.weight", &L.router, T_F32)) ||
          (rc = require(e, p + "ffn_gate_exps.weight", &L.exp_gate)) ||
          (rc = require(e, p + "ffn_up_exps.weight", &L.exp_up)) ||
          (rc = require(e, p + "ffn_down_exps.weight", &L.exp_down)))
        return rc;
      if (L.router->rows() != E || L.router->ne[0] != c.hidden_size || L.exp_gate->ne[0] != c.hidden_size ||
          L.exp_gate->ne[1] != Ie || L.exp_gate->ne[2] != El || L.exp_up->type != L.exp_gate->type ||
          L.exp_up->ne[1] != Ie || L.exp_up->ne[2] != El || L.exp_down->ne[0] != Ie ||
          L.exp_down->ne[1] != c.hidden_size || L.exp_down->ne[2] != El)
        return set_error(INFERNO_EINVAL, "layer %d: MoE tensor dims do not match the config", i);
      L.sh_gate = find(e, p + "ffn_gate_shexp.weight");
      if (L.sh_gate) {
        if ((rc = require(e, p + "ffn_up_shexp.weight", &L.sh_up)) ||
            (rc = require(e, p + "ffn_down_shexp.weight", &L.sh_down)))
          return rc;
        if (L.sh_gate->rows() != Ie || L.sh_down->ne[0] != Ie || L.sh_down->type != L.exp_down->type ||
            L.sh_up->type != L.sh_gate->type)
          return set_error(INFERNO_EINVAL,
                           "layer %d: the shared expert must have the routed experts' width and down type", i);
      }
      continue;
    }
    if ((rc = require(e, p + "ffn_gate.weight", &L.ffn_gate)) || (rc = require(e, p + "ffn_up.weight", &L.ffn_up)) ||
        (rc = require(e, p + "ffn_down.weight", &L.ffn_down)))
      return rc;
    if (L.ffn_gate->rows() != c.intermediate_size || L.ffn_down->ne[0] != c.intermediate_size)
      return set_error(INFERNO_EINVAL, "layer %d: FFN dims do not match the config", i);
    // (rows of more than 8192 inputs do not fit the tensor-core GEMV's shared
    // memory next to their staged activations: they stay GGUF-layout Q6_K on
    // the CUDA-core path)
    if (e->repack && L.ffn_down->type == T_Q6_K && L.ffn_down->rows() % 16 == 0 && c.intermediate_size % 256 == 0 &&
        c.intermediate_size <= 8192) {
      void* d = nullptr;
      if (cudaMalloc(&d, (L.ffn_down->bytes + 255) / 256 * 256) != cudaSuccess)
        return set_error(INFERNO_ENOMEM, "ffn_down regrouping: cudaMalloc failed");
      if ((rc = launch_repack_q6k(L.ffn_down->d, d, (int)L.ffn_down->rows(), c.intermediate_size, e->st))) {
        cudaFree(d);
        return rc;
      }
      INF_CUDA_TRY(cudaStreamSynchronize(e->st));
      L.ffn_down_raw = *L.ffn_down;          // kept for the batched (prefill) GEMVs
      e->allocs.push_back(L.ffn_down_raw.d);
      L.ffn_down->d = d;
      L.ffn_down->type = T_Q6_KR;
    }
  }
  const int H = c.hidden_size;
  if ((rc = dalloc(e, &e->x, H)) || (rc = dalloc(e, &e->qkv, e->C)) || (rc = dalloc(e, &e->z, e->di)) ||
      (rc = dalloc(e, &e->y, e->di)) || (rc = dalloc(e, &e->qg, (size_t)2 * c.n_heads * c.head_dim)) ||
      (rc = dalloc(e, &e->k, (size_t)c.n_kv_heads * c.head_dim)) ||
      (rc = dalloc(e, &e->v, (size_t)c.n_kv_heads * c.head_dim)) ||
      (rc = dalloc(e, &e->o, (size_t)c.n_heads * c.head_dim)) ||
      (rc = dalloc(e, &e->h, std::max(1, c.intermediate_size))) ||
      (rc = dalloc(e, &e->logits, c.vocab_size)) || (rc = dalloc(e, &e->hidden, (size_t)c.num_layers * H)) ||
      (rc = dalloc(e, &e->ctl, 1)) || (rc = dalloc(e, &e->prompt, c.max_ctx + 8)) ||
      (rc = dalloc(e, &e->out_tokens, c.max_ctx + 8)) || (rc = dalloc(e, &e->err, 1)))
    return rc;
  if (c.n_experts) {
    const int K = c.n_experts_used;
    if ((rc = dalloc(e, &e->moe_logits, c.n_experts)) || (rc = dalloc(e, &e->moe_idx, K + 1)) ||
        (rc = dalloc(e, &e->moe_w, K + 1)) || (rc = dalloc(e, &e->moe_h, (size_t)(K + 1) * c.expert_ffn)) ||
        (rc = dalloc(e, &e->moe_y, (size_t)(K + 1) * H)))
      return rc;
  }
  {
    // fused in_proj + GDN (one value head per q/k group, Q4_K projections):
    // opt-in -- its cluster launch cannot overlap the preceding kernel under
    // programmatic dependent launch and measured slower than the two kernels
    // (0.79 vs 0.67 ms/token on qwen35-0.8b)
    const char* nf = getenv("INFERNO_B200_FUSED_GDN");
    const char* pe = getenv("INFERNO_B200_PERSISTENT");
    const bool want = (nf && atoi(nf) != 0) && !(pe && atoi(pe) != 0) && c.tp_size == 1 && !e->dump &&
                      c.ssm_nk == c.ssm_nv && c.ssm_dk == 128 && c.ssm_dv == 128 && c.ssm_conv_kernel <= 4 &&
                      H % 256 == 0 && H <= 8192;
    for (auto& L : e->layers) {
      if (!want || !L.ssm || L.in_proj->type != T_Q4_K || L.gate->type != T_Q4_K) continue;
      const size_t rb = (size_t)(H / 256) * 144, blk = 128 * rb;
      const int nv = c.ssm_nv, nk = c.ssm_nk;
      if ((rc = dalloc(e, (uint8_t**)&L.wperm, (size_t)nv * 512 * rb))) return rc;
      const uint8_t* ip = (const uint8_t*)L.in_proj->d;
      const uint8_t* gp = (const uint8_t*)L.gate->d;
      uint8_t* dst = (uint8_t*)L.wperm;
      for (int h = 0; h < nv; ++h) {
        INF_CUDA_TRY(cudaMemcpyAsync(dst + (size_t)(4 * h + 0) * blk, ip + (size_t)h * blk, blk, cudaMemcpyDeviceToDevice, e->st));
        INF_CUDA_TRY(cudaMemcpyAsync(dst + (size_t)(4 * h + 1) * blk, ip + (size_t)(nk + h) * blk, blk, cudaMemcpyDeviceToDevice, e->st));
        INF_CUDA_TRY(cudaMemcpyAsync(dst + (size_t)(4 * h + 2) * blk, ip + (size_t)(2 * nk + h) * blk, blk, cudaMemcpyDeviceToDevice, e->st));
        INF_CUDA_TRY(cudaMemcpyAsync(dst + (size_t)(4 * h + 3) * blk, gp + (size_t)h * blk, blk, cudaMemcpyDeviceToDevice, e->st));
      }
    }
  }
  // the decode token's finalize kernel advances the GDN step counters unless a
  // fused in_proj + GDN layer advances its own
  e->token_steps = e->gdn_steps != nullptr;
  for (auto& L : e->layers)
    if (L.wperm) e->token_steps = false;
  e->xcur = e->x;
  if ((e->tp || e->ep) && (rc = setup_xch(e))) return rc;
  {
    const char* np = getenv("INFERNO_B200_NO_PREFILL");
    e->prefill = !(np && atoi(np) != 0) && !c.n_experts && !e->dump;
    if (e->prefill || e->nseq > 1) {
      const size_t T = PF_MAX_T;
      if ((rc = dalloc(e, &e->xb, T * H)) || (rc = dalloc(e, &e->qkvb, T * e->C)) ||
          (rc = dalloc(e, &e->zb, T * e->di)) || (rc = dalloc(e, &e->yb, T * e->di)) ||
          (rc = dalloc(e, &e->qgb, T * 2 * c.n_heads * c.head_dim)) ||
          (rc = dalloc(e, &e->kb, T * c.n_kv_heads * c.head_dim)) ||
          (rc = dalloc(e, &e->vb, T * c.n_kv_heads * c.head_dim)) ||
          (rc = dalloc(e, &e->ob, T * c.n_heads * c.head_dim)) || (rc = dalloc(e, &e->hb, T * c.intermediate_size)))
        return rc;
      if ((rc = setup_tc_prefill(e))) return rc;
    }
  }
  e->max_out = c.max_ctx + 8;
  // attention splits: multiples of 32 positions, at most 128 splits
  e->split_len = attn_split_len(c.max_ctx);
  if (const char* sl = getenv("INFERNO_ATT_SPLIT")) {      // measurement knob: positions per split
    const int v = atoi(sl);
    if (v >= 32 && v % 32 == 0 && (c.max_ctx + v - 1) / v <= 1024) e->split_len = v;
  }
  e->nsplit = (c.max_ctx + e->split_len - 1) / e->split_len;
  e->rd = (int)std::lround(c.head_dim * (double)c.partial_rotary_factor);   // src/LoaderCPU.jl:375
  if (any_attn) {
    // [PF_MAX_T] x the decode sizes: the chunked prefill runs T queries at once
    if ((rc = dalloc(e, &e->part_o, (size_t)PF_MAX_T * c.n_heads * e->nsplit * c.head_dim)) ||
        (rc = dalloc(e, &e->part_ml, (size_t)PF_MAX_T * c.n_heads * e->nsplit * 2)) ||
        (rc = dalloc(e, &e->att_counters, (size_t)PF_MAX_T * c.n_heads)))
      return rc;
    std::vector<float> cs, sn;
    build_rope(c.max_ctx, e->rd, c.rope_theta, cs, sn);
    if ((rc = dalloc(e, &e->rope_cos, cs.size() + 1)) || (rc = dalloc(e, &e->rope_sin, sn.size() + 1))) return rc;
    INF_CUDA_TRY(cudaMemcpy(e->rope_cos, cs.data(), cs.size() * 4, cudaMemcpyHostToDevice));
    INF_CUDA_TRY(cudaMemcpy(e->rope_sin, sn.data(), sn.size() * 4, cudaMemcpyHostToDevice));
  }
  {
    const char* pe = getenv("INFERNO_B200_PERSISTENT");
    // opt-in: the per-stage grid barrier currently costs more than PDL-chained
    // graph launches (0.96 vs 0.72 ms/token on qwen35-0.8b)
    e->persistent = !e->dump && !c.n_experts && c.tp_size == 1 && e->nseq == 1 && (pe && atoi(pe) != 0) && (e->embd->type == T_Q6_K || e->embd->type == T_Q4_K ||
                                                            e->embd->type == T_Q8_0 || e->embd->type == T_F32);
    if (e->persistent && (rc = build_persistent(e))) return rc;
  }
  INF_CUDA_TRY(cudaDeviceSynchronize());
  e->finalized = true;
  if (c.use_graphs && !e->dump && (rc = capture_token_graphs(e))) {
    e->finalized = false;
    return rc;
  }
  return 0;
}

}  // extern "C"

namespace inf {
namespace {

int capture_token_graphs(InfernoEngine* e) {
  int rc;
  if ((rc = capture(e, 1, false, &e->g1)) || (rc = capture(e, 1, true, &e->g1_logits)) ||
      (rc = capture(e, 8, false, &e->g8)))
    return rc;
  return 0;
}

void drop_graphs(InfernoEngine* e) {
  for (cudaGraphExec_t* g : {&e->g1, &e->g1_logits, &e->g8})
    if (*g) {
      cudaGraphExecDestroy(*g);
      *g = nullptr;
    }
  for (auto& kv : e->pf_graphs) cudaGraphExecDestroy(kv.second);
  e->pf_graphs.clear();
  e->pf_seen.clear();
}

// Bind the single-sequence calls (forward, decode, layer) to state slice b.
// The captured graphs hold the previous slice's pointers: they are dropped
// and captured again on next use.
int select_seq(InfernoEngine* e, int b) {
  if (b < 0 || b >= e->nseq) return set_error(INFERNO_EINVAL, "sequence %d outside [0, %d)", b, e->nseq);
  if (b == e->cur_seq) return 0;
  const InfernoConfig& c = e->cfg;
  const size_t kv = (size_t)c.max_ctx * c.n_kv_heads * c.head_dim;
  for (int i = 0; i < c.num_layers; ++i) {
    LayerBind& L = e->layers[i];
    if (L.ssm) {
      L.ring = L.ring0 + (size_t)b * c.ssm_conv_kernel * e->C;
      L.S = L.S0 + (size_t)b * c.ssm_nv * c.ssm_dv * c.ssm_dk;
      L.step = e->gdn_steps + (size_t)b * c.num_layers + i;
    } else {
      L.kc = L.kc0 + (size_t)b * kv;
      L.vc = L.vc0 + (size_t)b * kv;
    }
  }
  INF_CUDA_TRY(cudaStreamSynchronize(e->st));
  drop_graphs(e);
  e->cur_seq = b;
  return 0;
}

// After a batched step: per sequence the argmax becomes its next token, its
// output slot is written and its position and GDN step counters advance.
__global__ void batch_finalize_kernel(int B, int nl, unsigned long long* keys, int* tok, int* pos, int* out,
                                      int* step_ctr, int* steps) {
  pdl_wait();
  pdl_trigger();
  const int st = *step_ctr;
  for (int b = threadIdx.x; b < B; b += blockDim.x) {
    const unsigned long long key = keys[b];
    const int am = (int)(0xffffffffu - (uint32_t)(key & 0xffffffffull));
    tok[b] = am;
    out[st * B + b] = am;
    pos[b] += 1;
    keys[b] = 0ull;
  }
  if (steps)
    for (int i = threadIdx.x; i < B * nl; i += blockDim.x) steps[i] += 1;
  __syncthreads();
  if (threadIdx.x == 0) *step_ctr = st + 1;
}

// One lockstep decode step of sequences 0..B-1 (tokens bt_tok, positions
// bt_pos): the prefill machinery with one column per sequence, the GDN and
// attention kernels indexing each sequence's own state slice.
int enqueue_batch_step(InfernoEngine* e, int B) {
  const InfernoConfig& c = e->cfg;
  const int H = c.hidden_size, I = c.intermediate_size, hdq = c.n_heads * c.head_dim;
  const int kvd = c.n_kv_heads * c.head_dim;
  const size_t kvs = (size_t)c.max_ctx * kvd;
  int rc;
  if ((rc = launch_embed_row(e->embd->type, e->embd->d, (long long)e->embd->bytes / e->embd->rows(), H, e->bt_tok,
                             e->xb, c.vocab_size, e->st, false, B)))
    return set_error(INFERNO_ECUDA, "batch embedding launch failed (%d)", rc);
  for (int li = 0; li < c.num_layers; ++li) {
    LayerBind& L = e->layers[li];
    const float* an = (const float*)L.attn_norm->d;
    if (L.ssm) {
      if ((rc = bgemv(e, L.in_proj, H, {M(L.in_proj, e->qkvb)}, e->xb, B, H, e->C, PRO_RMSNORM, an, nullptr, 0,
                      EPI_STORE)) ||
          (rc = bgemv(e, L.gate, H, {M(L.gate, e->zb)}, e->xb, B, H, e->di, PRO_RMSNORM, an, nullptr, 0, EPI_STORE,
                      L.in_proj->wb && L.gate->wb)))
        return rc;
      GdnParams g{};
      g.x = e->xb;
      g.in_norm = an;
      g.eps = c.rms_eps;
      g.H = H;
      g.nv = c.ssm_nv;
      g.nk = c.ssm_nk;
      g.dv = c.ssm_dv;
      g.K = c.ssm_conv_kernel;
      g.C = e->C;
      g.qkv = e->qkvb;
      g.conv_w = (const float*)L.conv1d->d;
      g.ring = L.ring0;
      g.w_alpha = (const float*)L.alpha->d;
      g.w_beta = (const float*)L.beta->d;
      g.ssm_a = (const float*)L.ssm_a->d;
      g.dt_bias = (const float*)L.dt_bias->d;
      g.S = L.S0;
      g.y = e->yb;
      g.step = e->gdn_steps + li;
      g.done = L.done;
      g.self_advance = 0;
      g.z = e->zb;
      g.out_norm = (const float*)L.ssm_norm->d;
      g.xs = H;
      g.qkvs = e->C;
      g.zys = e->di;
      g.Ss = (long long)c.ssm_nv * c.ssm_dv * c.ssm_dk;
      g.rings = (long long)c.ssm_conv_kernel * e->C;
      g.steps_stride = c.num_layers;
      if ((rc = launch_gdn_head(g, e->st, false, B))) return rc;
      mark(e, K_GDN);
      if ((rc = bgemv(e, L.ssm_out, e->di, {M(L.ssm_out, e->xb)}, e->yb, B, e->di, H, PRO_NONE, nullptr, nullptr, 0,
                      EPI_ADD)))
        return rc;
    } else {
      if ((rc = bgemv(e, L.wq, H, {M(L.wq, e->qgb)}, e->xb, B, H, 2 * hdq, PRO_RMSNORM, an, nullptr, 0, EPI_STORE)))
        return rc;
      if (L.wk->type == L.wv->type) {
        if ((rc = bgemv(e, L.wk, H, {M(L.wk, e->kb), M(L.wv, e->vb)}, e->xb, B, H, kvd, PRO_RMSNORM, an, nullptr, 0,
                        EPI_STORE, L.wq->wb && L.wk->wb)))
          return rc;
      } else if ((rc = bgemv(e, L.wk, H, {M(L.wk, e->kb)}, e->xb, B, H, kvd, PRO_RMSNORM, an, nullptr, 0, EPI_STORE)) ||
                 (rc = bgemv(e, L.wv, H, {M(L.wv, e->vb)}, e->xb, B, H, kvd, PRO_RMSNORM, an, nullptr, 0, EPI_STORE))) {
        return rc;
      }
      AttnParams a{};
      a.qg = e->qgb;
      a.k = e->kb;
      a.v = e->vb;
      a.q_norm = (const float*)L.q_norm->d;
      a.k_norm = (const float*)L.k_norm->d;
      a.eps = c.rms_eps;
      a.rope_cos = e->rope_cos;
      a.rope_sin = e->rope_sin;
      a.rd = e->rd;
      a.kc = L.kc0;
      a.vc = L.vc0;
      a.nh = c.n_heads;
      a.nkv = c.n_kv_heads;
      a.ctx = c.max_ctx;
      a.split_len = e->split_len;
      a.nsplit = e->nsplit;
      a.pos = e->bt_pos;
      a.part_o = e->part_o;
      a.part_ml = e->part_ml;
      a.counters = e->att_counters;
      a.out = e->ob;
      a.err = e->err;
      a.qgs = 2LL * hdq;
      a.kvs = kvd;
      a.outs = hdq;
      a.caches = (long long)kvs;
      if ((rc = launch_attn_decode(a, e->st, false, B))) return rc;
      mark(e, K_ATTN);
      if ((rc = bgemv(e, L.wo, hdq, {M(L.wo, e->xb)}, e->ob, B, hdq, H, PRO_NONE, nullptr, nullptr, 0, EPI_ADD)))
        return rc;
    }
    if (c.n_experts) {
      // MoE FFN per sequence (each token routes to its own experts, as the
      // reference's token loop does, src/Model.jl:478-561): the
      // single-token expert chain on column b
      for (int b = 0; b < B; ++b) {
        e->xcur = e->xb + (size_t)b * H;
        if ((rc = enqueue_moe(e, L, false))) {
          e->xcur = e->x;
          return rc;
        }
      }
      e->xcur = e->x;
      continue;
    }
    DevTensor* down = L.ffn_down->type == T_Q6_KR ? &L.ffn_down_raw : L.ffn_down;
    if ((rc = bgemv(e, L.ffn_gate, H, {M(L.ffn_gate, e->hb), M(L.ffn_up, nullptr)}, e->xb, B, H, I, PRO_RMSNORM,
                    (const float*)L.post_norm->d, nullptr, 0, EPI_SWIGLU)) ||
        (rc = bgemv(e, down, I, {M(down, e->xb)}, e->hb, B, I, H, PRO_NONE, nullptr, nullptr, 0, EPI_ADD)))
      return rc;
  }
  // lm_head + first-max argmax per sequence (GGUF-layout rows, B columns)
  {
    GemvCall g;
    g.type = e->lm_raw->type;
    g.inner = H;
    g.mats[0] = GemvMat{e->lm_raw->d, nullptr, (int)e->lm_raw->rows()};
    g.nmats = 1;
    g.nb = B;
    g.x = e->xb;
    g.x_stride = H;
    g.y_stride = c.vocab_size;
    g.pro = PRO_RMSNORM;
    g.pro_w = (const float*)e->out_norm->d;
    g.eps = c.rms_eps;
    g.epi = EPI_ARGMAX;
    g.argmax = e->bt_keys;
    g.err = e->err;
    if ((rc = launch_gemv(g, e->st, false))) return rc;
    mark(e, K_LMHEAD);
  }
  batch_finalize_kernel<<<1, 128, 0, e->st>>>(B, c.num_layers, e->bt_keys, e->bt_tok, e->bt_pos, e->bt_out,
                                              e->bt_step, e->gdn_steps);
  INF_CUDA_TRY(cudaGetLastError());
  return 0;
}

}  // namespace
}  // namespace inf

extern "C" {

int inferno_select_sequence(InfernoEngine* e, int seq) {
  if (!e || !e->finalized) return set_error(INFERNO_ESTATE, "select_sequence: engine not finalized");
  INF_CUDA_TRY(cudaSetDevice(e->dev));
  return inf::select_seq(e, seq);
}

int inferno_decode_batch(InfernoEngine* e, const int32_t* toks, const int32_t* pos, int B, int n_steps,
                         int32_t* out_tokens) {
  using namespace inf;
  if (!e || !e->finalized) return set_error(INFERNO_ESTATE, "decode_batch: engine not finalized");
  INF_CUDA_TRY(cudaSetDevice(e->dev));
  const InfernoConfig& c = e->cfg;
  if (!toks || !pos || !out_tokens || B < 1 || B > e->nseq || n_steps < 1)
    return set_error(INFERNO_EINVAL, "decode_batch: B must be in [1, max_batch = %d]", e->nseq);
  if (!e->xb) return set_error(INFERNO_ESTATE, "decode_batch: the batched buffers are not allocated");
  for (int b = 0; b < B; ++b) {
    if (toks[b] < 0 || toks[b] >= c.vocab_size) return set_error(INFERNO_EINVAL, "decode_batch: token out of range");
    if (pos[b] < 0 || pos[b] + n_steps > c.max_ctx)
      return set_error(INFERNO_EINVAL, "decode_batch: sequence %d positions exceed max_ctx", b);
  }
  int rc;
  if (!e->bt_tok) {
    if ((rc = dalloc(e, &e->bt_tok, e->nseq)) || (rc = dalloc(e, &e->bt_pos, e->nseq)) ||
        (rc = dalloc(e, &e->bt_keys, e->nseq)) || (rc = dalloc(e, &e->bt_step, 1)))
      return rc;
  }
  if (e->bt_out_cap < n_steps * B) {
    if ((rc = dalloc(e, &e->bt_out, (size_t)n_steps * B))) return rc;
    e->bt_out_cap = n_steps * B;
  }
  // the batched kernels address every sequence's slice from sequence 0's
  if ((rc = select_seq(e, 0))) return rc;
  INF_CUDA_TRY(cudaMemcpyAsync(e->bt_tok, toks, (size_t)B * 4, cudaMemcpyHostToDevice, e->st));
  INF_CUDA_TRY(cudaMemcpyAsync(e->bt_pos, pos, (size_t)B * 4, cudaMemcpyHostToDevice, e->st));
  INF_CUDA_TRY(cudaMemsetAsync(e->bt_keys, 0, (size_t)B * 8, e->st));
  INF_CUDA_TRY(cudaMemsetAsync(e->bt_step, 0, 4, e->st));
  cudaGraphExec_t ge = nullptr;
  if (c.use_graphs) {
    auto it = e->bt_graphs.find(B);
    if (it == e->bt_graphs.end()) {
      // first call for this B runs eagerly (kernel attributes, scratch), the
      // step is captured once that worked
      if ((rc = enqueue_batch_step(e, B))) return rc;
      INF_CUDA_TRY(cudaStreamSynchronize(e->st));
      cudaGraph_t g = nullptr;
      INF_CUDA_TRY(cudaStreamBeginCapture(e->st, cudaStreamCaptureModeThreadLocal));
      rc = enqueue_batch_step(e, B);
      cudaError_t r1 = cudaStreamEndCapture(e->st, &g);
      if (rc) {
        if (g) cudaGraphDestroy(g);
        return rc;
      }
      if (r1 != cudaSuccess) return set_error(INFERNO_ECUDA, "batch capture: %s", cudaGetErrorString(r1));
      r1 = cudaGraphInstantiate(&ge, g, 0);
      cudaGraphDestroy(g);
      if (r1 != cudaSuccess) return set_error(INFERNO_ECUDA, "batch graph: %s", cudaGetErrorString(r1));
      e->bt_graphs[B] = ge;
      --n_steps;     // the eager step already ran
    } else {
      ge = it->second;
    }
  }
  INF_CUDA_TRY(cudaEventRecord(e->ev0, e->st));
  for (int t = 0; t < n_steps; ++t) {
    if (ge) INF_CUDA_TRY(cudaGraphLaunch(ge, e->st));
    else if ((rc = enqueue_batch_step(e, B))) return rc;
  }
  INF_CUDA_TRY(cudaEventRecord(e->ev1, e->st));
  INF_CUDA_TRY(cudaStreamSynchronize(e->st));
  float ms = 0.f;
  cudaEventElapsedTime(&ms, e->ev0, e->ev1);
  e->last_ms = ms;
  int done_steps = 0;
  INF_CUDA_TRY(cudaMemcpy(&done_steps, e->bt_step, 4, cudaMemcpyDeviceToHost));
  INF_CUDA_TRY(cudaMemcpy(out_tokens, e->bt_out, (size_t)done_steps * B * 4, cudaMemcpyDeviceToHost));
  return check_device_error(e);
}

}  // extern "C"

namespace inf {
namespace {

int pk_add_gemv(InfernoEngine* e, std::vector<PkStage>& v, int type, int inner, std::initializer_list<GemvMat> mats,
                const float* x, int pro, const float* pro_w, const float* pro_z, int group, int epi, bool embed_row) {
  GemvCall c;
  c.type = type;
  c.inner = inner;
  for (auto& m : mats) c.mats[c.nmats++] = m;
  c.x = x;
  c.pro = pro;
  c.pro_w = pro_w;
  c.pro_z = pro_z;
  c.pro_group = group;
  c.eps = e->cfg.rms_eps;
  c.epi = epi;
  PkStage S{};
  int rc = pk_plan_gemv(c, e->pk_slot, num_sms(e->dev), &S);
  if (rc) return rc;
  S.embed_row = embed_row ? 1 : 0;
  S.g.err = e->err;
  S.g.argmax = nullptr;
  e->pk_inner_pad = std::max(e->pk_inner_pad, (inner + GEMV_CHUNK - 1) / GEMV_CHUNK * GEMV_CHUNK);
  v.push_back(S);
  return 0;
}

// The stage program of one token (see decode.cu).
int build_persistent(InfernoEngine* e) {
  const InfernoConfig& c = e->cfg;
  const int H = c.hidden_size;
  e->pk_hidden_pad = (H + 31) / 32 * 32;
  // ring slots: what is left of 227 KB after the activation buffers
  int max_inner = H;
  max_inner = std::max(max_inner, e->di);
  max_inner = std::max(max_inner, c.intermediate_size);
  max_inner = std::max(max_inner, c.n_heads * c.head_dim);
  e->pk_inner_pad = (max_inner + GEMV_CHUNK - 1) / GEMV_CHUNK * GEMV_CHUNK;
  const size_t fixed = pk_smem_bytes(e->pk_hidden_pad, e->pk_inner_pad, 0);
  long long slot = ((long long)(227 * 1024 - 1024) - (long long)fixed) / 5;
  slot = slot / 128 * 128;
  if (slot < 16 * 1024) return set_error(INFERNO_EINVAL, "persistent kernel: no room for weight slots");
  e->pk_slot = (int)std::min<long long>(slot, 48 * 1024);
  std::vector<PkStage> v;
  int rc;
  for (int li = 0; li < c.num_layers; ++li) {
    LayerBind& L = e->layers[li];
    const bool first = li == 0;
    if (L.ssm) {
      if (L.in_proj->type != L.gate->type) return set_error(INFERNO_EINVAL, "persistent: in_proj/gate types differ");
      if ((rc = pk_add_gemv(e, v, L.in_proj->type, H, {M(L.in_proj, e->qkv), M(L.gate, e->z)}, e->x, PRO_RMSNORM,
                            (const float*)L.attn_norm->d, nullptr, 0, EPI_STORE, first)))
        return rc;
      PkStage g{};
      g.kind = PK_GDN;
      GdnParams& d = g.d;
      d.x = e->x;
      d.in_norm = (const float*)L.attn_norm->d;
      d.eps = c.rms_eps;
      d.H = H;
      d.nv = c.ssm_nv;
      d.nk = c.ssm_nk;
      d.dv = c.ssm_dv;
      d.K = c.ssm_conv_kernel;
      d.C = e->C;
      d.qkv = e->qkv;
      d.conv_w = (const float*)L.conv1d->d;
      d.ring = L.ring;
      d.w_alpha = (const float*)L.alpha->d;
      d.w_beta = (const float*)L.beta->d;
      d.ssm_a = (const float*)L.ssm_a->d;
      d.dt_bias = (const float*)L.dt_bias->d;
      d.S = L.S;
      d.y = e->y;
      d.step = L.step;
      d.done = L.done;
      if (c.ssm_conv_kernel > 8 || c.ssm_dv % 16) return set_error(INFERNO_EINVAL, "persistent: GDN dims");
      v.push_back(g);
      if ((rc = pk_add_gemv(e, v, L.ssm_out->type, e->di, {M(L.ssm_out, e->x)}, e->y, PRO_HEADNORM_GATE,
                            (const float*)L.ssm_norm->d, e->z, c.ssm_dv, EPI_ADD, false)))
        return rc;
    } else {
      if (L.wq->type != L.wk->type || L.wk->type != L.wv->type)
        return set_error(INFERNO_EINVAL, "persistent: q/k/v types differ");
      if ((rc = pk_add_gemv(e, v, L.wq->type, H, {M(L.wq, e->qg), M(L.wk, e->k), M(L.wv, e->v)}, e->x, PRO_RMSNORM,
                            (const float*)L.attn_norm->d, nullptr, 0, EPI_STORE, first)))
        return rc;
      PkStage a{};
      a.kind = PK_ATTN;
      AttnParams& p = a.a;
      p.qg = e->qg;
      p.k = e->k;
      p.v = e->v;
      p.q_norm = (const float*)L.q_norm->d;
      p.k_norm = (const float*)L.k_norm->d;
      p.eps = c.rms_eps;
      p.rope_cos = e->rope_cos;
      p.rope_sin = e->rope_sin;
      p.rd = e->rd;
      p.kc = L.kc;
      p.vc = L.vc;
      p.nh = c.n_heads;
      p.nkv = c.n_kv_heads;
      p.ctx = c.max_ctx;
      p.split_len = e->split_len;
      p.nsplit = e->nsplit;
      p.part_o = e->part_o;
      p.part_ml = e->part_ml;
      p.counters = e->att_counters;
      p.out = e->o;
      p.err = e->err;
      v.push_back(a);
      if ((rc = pk_add_gemv(e, v, L.wo->type, c.n_heads * c.head_dim, {M(L.wo, e->x)}, e->o, PRO_NONE, nullptr,
                            nullptr, 0, EPI_ADD, false)))
        return rc;
    }
    if ((rc = pk_add_gemv(e, v, L.ffn_gate->type, H, {M(L.ffn_gate, e->h), M(L.ffn_up, nullptr)}, e->x, PRO_RMSNORM,
                          (const float*)L.post_norm->d, nullptr, 0, EPI_SWIGLU, false)))
      return rc;
    if ((rc = pk_add_gemv(e, v, L.ffn_down->type, c.intermediate_size, {M(L.ffn_down, e->xcur)}, e->h, PRO_NONE,
                          nullptr, nullptr, 0, EPI_ADD, false)))
      return rc;
  }
  if ((rc = pk_add_gemv(e, v, e->lm_head->type, H, {M(e->lm_head, e->logits)}, e->x, PRO_RMSNORM,
                        (const float*)e->out_norm->d, nullptr, 0, EPI_ARGMAX, false)))
    return rc;
  for (auto& s : v) s.slot_bytes = e->pk_slot;
  e->pk_nstages = (int)v.size();
  e->pk_smem = pk_smem_bytes(e->pk_hidden_pad, e->pk_inner_pad, e->pk_slot);
  if ((rc = dalloc(e, &e->pk_stages, v.size())) || (rc = dalloc(e, &e->pk_barrier, 1)) ||
      (rc = dalloc(e, &e->pk_abort, 1)))
    return rc;
  INF_CUDA_TRY(cudaMemcpy(e->pk_stages, v.data(), v.size() * sizeof(PkStage), cudaMemcpyHostToDevice));
  return 0;
}

int run_persistent(InfernoEngine* e, int tok0, int pos0, int n_prompt, int n_steps) {
  PkParams P{};
  P.stages = e->pk_stages;
  P.n_stages = e->pk_nstages;
  P.n_steps = n_steps;
  P.tok0 = tok0;
  P.pos0 = pos0;
  P.n_prompt = n_prompt;
  P.prompt = e->prompt;
  P.out_tokens = e->out_tokens;
  P.max_out = e->max_out;
  P.ctl_last = &e->ctl->last;
  P.argkey = &e->ctl->argkey;
  P.barrier = e->pk_barrier;
  P.abort_flag = e->pk_abort;
  P.err = e->err;
  P.x = e->x;
  P.embd = (const uint8_t*)e->embd->d;
  P.embd_type = e->embd->type;
  P.embd_row_bytes = (long long)(e->embd->bytes / e->embd->rows());
  P.hidden = e->cfg.hidden_size;
  P.hidden_pad = e->pk_hidden_pad;
  P.max_inner_pad = e->pk_inner_pad;
  P.slot_bytes = e->pk_slot;
  P.trace = e->trace;
  INF_CUDA_TRY(cudaMemsetAsync(e->pk_barrier, 0, sizeof(unsigned), e->st));
  INF_CUDA_TRY(cudaMemsetAsync(e->pk_abort, 0, sizeof(int), e->st));
  INF_CUDA_TRY(cudaMemsetAsync(&e->ctl->argkey, 0, sizeof(unsigned long long), e->st));
  return pk_launch(P, e->pk_smem, e->st);
}

}  // namespace
}  // namespace inf

extern "C" {

static int ready(InfernoEngine* e) {
  if (!e) return set_error(INFERNO_EINVAL, "null engine");
  if (!e->finalized) return set_error(INFERNO_ESTATE, "engine not finalized");
  INF_CUDA_TRY(cudaSetDevice(e->dev));
  return 0;
}

static int set_ctl(InfernoEngine* e, int tok, int pos, int n_prompt) {
  Ctl h{};
  h.tok = tok;
  h.pos = pos;
  h.step = 0;
  h.n_prompt = n_prompt;
  h.argkey = 0;
  INF_CUDA_TRY(cudaMemcpyAsync(e->ctl, &h, sizeof h, cudaMemcpyHostToDevice, e->st));
  return 0;
}

int inferno_layer_forward(InfernoEngine* e, int layer, float* x_host, int pos) {
  int rc;
  if ((rc = ready(e))) return rc;
  if (layer < 0 || layer >= e->cfg.num_layers || !x_host) return set_error(INFERNO_EINVAL, "layer_forward: bad layer");
  if (pos < 0 || pos >= e->cfg.max_ctx) return set_error(INFERNO_EINVAL, "layer_forward: pos %d outside [0, %d)", pos, e->cfg.max_ctx);
  const int H = e->cfg.hidden_size;
  if (e->cfg.tp_size > 1)
    return set_error(INFERNO_ESTATE, "layer_forward is not available under tensor parallelism (use forward_tokens)");
  e->xcur = e->x;
  if ((rc = set_ctl(e, 0, pos, 1))) return rc;
  INF_CUDA_TRY(cudaMemcpyAsync(e->x, x_host, (size_t)H * 4, cudaMemcpyHostToDevice, e->st));
  if ((rc = enqueue_layer(e, layer, false))) return rc;
  INF_CUDA_TRY(cudaMemcpyAsync(x_host, e->x, (size_t)H * 4, cudaMemcpyDeviceToHost, e->st));
  INF_CUDA_TRY(cudaStreamSynchronize(e->st));
  return check_device_error(e);
}

int inferno_forward_tokens(InfernoEngine* e, const int32_t* tok, int n, int pos0, float* logits_out,
                           int32_t* argmax_out) {
  int rc;
  if ((rc = ready(e))) return rc;
  if (!tok || n <= 0) return set_error(INFERNO_EINVAL, "forward_tokens: no tokens");
  if (pos0 < 0 || pos0 + n > e->cfg.max_ctx)
    return set_error(INFERNO_EINVAL, "forward_tokens: positions [%d, %d) exceed max_ctx %d", pos0, pos0 + n, e->cfg.max_ctx);
  for (int i = 0; i < n; ++i)
    if (tok[i] < 0 || tok[i] >= e->cfg.vocab_size) return set_error(INFERNO_EINVAL, "forward_tokens: token %d out of range", tok[i]);
  INF_CUDA_TRY(cudaMemcpyAsync(e->prompt, tok, (size_t)n * 4, cudaMemcpyHostToDevice, e->st));
  if ((rc = set_ctl(e, tok[0], pos0, n))) return rc;
  if (e->prefill && !e->persistent && n > 1 && e->tp) {
    // tensor parallel: the first n - 1 tokens as chunks (residual sums by
    // all-reduce), the last one through the token path, whose vocab-split
    // lm_head and first-max reduction across ranks it already has
    for (int off = 0; off < n - 1; off += PF_MAX_T) {
      const int T = std::min(PF_MAX_T, n - 1 - off);
      if ((rc = enqueue_prefill_chunk(e, e->prompt + off, T, pos0 + off, false, false))) return rc;
    }
    if ((rc = set_ctl(e, tok[n - 1], pos0 + n - 1, 1))) return rc;
    if ((rc = run_steps(e, 1, logits_out != nullptr))) return rc;
  } else if (e->prefill && !e->persistent && n > 1) {
    // chunked prefill; afterwards the control block reads as if n decode
    // steps had run (position, step, last token = first-max of the last logits)
    auto enqueue_all = [&]() -> int {
      for (int off = 0; off < n; off += PF_MAX_T) {
        const int T = std::min(PF_MAX_T, n - off);
        const int r = enqueue_prefill_chunk(e, e->prompt + off, T, pos0 + off, off + T == n, logits_out != nullptr);
        if (r) return r;
      }
      return 0;
    };
    const long long key = ((long long)n << 32) | ((long long)pos0 << 1) | (logits_out ? 1 : 0);
    auto it = e->pf_graphs.find(key);
    if (it == e->pf_graphs.end() && e->cfg.use_graphs && e->pf_seen[key]++ > 0 && e->pf_graphs.size() < 16) {
      cudaGraph_t g = nullptr;
      cudaGraphExec_t ge = nullptr;
      INF_CUDA_TRY(cudaStreamBeginCapture(e->st, cudaStreamCaptureModeThreadLocal));
      rc = enqueue_all();
      cudaError_t r1 = cudaStreamEndCapture(e->st, &g);
      if (rc) {
        if (g) cudaGraphDestroy(g);
        return rc;
      }
      if (r1 != cudaSuccess) return set_error(INFERNO_ECUDA, "prefill capture: %s", cudaGetErrorString(r1));
      r1 = cudaGraphInstantiate(&ge, g, 0);
      cudaGraphDestroy(g);
      if (r1 != cudaSuccess) return set_error(INFERNO_ECUDA, "prefill graph: %s", cudaGetErrorString(r1));
      it = e->pf_graphs.emplace(key, ge).first;
    }
    if (it != e->pf_graphs.end()) {
      INF_CUDA_TRY(cudaGraphLaunch(it->second, e->st));
    } else if ((rc = enqueue_all())) {
      return rc;
    }
    Ctl h{};
    INF_CUDA_TRY(cudaMemcpyAsync(&h, e->ctl, sizeof h, cudaMemcpyDeviceToHost, e->st));
    INF_CUDA_TRY(cudaStreamSynchronize(e->st));
    const int am = (int)(0xffffffffu - (uint32_t)(h.argkey & 0xffffffffull));
    h.tok = am;
    h.last = am;
    h.pos = pos0 + n;
    h.step = n;
    h.n_prompt = n;
    h.argkey = 0ull;
    INF_CUDA_TRY(cudaMemcpyAsync(e->ctl, &h, sizeof h, cudaMemcpyHostToDevice, e->st));
  } else if (e->persistent) {
    if ((rc = run_persistent(e, tok[0], pos0, n, n))) return rc;
  } else if ((rc = run_steps(e, n, logits_out != nullptr))) {
    return rc;
  }
  Ctl h{};
  INF_CUDA_TRY(cudaMemcpyAsync(&h, e->ctl, sizeof h, cudaMemcpyDeviceToHost, e->st));
  if (logits_out)
    INF_CUDA_TRY(cudaMemcpyAsync(logits_out, e->logits, (size_t)e->cfg.vocab_size * 4, cudaMemcpyDeviceToHost, e->st));
  INF_CUDA_TRY(cudaStreamSynchronize(e->st));
  if ((rc = check_device_error(e))) return rc;
  if (argmax_out) *argmax_out = h.last;
  return 0;
}

// Every position's logits / first-max argmax over n tokens (the full_logits
// forward of mtp_verify_step!, src/ModelCPU.jl:1914-1930): the tokens run one
// at a time through the single-token graph with logits, so each position's
// result is exactly that of the decode path; the state advances over all n.
int inferno_forward_tokens_all(InfernoEngine* e, const int32_t* tok, int n, int pos0, float* logits_out,
                               int32_t* argmax_out) {
  int rc;
  if ((rc = ready(e))) return rc;
  if (!tok || n <= 0 || !argmax_out) return set_error(INFERNO_EINVAL, "forward_tokens_all: no tokens or output");
  const size_t V = (size_t)e->cfg.vocab_size;
  for (int i = 0; i < n; ++i)
    if ((rc = inferno_forward_tokens(e, tok + i, 1, pos0 + i, logits_out ? logits_out + (size_t)i * V : nullptr,
                                     argmax_out + i)))
      return rc;
  return 0;
}

int inferno_decode_greedy(InfernoEngine* e, int32_t tok, int pos, int n_steps, int32_t* out_tokens) {
  int rc;
  if ((rc = ready(e))) return rc;
  if (n_steps <= 0 || !out_tokens) return set_error(INFERNO_EINVAL, "decode_greedy: bad n_steps/out");
  if (pos < 0 || pos + n_steps > e->cfg.max_ctx)
    return set_error(INFERNO_EINVAL, "decode_greedy: positions [%d, %d) exceed max_ctx %d", pos, pos + n_steps,
                     e->cfg.max_ctx);
  if (tok < 0 || tok >= e->cfg.vocab_size) return set_error(INFERNO_EINVAL, "decode_greedy: token out of range");
  if (n_steps > e->max_out) return set_error(INFERNO_EINVAL, "decode_greedy: n_steps too large");
  if ((rc = set_ctl(e, tok, pos, 1))) return rc;
  INF_CUDA_TRY(cudaEventRecord(e->ev0, e->st));
  if (e->persistent) {
    if ((rc = run_persistent(e, tok, pos, 1, n_steps))) return rc;
  } else if ((rc = run_steps(e, n_steps, false))) {
    return rc;
  }
  INF_CUDA_TRY(cudaEventRecord(e->ev1, e->st));
  INF_CUDA_TRY(cudaMemcpyAsync(out_tokens, e->out_tokens, (size_t)n_steps * 4, cudaMemcpyDeviceToHost, e->st));
  INF_CUDA_TRY(cudaStreamSynchronize(e->st));
  cudaEventElapsedTime(&e->last_ms, e->ev0, e->ev1);
  return check_device_error(e);
}

float inferno_last_decode_ms(InfernoEngine* e) { return e ? e->last_ms : -1.f; }

int inferno_decode_sample(InfernoEngine* e, int32_t tok, int pos, int n_steps, const InfernoSampling* s,
                          const int32_t* seen_tokens, int n_seen, int32_t* out_tokens) {
  int rc;
  if ((rc = ready(e))) return rc;
  const InfernoConfig& c = e->cfg;
  if (!s || n_steps <= 0 || !out_tokens || n_seen < 0 || (n_seen && !seen_tokens))
    return set_error(INFERNO_EINVAL, "decode_sample: bad arguments");
  if (s->temperature < 0.f || s->top_p <= 0.f || s->top_p > 1.f || s->min_p < 0.f || s->min_p >= 1.f ||
      s->repetition_penalty <= 0.f)
    return set_error(INFERNO_EINVAL, "decode_sample: sampling parameter out of range");
  if (pos < 0 || pos + n_steps > c.max_ctx)
    return set_error(INFERNO_EINVAL, "decode_sample: positions [%d, %d) exceed max_ctx %d", pos, pos + n_steps, c.max_ctx);
  if (tok < 0 || tok >= c.vocab_size || n_steps > e->max_out) return set_error(INFERNO_EINVAL, "decode_sample: bad token / n_steps");
  if (e->persistent) return set_error(INFERNO_ESTATE, "decode_sample: not available with the persistent kernel");
  if (!e->seen && (rc = dalloc(e, &e->seen, c.vocab_size))) return rc;
  std::vector<uint8_t> mark(c.vocab_size, 0);
  for (int i = 0; i < n_seen; ++i)
    if (seen_tokens[i] >= 0 && seen_tokens[i] < c.vocab_size) mark[seen_tokens[i]] = 1;
  INF_CUDA_TRY(cudaMemcpyAsync(e->seen, mark.data(), mark.size(), cudaMemcpyHostToDevice, e->st));
  SampleArgs a{s->temperature, s->top_p, s->min_p, s->presence_penalty, s->repetition_penalty, s->top_k, s->seed};
  if ((rc = set_ctl(e, tok, pos, 1))) return rc;
  // one graph per call: the parameters are kernel arguments of the sampler
  e->sampling = &a;
  cudaGraphExec_t g = nullptr;
  rc = capture(e, 1, true, &g);
  e->sampling = nullptr;
  if (rc) return rc;
  INF_CUDA_TRY(cudaEventRecord(e->ev0, e->st));
  for (int t = 0; t < n_steps && !rc; ++t)
    if (cudaGraphLaunch(g, e->st) != cudaSuccess) rc = set_error(INFERNO_ECUDA, "decode_sample: graph launch failed");
  INF_CUDA_TRY(cudaEventRecord(e->ev1, e->st));
  INF_CUDA_TRY(cudaStreamSynchronize(e->st));
  cudaGraphExecDestroy(g);
  if (rc) return rc;
  cudaEventElapsedTime(&e->last_ms, e->ev0, e->ev1);
  INF_CUDA_TRY(cudaMemcpy(out_tokens, e->out_tokens, (size_t)n_steps * 4, cudaMemcpyDeviceToHost));
  return check_device_error(e);
}

int inferno_reset_states(InfernoEngine* e) {
  int rc;
  if ((rc = ready(e))) return rc;
  for (auto& b : e->state_bufs) INF_CUDA_TRY(cudaMemsetAsync(b.first, 0, b.second, e->st));
  INF_CUDA_TRY(cudaStreamSynchronize(e->st));
  return 0;
}

int inferno_dump_hidden(InfernoEngine* e, int layer, float* out) {
  int rc;
  if ((rc = ready(e))) return rc;
  if (!e->dump) return set_error(INFERNO_ESTATE, "dump_hidden needs INFERNO_B200_DUMP=1 at engine creation");
  if (layer < 0 || layer >= e->cfg.num_layers || !out) return set_error(INFERNO_EINVAL, "dump_hidden: bad layer");
  INF_CUDA_TRY(cudaMemcpy(out, e->hidden + (size_t)layer * e->cfg.hidden_size, (size_t)e->cfg.hidden_size * 4,
                          cudaMemcpyDeviceToHost));
  return 0;
}

int64_t inferno_state_size(InfernoEngine* e) {
  if (ready(e)) return INFERNO_ESTATE;
  int64_t s = 0;
  for (auto& b : e->state_bufs) s += (int64_t)b.second;
  return s;
}

int inferno_state_export(InfernoEngine* e, void* host, int64_t nbytes) {
  int rc;
  if ((rc = ready(e))) return rc;
  if (nbytes < inferno_state_size(e) || !host) return set_error(INFERNO_EINVAL, "state_export: buffer too small");
  char* p = (char*)host;
  for (auto& b : e->state_bufs) {
    INF_CUDA_TRY(cudaMemcpyAsync(p, b.first, b.second, cudaMemcpyDeviceToHost, e->st));
    p += b.second;
  }
  INF_CUDA_TRY(cudaStreamSynchronize(e->st));
  return 0;
}

int inferno_state_import(InfernoEngine* e, const void* host, int64_t nbytes) {
  int rc;
  if ((rc = ready(e))) return rc;
  if (nbytes != inferno_state_size(e) || !host) return set_error(INFERNO_EINVAL, "state_import: size mismatch");
  const char* p = (const char*)host;
  for (auto& b : e->state_bufs) {
    INF_CUDA_TRY(cudaMemcpyAsync(b.first, p, b.second, cudaMemcpyHostToDevice, e->st));
    p += b.second;
  }
  INF_CUDA_TRY(cudaStreamSynchronize(e->st));
  return 0;
}

int inferno_state_save_device(InfernoEngine* e) {
  int rc;
  if ((rc = ready(e))) return rc;
  size_t tot = 0;
  for (auto& b : e->state_bufs) tot += b.second;
  if (!e->snapshot) {
    if (cudaMalloc(&e->snapshot, tot) != cudaSuccess) return set_error(INFERNO_ENOMEM, "snapshot alloc (%zu B)", tot);
    e->state_bytes = tot;
  }
  char* p = (char*)e->snapshot;
  for (auto& b : e->state_bufs) {
    INF_CUDA_TRY(cudaMemcpyAsync(p, b.first, b.second, cudaMemcpyDeviceToDevice, e->st));
    p += b.second;
  }
  return 0;
}

int inferno_state_restore_device(InfernoEngine* e) {
  int rc;
  if ((rc = ready(e))) return rc;
  if (!e->snapshot) return set_error(INFERNO_ESTATE, "no device snapshot saved");
  const char* p = (const char*)e->snapshot;
  for (auto& b : e->state_bufs) {
    INF_CUDA_TRY(cudaMemcpyAsync(b.first, p, b.second, cudaMemcpyDeviceToDevice, e->st));
    p += b.second;
  }
  return 0;
}

int inferno_comm_mode(InfernoEngine* e) {
  int rc;
  if ((rc = ready(e))) return rc;
  if (e->cfg.tp_size <= 1) return 0;
  return e->xch ? 1 : 2;
}

int inferno_kernels_per_token(InfernoEngine* e) {
  int rc;
  if ((rc = ready(e))) return rc;
  return e->persistent ? 0 : e->token_launches;
}

int inferno_profile_tokens(InfernoEngine* e, int32_t tok, int pos, int n_tokens, float* ms_by_class,
                           int32_t* launches_by_class) {
  int rc;
  if ((rc = ready(e))) return rc;
  if (n_tokens <= 0 || pos < 0 || pos + n_tokens > e->cfg.max_ctx || !ms_by_class || !launches_by_class)
    return set_error(INFERNO_EINVAL, "profile_tokens: bad arguments");
  for (int k = 0; k < K_NCLASS; ++k) { ms_by_class[k] = 0.f; launches_by_class[k] = 0; }
  if ((rc = set_ctl(e, tok, pos, 1))) return rc;
  for (int t = 0; t < n_tokens; ++t) {
    e->profiling = true;
    rc = enqueue_token(e, false, false);
    e->profiling = false;
    if (!rc) {
      cudaError_t r = cudaStreamSynchronize(e->st);
      if (r != cudaSuccess) rc = set_error(INFERNO_ECUDA, "profile sync: %s", cudaGetErrorString(r));
    }
    for (size_t i = 1; i < e->prof_ev.size() && !rc; ++i) {
      float ms = 0.f;
      cudaEventElapsedTime(&ms, e->prof_ev[i - 1], e->prof_ev[i]);
      int k = e->prof_kind[i];
      if (k >= 0 && k < K_NCLASS) { ms_by_class[k] += ms; launches_by_class[k] += 1; }
    }
    for (auto ev : e->prof_ev) cudaEventDestroy(ev);
    e->prof_ev.clear();
    e->prof_kind.clear();
    if (rc) return rc;
  }
  return check_device_error(e);
}

int inferno_debug_trace(InfernoEngine* e, unsigned long long* out, int n) {
  int rc;
  if ((rc = ready(e))) return rc;
  if (!e->trace) return set_error(INFERNO_ESTATE, "engine created without INFERNO_B200_TRACE");
  if (!out) {   // clear: the stamps of the next token start from zero
    INF_CUDA_TRY(cudaDeviceSynchronize());
    INF_CUDA_TRY(cudaMemset(e->trace, 0, 8 * 8192));
    return 0;
  }
  if (n > 8192) n = 8192;
  INF_CUDA_TRY(cudaMemcpy(out, e->trace, (size_t)n * 8, cudaMemcpyDeviceToHost));
  return 0;
}

int inferno_tp_unique_id(void* out, int nbytes) {
  if (!out || nbytes < (int)sizeof(ncclUniqueId))
    return set_error(INFERNO_EINVAL, "tp_unique_id: buffer must hold %d bytes", (int)sizeof(ncclUniqueId));
  ncclUniqueId id;
  ncclResult_t r = ncclGetUniqueId(&id);
  if (r != ncclSuccess) return set_error(INFERNO_ENCCL, "ncclGetUniqueId: %s", ncclGetErrorString(r));
  memcpy(out, &id, sizeof id);
  return 0;
}

int inferno_engine_destroy(InfernoEngine* e) {
  if (!e) return 0;
  cudaSetDevice(e->dev);
  cudaStreamSynchronize(e->st);
  if (e->g1) cudaGraphExecDestroy(e->g1);
  if (e->g1_logits) cudaGraphExecDestroy(e->g1_logits);
  if (e->g8) cudaGraphExecDestroy(e->g8);
  for (auto& kv : e->pf_graphs) cudaGraphExecDestroy(kv.second);
  if (e->snapshot) cudaFree(e->snapshot);
  if (e->trace) cudaFree(e->trace);
  for (auto& kv : e->tensors) cudaFree(kv.second.d);
  for (void* p : e->allocs) cudaFree(p);
  if (e->ev0) cudaEventDestroy(e->ev0);
  if (e->ev1) cudaEventDestroy(e->ev1);
  for (int q = 0; q < 8; ++q)
    if (e->xch && q != e->cfg.tp_rank && e->xch_peer[q]) cudaIpcCloseMemHandle(e->xch_peer[q]);
  if (e->comm) ncclCommDestroy(e->comm);
  cudaStreamDestroy(e->st);
  delete e;
  return 0;
}

}  // extern "C"
