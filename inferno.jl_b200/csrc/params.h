// Parameter blocks of the decode-step kernels (shared by the kernels and the
// engine that launches them).
#pragma once
#include <cuda_runtime.h>

namespace inf {

struct GdnParams {
  const float* x;          // residual stream (pre-norm) [H]
  const float* in_norm;    // [H]
  float eps;
  int H, nv, nk, dv, K, C;
  const float* qkv;        // in_proj output [C]
  const float* conv_w;     // [C][K] (GGUF ssm_conv1d data, w[c,k] at k + K*c)
  float* ring;             // [K][C]
  const float* w_alpha;    // [nv][H]
  const float* w_beta;     // [nv][H]
  const float* ssm_a;      // [nv]
  const float* dt_bias;    // [nv]
  float* S;                // [nv][dv][dk]
  float* y;                // [nv*dv] pre-norm output
  int* step;               // per-layer step counter
  int* done;               // per-layer CTA completion counter
  // 1: the last CTA advances *step (via `done`); 0: the caller advances it
  // after the kernel (the decode token's finalize kernel does it for every layer)
  int self_advance = 1;
  // whole-head kernel (gdn_head_kernel): the per-head output RMSNorm and
  // SiLU(z) gate are applied in the step, y then holds the gated output
  const float* z = nullptr;        // [nv*dv] attn_gate GEMV output
  const float* out_norm = nullptr; // [dv] ssm_norm weight
  // batched decode (gdn_head_kernel, blockIdx.y = sequence b): sequence b's
  // x / qkv / z / y rows, state, conv ring and step counter sit these many
  // elements after sequence 0's
  long long xs = 0, qkvs = 0, zys = 0, Ss = 0, rings = 0;
  int steps_stride = 0;
  unsigned long long* trace = nullptr;   // debug timeline slots (KT_*, common.cuh)
};

struct AttnParams {
  const float* qg;       // [nh][2*hd]: per head q then gate (src/ModelCPU.jl:766-772)
  const float* k;        // [nkv*hd] new key (pre-norm)
  const float* v;        // [nkv*hd]
  const float* q_norm;   // [hd]
  const float* k_norm;   // [hd]
  float eps;
  const float* rope_cos; // [ctx][rd/2]
  const float* rope_sin;
  int rd;
  float* kc;             // [ctx][nkv][hd]
  float* vc;
  int nh, nkv, ctx, split_len, nsplit;
  const int* pos;        // device scalar
  float* part_o;         // [nh][nsplit][hd]
  float* part_ml;        // [nh][nsplit][2]
  int* counters;         // [nkv]
  float* out;            // [nh*hd] gated attention output
  int* err;
  // batched decode (blockIdx.z = sequence b): b's qg / k / v / out rows and
  // KV cache lie these many floats after sequence 0's; pos[b] is its position;
  // part_o / part_ml / counters hold one block per sequence
  long long qgs = 0, kvs = 0, outs = 0, caches = 0;
  unsigned long long* trace = nullptr;   // debug timeline slots (KT_*, common.cuh)
};

int launch_gdn_step(const GdnParams& p, cudaStream_t st, bool pdl);
// one CTA per head, output norm + gate fused (y = gated output); the caller
// advances the step counter
int launch_gdn_head(const GdnParams& p, cudaStream_t st, bool pdl, int nseq = 1);
int launch_attn_decode(const AttnParams& p, cudaStream_t st, bool pdl, int nseq = 1);

}  // namespace inf
