// Stage program and parameters of the persistent decode kernel (decode.cu).
#pragma once
#include "gemv.cuh"
#include "params.h"

namespace inf {

enum PkKind : int { PK_GEMV = 0, PK_GDN = 1, PK_ATTN = 2 };

struct alignas(16) PkStage {
  int kind;
  int type;          // GEMV: ggml type
  int R;             // GEMV: rows per warp (2 or 4)
  int embed_row;     // GEMV: input is this token's embedding row (first stage)
  int slot_bytes;
  const float* xsrc; // GEMV input vector (global)
  GemvParams g;
  GdnParams d;
  AttnParams a;
};

struct PkParams {
  const PkStage* stages;
  int n_stages;
  int n_steps;       // tokens to run
  int tok0, pos0, n_prompt;
  const int* prompt; // device prompt ids (n_prompt)
  int* out_tokens;   // argmax of step t written at t - (n_prompt - 1)
  int max_out;
  int* ctl_last;     // argmax of the last step
  unsigned long long* argkey;
  unsigned* barrier; // grid barrier counter (zeroed before launch)
  int* abort_flag;
  int* err;
  float* x;          // residual stream
  const uint8_t* embd;
  int embd_type;
  long long embd_row_bytes;
  int hidden, hidden_pad, max_inner_pad;
  int slot_bytes;
  unsigned long long* trace;   // debug: per-stage stamps of CTA 0 for token 1 (null = off)
};

int pk_plan_gemv(const GemvCall& c, int slot_cap, int sms, PkStage* S);
size_t pk_smem_bytes(int hidden_pad, int max_inner_pad, int slot_bytes);
int pk_launch(const PkParams& P, size_t smem, cudaStream_t st);

}  // namespace inf
