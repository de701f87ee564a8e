// ORACLE -- test infrastructure, not product code.
//
// A plain C++17 restatement of Inferno.jl's CPU decode path, used only by the
// tests, by __graft_entry__.smoke() and by bench.py's CPU-baseline leg as the
// checker for the CUDA engine.  It is never linked into libinferno_b200.so.
//
// Every function cites the reference line it follows (paths are relative to
// the Inferno.jl source tree).  Compile with -ffp-contract=off: Julia does not
// fuse a*b-c, and the dequantizers below must reproduce src/Dequant.jl's fp32
// rounding sequence bit for bit.
//
// What is restated:
//   * dequantization of Q4_K / Q5_K / Q6_K / Q8_0 / IQ2_XXS (src/Dequant.jl)
//   * fp32 GEMV on dequantized weights (src/ModelCPU.jl:435-444, BLAS sgemv)
//   * RMSNorm, RoPE, KV cache, MLP, Gated DeltaNet, gated full attention with
//     FlashAttention.jl's online softmax, decoder layer, forward, lm_head and
//     greedy argmax (src/ModelCPU.jl, src/FlashAttention.jl)
//   * MoE routing (src/Model.jl:497-526), restated for the config-5 shape
//   * the isolated delta-rule recurrence used by the config-3 GDN checks.
#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <map>
#include <memory>
#include <numeric>
#include <string>
#include <vector>
#ifdef _OPENMP
#include <omp.h>
#endif

namespace {

enum { T_F32 = 0, T_F16 = 1, T_Q8_0 = 8, T_Q4_K = 12, T_Q5_K = 13, T_Q6_K = 14, T_IQ2_XXS = 16 };

const uint64_t kIq2xxsGrid[256] = {
#include "../inferno.jl_b200/csrc/iq2xxs_grid.inc"
};

// exact IEEE half -> float (Julia Float32(reinterpret(Float16, ...)))
float h2f(uint16_t h) {
  uint32_t s = (uint32_t)(h >> 15) << 31, e = (h >> 10) & 31, m = h & 1023, bits;
  if (e == 0) {
    if (m == 0) bits = s;
    else {  // subnormal: renormalise
      int sh = 0;
      while (!(m & 1024)) { m <<= 1; ++sh; }
      m &= 1023;
      bits = s | (uint32_t)(127 - 15 - sh + 1) << 23 | m << 13;
    }
  } else if (e == 31) bits = s | 0x7f800000u | m << 13;
  else bits = s | (e + 112) << 23 | m << 13;
  float f;
  memcpy(&f, &bits, 4);
  return f;
}
inline uint16_t rd16(const uint8_t* p) { return (uint16_t)(p[0] | p[1] << 8); }
inline uint32_t rd32(const uint8_t* p) { return (uint32_t)p[0] | p[1] << 8 | p[2] << 16 | (uint32_t)p[3] << 24; }

// KSIGNS_IQ2XS (src/QuantsData.jl:7-16): i with bit 7 = parity(i)
inline uint8_t ksigns(uint32_t i) { return (uint8_t)(i | (__builtin_popcount(i) & 1) << 7); }

// src/Dequant.jl:12-54 (note the "- 8" on every grid byte, pinned by
// tests/unit/core_components.jl:114-122)
void dq_iq2_xxs(const uint8_t* data, int64_t n, float* y) {
  for (int64_t i = 0; i < n / 256; ++i) {
    const uint8_t* b = data + i * 66;
    float d = h2f(rd16(b));
    for (int ib = 0; ib < 8; ++ib) {
      uint32_t a1 = rd32(b + 2 + ib * 8), a2 = rd32(b + 2 + ib * 8 + 4);
      float db = d * (0.5f + (float)(a2 >> 28)) * 0.25f;
      for (int l = 0; l < 4; ++l) {
        uint64_t g = kIq2xxsGrid[(a1 >> (8 * l)) & 0xff];
        uint8_t s = ksigns((a2 >> (7 * l)) & 127);
        for (int j = 0; j < 8; ++j) {
          int v = (int)(int8_t)((g >> (8 * j)) & 0xff) - 8;
          float sg = (s & (1u << j)) ? -1.0f : 1.0f;
          y[i * 256 + ib * 32 + l * 8 + j] = db * (float)v * sg;
        }
      }
    }
  }
}

// src/Dequant.jl:304-321
void dq_q8_0(const uint8_t* data, int64_t n, float* y) {
  for (int64_t i = 0; i < n / 32; ++i) {
    const uint8_t* b = data + i * 34;
    float d = h2f(rd16(b));
    for (int j = 0; j < 32; ++j) y[i * 32 + j] = d * (float)(int8_t)b[2 + j];
  }
}

// 6-bit scale/min unpack shared by Q4_K and Q5_K (src/Dequant.jl:345-362, 412-425)
inline void kscale(const uint8_t* sc, int is, uint8_t& s, uint8_t& m) {
  if (is < 4) {
    s = sc[is] & 63;
    m = sc[is + 4] & 63;
  } else {
    s = (sc[is + 4] & 0x0f) | ((sc[is - 4] >> 6) << 4);
    m = (sc[is + 4] >> 4) | ((sc[is] >> 6) << 4);
  }
}

// src/Dequant.jl:325-375: w = d1*q - min1 with separate fp32 roundings
void dq_q4_k(const uint8_t* data, int64_t n, float* y) {
  for (int64_t i = 0; i < n / 256; ++i) {
    const uint8_t* b = data + i * 144;
    float d = h2f(rd16(b)), dmin = h2f(rd16(b + 2));
    const uint8_t* sc = b + 4;
    const uint8_t* qs = b + 16;
    for (int j = 0; j < 4; ++j) {
      uint8_t s1, m1, s2, m2;
      kscale(sc, 2 * j, s1, m1);
      kscale(sc, 2 * j + 1, s2, m2);
      float d1 = d * (float)s1, mn1 = dmin * (float)m1;
      float d2 = d * (float)s2, mn2 = dmin * (float)m2;
      for (int l = 0; l < 32; ++l) {
        uint8_t q = qs[j * 32 + l];
        y[i * 256 + j * 64 + l] = d1 * (float)(q & 0x0f) - mn1;
        y[i * 256 + j * 64 + 32 + l] = d2 * (float)(q >> 4) - mn2;
      }
    }
  }
}

// src/Dequant.jl:379-441
void dq_q5_k(const uint8_t* data, int64_t n, float* y) {
  for (int64_t i = 0; i < n / 256; ++i) {
    const uint8_t* b = data + i * 176;
    float d = h2f(rd16(b)), dmin = h2f(rd16(b + 2));
    const uint8_t* sc = b + 4;
    const uint8_t* qh = b + 16;
    const uint8_t* qs = b + 48;
    for (int j = 0; j < 4; ++j) {
      uint8_t s1, m1, s2, m2;
      kscale(sc, 2 * j, s1, m1);
      kscale(sc, 2 * j + 1, s2, m2);
      float d1 = d * (float)s1, mn1 = dmin * (float)m1;
      float d2 = d * (float)s2, mn2 = dmin * (float)m2;
      uint8_t u1 = (uint8_t)(1u << (2 * j)), u2 = (uint8_t)(1u << (2 * j + 1));
      for (int l = 0; l < 32; ++l) {
        uint8_t q = qs[j * 32 + l], h = qh[l];
        y[i * 256 + j * 64 + l] = d1 * (float)((q & 0x0f) + ((h & u1) ? 16 : 0)) - mn1;
        y[i * 256 + j * 64 + 32 + l] = d2 * (float)((q >> 4) + ((h & u2) ? 16 : 0)) - mn2;
      }
    }
  }
}

// src/Dequant.jl:558-601: w = (d*sc)*q, two roundings
void dq_q6_k(const uint8_t* data, int64_t n, float* y) {
  for (int64_t i = 0; i < n / 256; ++i) {
    const uint8_t* b = data + i * 210;
    const uint8_t* ql = b;
    const uint8_t* qh = b + 128;
    const int8_t* sc = (const int8_t*)(b + 192);
    float d = h2f(rd16(b + 208));
    for (int ns = 0; ns < 2; ++ns) {
      const uint8_t* L = ql + ns * 64;
      const uint8_t* Hh = qh + ns * 32;
      const int8_t* S = sc + ns * 8;
      float* o = y + i * 256 + ns * 128;
      for (int l = 0; l < 32; ++l) {
        int is = l / 16;
        uint8_t h = Hh[l];
        int q1 = (int)((L[l] & 0x0f) | ((h & 3) << 4)) - 32;
        int q2 = (int)((L[l + 32] & 0x0f) | (((h >> 2) & 3) << 4)) - 32;
        int q3 = (int)((L[l] >> 4) | (((h >> 4) & 3) << 4)) - 32;
        int q4 = (int)((L[l + 32] >> 4) | (((h >> 6) & 3) << 4)) - 32;
        o[l] = d * (float)S[is] * (float)q1;
        o[l + 32] = d * (float)S[is + 2] * (float)q2;
        o[l + 64] = d * (float)S[is + 4] * (float)q3;
        o[l + 96] = d * (float)S[is + 6] * (float)q4;
      }
    }
  }
}

int block_elems(int t) { return (t == T_Q8_0) ? 32 : (t == T_F32 || t == T_F16) ? 1 : 256; }
int block_bytes(int t) {
  switch (t) {
    case T_F32: return 4;
    case T_F16: return 2;
    case T_Q8_0: return 34;
    case T_Q4_K: return 144;
    case T_Q5_K: return 176;
    case T_Q6_K: return 210;
    case T_IQ2_XXS: return 66;
  }
  return -1;
}

int dequant(int t, const uint8_t* src, int64_t n, float* dst) {
  if (n % block_elems(t)) return -1;
  switch (t) {
    case T_F32: memcpy(dst, src, n * 4); return 0;
    case T_F16: for (int64_t i = 0; i < n; ++i) dst[i] = h2f(rd16(src + 2 * i)); return 0;
    case T_Q8_0: dq_q8_0(src, n, dst); return 0;
    case T_Q4_K: dq_q4_k(src, n, dst); return 0;
    case T_Q5_K: dq_q5_k(src, n, dst); return 0;
    case T_Q6_K: dq_q6_k(src, n, dst); return 0;
    case T_IQ2_XXS: dq_iq2_xxs(src, n, dst); return 0;
  }
  return -2;
}

// fp32 dot with 8 partial sums (the order of an 8-wide SIMD sgemv)
inline float dot(const float* a, const float* b, int n) {
  float s[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  int i = 0;
  for (; i + 8 <= n; i += 8)
    for (int k = 0; k < 8; ++k) s[k] += a[i + k] * b[i + k];
  float r = ((s[0] + s[4]) + (s[1] + s[5])) + ((s[2] + s[6]) + (s[3] + s[7]));
  for (; i < n; ++i) r += a[i] * b[i];
  return r;
}

// A weight matrix: (outer x inner), row-major GGUF blocks.  Either fully
// dequantized at load (what load_model_cpu does by default,
// src/LoaderCPU.jl:334-341) or dequantized row by row on use (for shapes whose
// fp32 copy would not fit in host memory) -- the values are identical.
struct Mat {
  int type = -1;
  int64_t inner = 0, outer = 0;
  std::vector<uint8_t> raw;
  std::vector<float> f32;
  bool empty() const { return type < 0; }
  int64_t rowb() const { return inner / block_elems(type) * block_bytes(type); }
  void load(int t, int64_t in, int64_t out, const uint8_t* d, bool deq) {
    type = t; inner = in; outer = out;
    int64_t nb = rowb() * out;
    if (deq) {
      f32.resize((size_t)(in * out));
      dequant(t, d, in * out, f32.data());
    } else raw.assign(d, d + nb);
  }
  void row(int64_t r, float* buf) const {
    if (!f32.empty()) memcpy(buf, f32.data() + r * inner, inner * 4);
    else dequant(type, raw.data() + r * rowb(), inner, buf);
  }
  // y[r] = W[r,:] . x ; ModelCPU.mul! -> LinearAlgebra.mul! (src/ModelCPU.jl:435-444)
  void gemv(const float* x, float* y) const { gemv_rows(x, y, 0, outer); }
  void gemv_rows(const float* x, float* y, int64_t r0, int64_t r1) const {
    if (!f32.empty()) {
#pragma omp parallel for schedule(static) if (r1 - r0 > 64)
      for (int64_t r = r0; r < r1; ++r) y[r - r0] = dot(f32.data() + r * inner, x, (int)inner);
    } else {
#pragma omp parallel
      {
        std::vector<float> buf(inner);
#pragma omp for schedule(static)
        for (int64_t r = r0; r < r1; ++r) {
          row(r, buf.data());
          y[r - r0] = dot(buf.data(), x, (int)inner);
        }
      }
    }
  }
};

// src/ModelCPU.jl:110-122
void rmsnorm(float* out, const float* x, const float* w, int n, float eps) {
  float ss = 0.0f;
  for (int i = 0; i < n; ++i) ss += x[i] * x[i];
  float scale = 1.0f / std::sqrt(ss / (float)n + eps);
  for (int i = 0; i < n; ++i) out[i] = x[i] * scale * w[i];
}

inline float silu(float g) { return g / (1.0f + std::exp(-g)); }

// src/FlashAttention.jl:16-74 (BLOCK_N = 64 online softmax).  cache layout
// (head_dim, n_kv, seq) column-major: element (d, h, p) at d + hd*(h + nkv*p).
void flash_attention(float* out, const float* q, const float* ck, const float* cv, int kvh,
                     int seq_len, float scale, int hd, int nkv) {
  const int BN = 64;
  std::fill(out, out + hd, 0.0f);
  float m = -INFINITY, l = 0.0f;
  std::vector<float> sc(BN);
  for (int j = 0; j < seq_len; j += BN) {
    int je = std::min(j + BN, seq_len), bl = je - j;
    float mx = -INFINITY;
    for (int nn = 0; nn < bl; ++nn) {
      const float* k = ck + (size_t)hd * (kvh + (size_t)nkv * (j + nn));
      float s = 0.0f;
      for (int d = 0; d < hd; ++d) s += q[d] * k[d];
      sc[nn] = s * scale;
      mx = std::max(mx, sc[nn]);
    }
    float mnew = std::max(m, mx);
    float sf = std::exp(m - mnew);
    if (mnew > m) {
      for (int d = 0; d < hd; ++d) out[d] *= sf;
      l *= sf;
    }
    for (int nn = 0; nn < bl; ++nn) {
      const float* v = cv + (size_t)hd * (kvh + (size_t)nkv * (j + nn));
      float p = std::exp(sc[nn] - mnew);
      l += p;
      for (int d = 0; d < hd; ++d) out[d] += p * v[d];
    }
    m = mnew;
  }
  float il = 1.0f / l;
  for (int d = 0; d < hd; ++d) out[d] *= il;
}

// tests/flash_attention_verification.jl:9-50 (exact softmax, for the KAT)
void standard_attention(float* out, const float* q, const float* ck, const float* cv, int kvh,
                        int seq_len, float scale, int hd, int nkv) {
  std::vector<float> s(seq_len);
  for (int i = 0; i < seq_len; ++i) {
    const float* k = ck + (size_t)hd * (kvh + (size_t)nkv * i);
    float a = 0.0f;
    for (int d = 0; d < hd; ++d) a += k[d] * q[d];
    s[i] = a * scale;
  }
  float mx = *std::max_element(s.begin(), s.end());
  float sum = 0.0f;
  for (auto& v : s) { v = std::exp(v - mx); sum += v; }
  for (auto& v : s) v /= sum;
  for (int d = 0; d < hd; ++d) {
    float a = 0.0f;
    for (int i = 0; i < seq_len; ++i) a += cv[(size_t)hd * (kvh + (size_t)nkv * i) + d] * s[i];
    out[d] = a;
  }
}

struct Layer {
  bool is_ssm = false;
  std::vector<float> in_norm, post_norm;
  // GDN (src/ModelCPU.jl:476-523)
  Mat in_proj, gate_proj, ssm_out, alpha, beta;
  std::vector<float> conv_w;   // GGUF ssm_conv1d data: w[c,k] = data[k + K*c]
  std::vector<float> ssm_a, dt_bias, ssm_norm;
  std::vector<float> conv_state;  // (C, K) column-major: [c + C*k]
  std::vector<float> S;           // (dv, dk, nv) column-major: [i + dv*(j + dk*h)]
  // attention (src/ModelCPU.jl:730-754)
  Mat wq, wk, wv, wo;
  std::vector<float> q_norm, k_norm;
  std::vector<float> kc, vc;      // (hd, nkv, ctx)
  // FFN
  Mat gate, up, down;
  // MoE
  Mat router, exp_gate, exp_up, exp_down, sh_gate, sh_up, sh_down;
};

struct Model {
  // int params
  int H, L, nh, nkv, hd, ffn, vocab, nv, nk, dk, dv, convk, ctx, nexp, nused, effn, sffn;
  float eps, theta, prf;
  bool deq_at_load = true;
  std::map<std::string, std::pair<std::vector<int64_t>, std::pair<int, std::vector<uint8_t>>>> pending;
  Mat embd, lm_head;
  std::vector<float> out_norm;
  std::vector<Layer> layers;
  int rd = 0;
  std::vector<float> rope_cos, rope_sin;  // (half, ctx)
  std::vector<std::vector<float>> hidden;  // after each layer, last token
};

std::vector<float> f32vec(const std::vector<uint8_t>& raw) {
  std::vector<float> v(raw.size() / 4);
  memcpy(v.data(), raw.data(), v.size() * 4);
  return v;
}

// src/ModelCPU.jl:134-153 (inv_freq in Float64 rounded to Float32; angle in
// Float32; cos/sin of the Float32 angle, correctly rounded): row of position p
void rope_row(float theta, int rd, int p, float* c, float* s) {
  for (int i = 0; i < rd / 2; ++i) {
    float inv = (float)(1.0 / std::pow((double)theta, (2.0 * i) / (double)rd));
    float f = inv * (float)p;
    c[i] = (float)std::cos((double)f);
    s[i] = (float)std::sin((double)f);
  }
}

void build_rope(Model& m) {
  int half = m.rd / 2;
  m.rope_cos.assign((size_t)half * m.ctx, 0.0f);
  m.rope_sin.assign((size_t)half * m.ctx, 0.0f);
  for (int p = 0; p < m.ctx; ++p)
    rope_row(m.theta, m.rd, p, m.rope_cos.data() + (size_t)p * half, m.rope_sin.data() + (size_t)p * half);
}

// src/ModelCPU.jl:187-231 on nheads heads of hd, with the RoPE row (c, s)
// of the current position
void rmsnorm_rotary_row(float* x, int nheads, int hd, int rd, const float* c, const float* s, const float* w,
                        float eps) {
  int half = rd / 2;
  for (int h = 0; h < nheads; ++h) {
    float* v = x + (size_t)h * hd;
    float ss = 0.0f;
    for (int i = 0; i < hd; ++i) ss += v[i] * v[i];
    float rms = std::sqrt(ss / (float)hd + eps);
    float inv = 1.0f / rms;
    for (int i = 0; i < hd; ++i) v[i] = v[i] * inv * w[i];
    for (int i = 0; i < half; ++i) {
      float x1 = v[i], x2 = v[i + half];
      v[i] = x1 * c[i] - x2 * s[i];
      v[i + half] = x1 * s[i] + x2 * c[i];
    }
  }
}

// src/ModelCPU.jl:766-851 after the q/k/v projections: q/k RMSNorm + partial
// RoPE, KV-cache append at pos, flash attention per query head (blocked GQA
// kv = h / (nh/nkv)), sigmoid gate.  qg holds [q | gate] per head; the cache
// is (hd, nkv, ctx) column-major.
void attention_step(const float* qg, const float* k_in, const float* v_in, const float* q_norm,
                    const float* k_norm, float eps, int nh, int nkv, int hd, int rd, const float* rc,
                    const float* rs, float* kc, float* vc, int pos, float* out) {
  std::vector<float> k(k_in, k_in + (size_t)nkv * hd), q(nh * hd), gt(nh * hd);
  for (int h = 0; h < nh; ++h)
    for (int i = 0; i < hd; ++i) {
      q[h * hd + i] = qg[h * 2 * hd + i];
      gt[h * hd + i] = qg[h * 2 * hd + hd + i];
    }
  rmsnorm_rotary_row(q.data(), nh, hd, rd, rc, rs, q_norm, eps);
  rmsnorm_rotary_row(k.data(), nkv, hd, rd, rc, rs, k_norm, eps);
  for (int h = 0; h < nkv; ++h)
    for (int d = 0; d < hd; ++d) {
      kc[d + (size_t)hd * (h + (size_t)nkv * pos)] = k[h * hd + d];
      vc[d + (size_t)hd * (h + (size_t)nkv * pos)] = v_in[h * hd + d];
    }
  int gqa = nh / nkv;
  float scale = 1.0f / std::sqrt((float)hd);
  for (int h = 0; h < nh; ++h)
    flash_attention(out + (size_t)h * hd, q.data() + h * hd, kc, vc, h / gqa, pos + 1, scale, hd, nkv);
  for (size_t i = 0; i < gt.size(); ++i) out[i] *= 1.0f / (1.0f + std::exp(-gt[i]));
}

// src/ModelCPU.jl:447-473
void mlp(const Layer& ly, const float* x, float* out, int H, int I) {
  std::vector<float> g(I), u(I);
  ly.gate.gemv(x, g.data());
  for (auto& v : g) v = silu(v);
  ly.up.gemv(x, u.data());
  for (int i = 0; i < I; ++i) g[i] *= u[i];
  ly.down.gemv(g.data(), out);
  (void)H;
}

// src/Model.jl:497-526 restated on fp32: softmax router, stable top-k (ties to
// the lower expert index, as sortperm(rev=true) does), renormalised weights,
// sum of SwiGLU experts.  Plus an always-on shared expert (config 5; the
// reference has none, so that term is parity-unpinned).
void moe(const Layer& ly, const Model& m, const float* x, float* out) {
  int E = m.nexp, K = m.nused, H = m.H, I = m.effn;
  std::vector<float> lg(E);
  ly.router.gemv(x, lg.data());
  float mx = *std::max_element(lg.begin(), lg.end());
  std::vector<float> p(E);
  float sum = 0.0f;
  for (int e = 0; e < E; ++e) { p[e] = std::exp(lg[e] - mx); }
  for (int e = 0; e < E; ++e) sum += p[e];
  for (int e = 0; e < E; ++e) p[e] /= sum;
  std::vector<int> idx(E);
  std::iota(idx.begin(), idx.end(), 0);
  std::stable_sort(idx.begin(), idx.end(), [&](int a, int b) { return p[a] > p[b]; });
  float tsum = 0.0f;
  for (int i = 0; i < K; ++i) tsum += p[idx[i]];
  std::fill(out, out + H, 0.0f);
  std::vector<float> g(I), u(I), r(H);
  for (int i = 0; i < K; ++i) {
    int e = idx[i];
    float w = p[e] / tsum;
    ly.exp_gate.gemv_rows(x, g.data(), (int64_t)e * I, (int64_t)(e + 1) * I);
    ly.exp_up.gemv_rows(x, u.data(), (int64_t)e * I, (int64_t)(e + 1) * I);
    for (int j = 0; j < I; ++j) g[j] = silu(g[j]) * u[j];
    ly.exp_down.gemv_rows(g.data(), r.data(), (int64_t)e * H, (int64_t)(e + 1) * H);
    for (int j = 0; j < H; ++j) out[j] += w * r[j];
  }
  if (!ly.sh_gate.empty()) {
    int S = (int)ly.sh_gate.outer;
    std::vector<float> sg(S), su(S);
    ly.sh_gate.gemv(x, sg.data());
    ly.sh_up.gemv(x, su.data());
    for (int j = 0; j < S; ++j) sg[j] = silu(sg[j]) * su[j];
    ly.sh_down.gemv(sg.data(), r.data());
    for (int j = 0; j < H; ++j) out[j] += r[j];
  }
}

// src/ModelCPU.jl:531-700
void gdn(Model& m, Layer& ly, const float* x, float* out) {
  int C = (int)ly.in_proj.outer, K = m.convk, di = m.nv * m.dv;
  int nk = m.nk, nv = m.nv, dk = m.dk, dv = m.dv;
  std::vector<float> qkv(C), z(di), xc(C), al(nv), be(nv), y(di, 0.0f);
  ly.in_proj.gemv(x, qkv.data());
  ly.gate_proj.gemv(x, z.data());
  for (int j = 0; j < K - 1; ++j)
    for (int c = 0; c < C; ++c) ly.conv_state[c + (size_t)C * j] = ly.conv_state[c + (size_t)C * (j + 1)];
  for (int c = 0; c < C; ++c) ly.conv_state[c + (size_t)C * (K - 1)] = qkv[c];
  for (int c = 0; c < C; ++c) {
    float v = 0.0f;
    for (int k = 0; k < K; ++k) v += ly.conv_state[c + (size_t)C * k] * ly.conv_w[k + (size_t)K * c];
    xc[c] = v / (1.0f + std::exp(-v));
  }
  const float* q_all = xc.data();
  const float* k_all = xc.data() + nk * dk;
  const float* v_all = xc.data() + 2 * nk * dk;
  ly.alpha.gemv(x, al.data());
  ly.beta.gemv(x, be.data());
  const float eps = 1.0e-6f;
  std::vector<float> qn(dk), kn(dk), sk(dv), dd(dv);
  for (int h = 0; h < nv; ++h) {
    int g = h % nk;  // modulo head map (src/ModelCPU.jl:587)
    const float* qg = q_all + g * dk;
    const float* kg = k_all + g * dk;
    const float* vg = v_all + h * dv;
    float scale = 1.0f / std::sqrt((float)dk);
    float qs = 0.0f, ks = 0.0f;
    for (int i = 0; i < dk; ++i) { qs += qg[i] * qg[i]; ks += kg[i] * kg[i]; }
    float qnv = 1.0f / (std::sqrt(qs) + eps) * scale;
    float knv = 1.0f / (std::sqrt(ks) + eps);
    for (int i = 0; i < dk; ++i) { qn[i] = qg[i] * qnv; kn[i] = kg[i] * knv; }
    double a = std::min(20.0, std::max(-20.0, (double)al[h] + (double)ly.dt_bias[h]));
    double sp = std::log(1.0 + std::exp(a));
    float decay = (float)((double)ly.ssm_a[h] * sp);
    float dapply = std::exp(decay);
    double bv = std::min(20.0, std::max(-20.0, (double)be[h]));
    float bg = (float)(1.0 / (1.0 + std::exp(-bv)));
    float* S = ly.S.data() + (size_t)dv * dk * h;  // S[i + dv*j]
    for (size_t t = 0; t < (size_t)dv * dk; ++t) S[t] *= dapply;
    for (int i = 0; i < dv; ++i) {
      float s = 0.0f;
      for (int j = 0; j < dk; ++j) s += S[i + (size_t)dv * j] * kn[j];
      sk[i] = s;
    }
    for (int i = 0; i < dv; ++i) dd[i] = bg * (vg[i] - sk[i]);
    for (int j = 0; j < dk; ++j)
      for (int i = 0; i < dv; ++i) S[i + (size_t)dv * j] += dd[i] * kn[j];
    for (int i = 0; i < dv; ++i) {
      float s = 0.0f;
      for (int j = 0; j < dk; ++j) s += S[i + (size_t)dv * j] * qn[j];
      y[h * dv + i] = s;
    }
  }
  for (int h = 0; h < nv; ++h) rmsnorm(y.data() + h * dv, y.data() + h * dv, ly.ssm_norm.data(), dv, m.eps);
  for (int i = 0; i < di; ++i) y[i] = y[i] * z[i] * (1.0f / (1.0f + std::exp(-z[i])));
  ly.ssm_out.gemv(y.data(), out);
}

// src/ModelCPU.jl:756-856
void attention(Model& m, Layer& ly, const float* x, int pos, float* out) {
  int nh = m.nh, nkv = m.nkv, hd = m.hd, half = m.rd / 2;
  std::vector<float> qg(2 * nh * hd), k(nkv * hd), v(nkv * hd), o(nh * hd, 0.0f);
  ly.wq.gemv(x, qg.data());
  ly.wk.gemv(x, k.data());
  ly.wv.gemv(x, v.data());
  attention_step(qg.data(), k.data(), v.data(), ly.q_norm.data(), ly.k_norm.data(), m.eps, nh, nkv, hd, m.rd,
                 m.rope_cos.data() + (size_t)pos * half, m.rope_sin.data() + (size_t)pos * half, ly.kc.data(),
                 ly.vc.data(), pos, o.data());
  ly.wo.gemv(o.data(), out);
}

// src/ModelCPU.jl:870-891
void layer_forward(Model& m, int li, float* x, int pos) {
  Layer& ly = m.layers[li];
  int H = m.H;
  std::vector<float> xn(H), r(H);
  rmsnorm(xn.data(), x, ly.in_norm.data(), H, m.eps);
  if (ly.is_ssm) gdn(m, ly, xn.data(), r.data());
  else attention(m, ly, xn.data(), pos, r.data());
  for (int i = 0; i < H; ++i) x[i] += r[i];
  rmsnorm(xn.data(), x, ly.post_norm.data(), H, m.eps);
  if (m.nexp) moe(ly, m, xn.data(), r.data());
  else mlp(ly, xn.data(), r.data(), H, m.ffn);
  for (int i = 0; i < H; ++i) x[i] += r[i];
}

}  // namespace

// ---------------------------------------------------------------------------
// The reference's Q8_K activation path (src/kernels/quant_kernels.c), restated
// scalar with the lane structure of its AVX2 + FMA build: 256-bit integer
// lane k of a 32-byte chunk covers bytes 4k..4k+3, so a block contributes
// eight exact int32 lane sums; each lane keeps its own float accumulator
// (fma over the blocks in order) and the eight accumulators are combined in
// hsum_float_8's order (quant_kernels.c:91-98).
// ---------------------------------------------------------------------------
namespace q8k {

constexpr int QK = 256;
constexpr int Q8K_BYTES = 292;  // float d; int8 qs[256]; int16 bsums[16]

float hsum8(const float a[8]) {
  float s0 = a[4] + a[0], s1 = a[5] + a[1], s2 = a[6] + a[2], s3 = a[7] + a[3];
  return (s0 + s2) + (s1 + s3);
}

// 6-bit scale / min of sub-block j (the utmp shuffle of quant_kernels.c:224-230)
void k4_scale_min(const uint8_t* s, int j, int* sc, int* m) {
  if (j < 4) { *sc = s[j] & 63; *m = s[j + 4] & 63; }
  else { *sc = (s[j + 4] & 15) | ((s[j - 4] >> 6) << 4); *m = (s[j + 4] >> 4) | ((s[j] >> 6) << 4); }
}

// Q4_K / Q5_K (quant_kernels.c:204-255, :311-398): lane k of block i is
// sum_j sc[2j] * sum_{b=4k..4k+3} lo_j[b] q8[64j+b] + sc[2j+1] * sum hi_j[b] q8[64j+32+b]
template <bool Q5>
float vec_dot_k45(const uint8_t* x, const uint8_t* y, int nb) {
  const int bb = Q5 ? 176 : 144;
  float acc[8] = {0}, accm[4] = {0}, summs = 0.0f;
  for (int i = 0; i < nb; ++i) {
    const uint8_t* xb = x + (size_t)i * bb;
    const uint8_t* yb = y + (size_t)i * Q8K_BYTES;
    float yd;
    memcpy(&yd, yb, 4);
    const int8_t* q8 = (const int8_t*)(yb + 4);
    int16_t bs[16];
    memcpy(bs, yb + 260, 32);
    const float d = yd * h2f(rd16(xb)), dmin = -yd * h2f(rd16(xb + 2));
    const uint8_t* sc6 = xb + 4;
    const uint8_t* qh = Q5 ? xb + 16 : nullptr;
    const uint8_t* qs = xb + (Q5 ? 48 : 16);
    int sc[8], mn[8];
    for (int j = 0; j < 8; ++j) k4_scale_min(sc6, j, &sc[j], &mn[j]);
    int32_t lane[8] = {0};
    for (int j = 0; j < 4; ++j)
      for (int k = 0; k < 8; ++k) {
        int lo = 0, hi = 0;
        for (int b = 4 * k; b < 4 * k + 4; ++b) {
          int ql = qs[32 * j + b] & 15, qhh = qs[32 * j + b] >> 4;
          if (Q5) { ql |= ((qh[b] >> (2 * j)) & 1) << 4; qhh |= ((qh[b] >> (2 * j + 1)) & 1) << 4; }
          lo += ql * q8[64 * j + b];
          hi += qhh * q8[64 * j + 32 + b];
        }
        lane[k] += sc[2 * j] * lo + sc[2 * j + 1] * hi;
      }
    for (int k = 0; k < 8; ++k) acc[k] = fmaf(d, (float)lane[k], acc[k]);
    int32_t prod[4];
    for (int l = 0; l < 4; ++l) {
      const int16_t s0 = (int16_t)(bs[4 * l] + bs[4 * l + 1]), s1 = (int16_t)(bs[4 * l + 2] + bs[4 * l + 3]);
      prod[l] = mn[2 * l] * s0 + mn[2 * l + 1] * s1;
    }
    if (Q5) {
      // scalar `summs += dmin * hsum` of the FMA build is contracted to an fma
      summs = fmaf(dmin, (float)((prod[0] + prod[1]) + (prod[2] + prod[3])), summs);
    } else {
      for (int l = 0; l < 4; ++l) accm[l] = fmaf(dmin, (float)prod[l], accm[l]);
    }
  }
  if (Q5) return hsum8(acc) + summs;
  return hsum8(acc) + ((accm[0] + accm[2]) + (accm[1] + accm[3]));
}

// Q6_K (quant_kernels.c:440-519): chunk t of half j holds values
// 128j + 32t + b with scales 8j+2t (bytes 0-15) and 8j+2t+1 (bytes 16-31)
float vec_dot_q6(const uint8_t* x, const uint8_t* y, int nb) {
  float acc[8] = {0};
  for (int i = 0; i < nb; ++i) {
    const uint8_t* xb = x + (size_t)i * 210;
    const uint8_t* yb = y + (size_t)i * Q8K_BYTES;
    float yd;
    memcpy(&yd, yb, 4);
    const int8_t* q8 = (const int8_t*)(yb + 4);
    const uint8_t *ql = xb, *qh = xb + 128;
    const int8_t* sc = (const int8_t*)(xb + 192);
    const float d = yd * h2f(rd16(xb + 208));
    int32_t lane[8] = {0};
    for (int j = 0; j < 2; ++j)
      for (int t = 0; t < 4; ++t)
        for (int k = 0; k < 8; ++k) {
          int s = 0;
          for (int b = 4 * k; b < 4 * k + 4; ++b) {
            const uint8_t lb = ql[64 * j + (t & 1) * 32 + b];
            const int q = ((t < 2 ? lb : lb >> 4) & 15) | (((qh[32 * j + b] >> (2 * t)) & 3) << 4);
            s += (q - 32) * q8[128 * j + 32 * t + b];
          }
          lane[k] += sc[8 * j + 2 * t + (k >= 4)] * s;
        }
    for (int k = 0; k < 8; ++k) acc[k] = fmaf(d, (float)lane[k], acc[k]);
  }
  return hsum8(acc);
}

// Q8_0 x Q8_0 (quant_kernels.c:531-559, mul_sum_i8_pairs_float :146-158):
// |x| times y carrying x's sign (int8 wrap of -(-128)), pair sums saturated to int16
float vec_dot_q80(const uint8_t* x, const uint8_t* y, int nb) {
  float acc[8] = {0};
  for (int i = 0; i < nb; ++i) {
    const uint8_t* xb = x + (size_t)i * 34;
    const uint8_t* yb = y + (size_t)i * 34;
    const float d = h2f(rd16(xb)) * h2f(rd16(yb));
    const int8_t *qx = (const int8_t*)(xb + 2), *qy = (const int8_t*)(yb + 2);
    for (int k = 0; k < 8; ++k) {
      int32_t s = 0;
      for (int p = 0; p < 2; ++p) {
        int pair = 0;
        for (int b = 4 * k + 2 * p; b < 4 * k + 2 * p + 2; ++b) {
          const int ax = qx[b] < 0 ? -(int)qx[b] : qx[b];
          const int sy = qx[b] < 0 ? (int8_t)(-qy[b]) : (qx[b] == 0 ? 0 : qy[b]);
          pair += ax * sy;
        }
        s += std::min(32767, std::max(-32768, pair));
      }
      acc[k] = fmaf(d, (float)s, acc[k]);
    }
  }
  return hsum8(acc);
}

// quantize_row_q8_K (quant_kernels.c:166-196)
void quantize_q8k(const float* x, uint8_t* y, int64_t k) {
  for (int64_t i = 0; i < k / QK; ++i) {
    const float* src = x + i * QK;
    uint8_t* yb = y + i * Q8K_BYTES;
    float amax = 0.0f;
    for (int j = 0; j < QK; ++j) {
      float ax = fabsf(src[j]);
      if (ax > amax) amax = ax;
    }
    const float d = amax / 127.0f, id = d != 0.0f ? 1.0f / d : 0.0f;
    memcpy(yb, &d, 4);
    for (int j = 0; j < QK; j += 16) {
      int sum = 0;
      for (int l = 0; l < 16; ++l) {
        const int8_t q = (int8_t)roundf(src[j + l] * id);
        yb[4 + j + l] = (uint8_t)q;
        sum += q;
      }
      const int16_t s16 = (int16_t)sum;
      memcpy(yb + 260 + 2 * (j / 16), &s16, 2);
    }
  }
}

// q*_k_gemv / q8_0_gemv (quant_kernels.c:602-697): the reference library's
// GEMV numerics -- x quantized once to Q8_K, one vec_dot per row; Q8_0 keeps
// fp32 x and lane k takes fma(d, q[8c+k] * x[8c+k], acc) per block and chunk c.
void ref_gemv(int type, const uint8_t* W, const float* x, float* out, int inner, int outer) {
  if (type == 8) {
    const int nb = inner / 32;
    for (int r = 0; r < outer; ++r) {
      float acc[8] = {0};
      for (int b = 0; b < nb; ++b) {
        const uint8_t* blk = W + ((size_t)r * nb + b) * 34;
        const float d = h2f(rd16(blk));
        for (int c = 0; c < 4; ++c)
          for (int k = 0; k < 8; ++k) {
            const float p = (float)(int8_t)blk[2 + 8 * c + k] * x[b * 32 + 8 * c + k];
            acc[k] = fmaf(d, p, acc[k]);
          }
      }
      out[r] = hsum8(acc);
    }
    return;
  }
  const int nb = inner / QK, bb = type == 12 ? 144 : type == 13 ? 176 : 210;
  std::vector<uint8_t> y8((size_t)nb * Q8K_BYTES);
  quantize_q8k(x, y8.data(), inner);
  for (int r = 0; r < outer; ++r) {
    const uint8_t* w = W + (size_t)r * nb * bb;
    out[r] = type == 12 ? vec_dot_k45<false>(w, y8.data(), nb)
             : type == 13 ? vec_dot_k45<true>(w, y8.data(), nb) : vec_dot_q6(w, y8.data(), nb);
  }
}

}  // namespace q8k

extern "C" {

void orc_quantize_row_q8_K(const float* x, uint8_t* y, int64_t k) { q8k::quantize_q8k(x, y, k); }
void orc_ref_gemv(int type, const uint8_t* W, const float* x, float* out, int inner, int outer) {
  q8k::ref_gemv(type, W, x, out, inner, outer);
}
float orc_vec_dot_q8k(int type, const uint8_t* x, const uint8_t* y, int nb) {
  switch (type) {
    case 12: return q8k::vec_dot_k45<false>(x, y, nb);
    case 13: return q8k::vec_dot_k45<true>(x, y, nb);
    case 14: return q8k::vec_dot_q6(x, y, nb);
    case 8: return q8k::vec_dot_q80(x, y, nb);
  }
  return NAN;
}

int orc_dequant(int type, const uint8_t* src, int64_t n, float* dst) { return dequant(type, src, n, dst); }

// y[b*outer + r] = sum_i W[r,i] * x[b*inner + i]  (dequantize, then fp32 dot)
int orc_gemv(int type, const uint8_t* W, const float* x, float* y, int inner, int outer, int batch) {
  if (inner % block_elems(type)) return -1;
  int64_t rb = (int64_t)inner / block_elems(type) * block_bytes(type);
#pragma omp parallel
  {
    std::vector<float> buf(inner);
#pragma omp for schedule(static)
    for (int r = 0; r < outer; ++r) {
      dequant(type, W + (int64_t)r * rb, inner, buf.data());
      for (int b = 0; b < batch; ++b) y[(int64_t)b * outer + r] = dot(buf.data(), x + (int64_t)b * inner, inner);
    }
  }
  return 0;
}

void orc_flash_attention(float* out, const float* q, const float* ck, const float* cv, int kvh, int seq_len,
                         float scale, int hd, int nkv) {
  flash_attention(out, q, ck, cv, kvh, seq_len, scale, hd, nkv);
}
// one gated attention step (attention_step above) at position pos; the RoPE
// row of pos is built from theta as build_rope does
void orc_attention_step(const float* qg, const float* k, const float* v, const float* q_norm, const float* k_norm,
                        float eps, int nh, int nkv, int hd, int rd, float theta, float* kc, float* vc, int pos,
                        float* out) {
  std::vector<float> c(rd / 2), s(rd / 2);
  rope_row(theta, rd, pos, c.data(), s.data());
  attention_step(qg, k, v, q_norm, k_norm, eps, nh, nkv, hd, rd, c.data(), s.data(), kc, vc, pos, out);
}
void orc_standard_attention(float* out, const float* q, const float* ck, const float* cv, int kvh, int seq_len,
                            float scale, int hd, int nkv) {
  standard_attention(out, q, ck, cv, kvh, seq_len, scale, hd, nkv);
}

// Config-3 isolated delta rule: per step t and head h, with given L2-normalised
// q/k, v, beta and log-decay g (src/ModelCPU.jl:640-674 without the
// projections): S = S*exp(g); S += beta*(v - S k) k^T; y = S q.
// Layouts: q,k (T, H, dk); v,y (T, H, dv); beta,g (T, H); S (H, dv, dk) row-major.
void orc_gdn_recurrence(int T, int H, int dk, int dv, const float* q, const float* k, const float* v,
                        const float* beta, const float* g, float* S, float* y) {
#pragma omp parallel for schedule(static)
  for (int h = 0; h < H; ++h) {
    std::vector<float> sk(dv);
    float* Sh = S + (size_t)h * dv * dk;
    for (int t = 0; t < T; ++t) {
      const float* qt = q + ((size_t)t * H + h) * dk;
      const float* kt = k + ((size_t)t * H + h) * dk;
      const float* vt = v + ((size_t)t * H + h) * dv;
      float e = std::exp(g[(size_t)t * H + h]), b = beta[(size_t)t * H + h];
      for (int i = 0; i < dv; ++i) {
        float* row = Sh + (size_t)i * dk;
        float s = 0.0f;
        for (int j = 0; j < dk; ++j) { row[j] *= e; s += row[j] * kt[j]; }
        float d = b * (vt[i] - s);
        float o = 0.0f;
        for (int j = 0; j < dk; ++j) { row[j] += d * kt[j]; o += row[j] * qt[j]; }
        y[((size_t)t * H + h) * dv + i] = o;
      }
    }
  }
}

// src/ModelCPU.jl:1202-1225 (penalties for the seen tokens) then
// softmax_sample (:1123-1200) with the uniform draw r given; 0-based result.
int orc_softmax_sample(const float* logits_in, int V, float temperature, float top_p, int top_k, float min_p,
                       float presence, float repetition, const int* seen, int n_seen, float r) {
  std::vector<float> l(logits_in, logits_in + V);
  std::vector<char> mark(V, 0);
  for (int i = 0; i < n_seen; ++i)
    if (seen[i] >= 0 && seen[i] < V) mark[seen[i]] = 1;
  if (presence != 0.0f)
    for (int i = 0; i < V; ++i)
      if (mark[i]) l[i] -= presence;
  if (repetition != 1.0f)
    for (int i = 0; i < V; ++i)
      if (mark[i]) l[i] = l[i] > 0 ? l[i] / repetition : l[i] * repetition;
  if (temperature == 0.0f) return (int)(std::max_element(l.begin(), l.end()) - l.begin());   // first max
  if (temperature != 1.0f)
    for (auto& v : l) v = v / temperature;
  // stable descending order: ties keep the lower index first (sortperm rev=true)
  auto desc = [](const std::vector<float>& a) {
    std::vector<int> idx(a.size());
    std::iota(idx.begin(), idx.end(), 0);
    std::stable_sort(idx.begin(), idx.end(), [&](int x, int y) { return a[x] > a[y]; });
    return idx;
  };
  if (top_k > 0) {
    std::vector<int> idx = desc(l);
    std::vector<char> keep(V, 0);
    for (int i = 0; i < std::min(top_k, V); ++i) keep[idx[i]] = 1;
    for (int i = 0; i < V; ++i)
      if (!keep[i]) l[i] = -INFINITY;
  }
  const float mx = *std::max_element(l.begin(), l.end());
  std::vector<float> p(V);
  float s = 0.0f;
  for (int i = 0; i < V; ++i) { p[i] = std::exp(l[i] - mx); s += p[i]; }
  for (auto& v : p) v = v / s;
  if (top_p < 1.0f) {
    std::vector<int> idx = desc(p);
    std::vector<char> keep(V, 0);
    float c = 0.0f;
    for (int i : idx) {
      keep[i] = 1;
      c += p[i];
      if (c >= top_p) break;
    }
    float t = 0.0f;
    for (int i = 0; i < V; ++i) {
      if (!keep[i]) p[i] = 0.0f;
      t += p[i];
    }
    if (t > 0.0f)
      for (auto& v : p) v = v / t;
  }
  if (min_p > 0.0f) {
    const float th = *std::max_element(p.begin(), p.end()) * min_p;
    float t = 0.0f;
    for (int i = 0; i < V; ++i) {
      if (p[i] < th) p[i] = 0.0f;
      t += p[i];
    }
    if (t > 0.0f)
      for (auto& v : p) v = v / t;
  }
  float c = 0.0f;
  for (int i = 0; i < V; ++i) {
    c += p[i];
    if (r <= c) return i;
  }
  return V - 1;
}

// ---- model ------------------------------------------------------------------
// ip: [hidden, layers, n_heads, n_kv, head_dim, ffn, vocab, nv, nk, dk, dv,
//      conv_k, ctx, n_experts, n_used, expert_ffn, shexp_ffn, dequant_at_load]
// fp: [eps, rope_theta, partial_rotary_factor]
void* orc_model_create(const int64_t* ip, const double* fp) {
  auto* m = new Model();
  m->H = (int)ip[0]; m->L = (int)ip[1]; m->nh = (int)ip[2]; m->nkv = (int)ip[3]; m->hd = (int)ip[4];
  m->ffn = (int)ip[5]; m->vocab = (int)ip[6]; m->nv = (int)ip[7]; m->nk = (int)ip[8]; m->dk = (int)ip[9];
  m->dv = (int)ip[10]; m->convk = (int)ip[11]; m->ctx = (int)ip[12]; m->nexp = (int)ip[13];
  m->nused = (int)ip[14]; m->effn = (int)ip[15]; m->sffn = (int)ip[16]; m->deq_at_load = ip[17] != 0;
  m->eps = (float)fp[0]; m->theta = (float)fp[1]; m->prf = (float)fp[2];
  m->layers.resize(m->L);
  return m;
}

void orc_model_destroy(void* h) { delete (Model*)h; }

int orc_model_set_tensor(void* h, const char* name, int type, const int64_t* ne, int ndim, const uint8_t* data,
                         int64_t nbytes) {
  auto* m = (Model*)h;
  std::vector<int64_t> dims(ne, ne + ndim);
  m->pending[name] = {dims, {type, std::vector<uint8_t>(data, data + nbytes)}};
  return 0;
}

int orc_model_finalize(void* h) {
  auto* m = (Model*)h;
  auto take = [&](const std::string& n, Mat& M, bool deq) -> bool {
    auto it = m->pending.find(n);
    if (it == m->pending.end()) return false;
    auto& d = it->second.first;
    int64_t inner = d[0], outer = 1;
    for (size_t i = 1; i < d.size(); ++i) outer *= d[i];
    M.load(it->second.second.first, inner, outer, it->second.second.second.data(), deq);
    m->pending.erase(it);
    return true;
  };
  auto takef = [&](const std::string& n, std::vector<float>& v) -> bool {
    auto it = m->pending.find(n);
    if (it == m->pending.end()) return false;
    if (it->second.second.first != T_F32) return false;
    v = f32vec(it->second.second.second);
    m->pending.erase(it);
    return true;
  };
  bool dq = m->deq_at_load;
  if (!take("token_embd.weight", m->embd, false)) return -1;
  if (!take("output.weight", m->lm_head, dq)) {
    // tied lm_head (src/LoaderCPU.jl:358-371): fp32 copy of the embedding
    m->lm_head = m->embd;
    if (dq) {
      m->lm_head.f32.resize((size_t)m->embd.inner * m->embd.outer);
      dequant(m->embd.type, m->embd.raw.data(), m->embd.inner * m->embd.outer, m->lm_head.f32.data());
      m->lm_head.raw.clear();
      m->lm_head.raw.shrink_to_fit();
    }
  }
  if (!takef("output_norm.weight", m->out_norm)) return -2;
  for (int i = 0; i < m->L; ++i) {
    std::string p = "blk." + std::to_string(i) + ".";
    Layer& ly = m->layers[i];
    if (!takef(p + "attn_norm.weight", ly.in_norm) || !takef(p + "post_attention_norm.weight", ly.post_norm))
      return -3;
    ly.is_ssm = m->pending.count(p + "ssm_a") > 0;  // src/LoaderCPU.jl:431
    if (ly.is_ssm) {
      if (!take(p + "attn_qkv.weight", ly.in_proj, dq) || !take(p + "attn_gate.weight", ly.gate_proj, dq) ||
          !take(p + "ssm_out.weight", ly.ssm_out, dq) || !take(p + "ssm_alpha.weight", ly.alpha, true) ||
          !take(p + "ssm_beta.weight", ly.beta, true) || !takef(p + "ssm_conv1d.weight", ly.conv_w) ||
          !takef(p + "ssm_a", ly.ssm_a) || !takef(p + "ssm_dt.bias", ly.dt_bias) ||
          !takef(p + "ssm_norm.weight", ly.ssm_norm))
        return -4;
      ly.conv_state.assign((size_t)ly.in_proj.outer * m->convk, 0.0f);
      ly.S.assign((size_t)m->nv * m->dv * m->dk, 0.0f);
    } else {
      if (!take(p + "attn_q.weight", ly.wq, dq) || !take(p + "attn_k.weight", ly.wk, dq) ||
          !take(p + "attn_v.weight", ly.wv, dq) || !take(p + "attn_output.weight", ly.wo, dq) ||
          !takef(p + "attn_q_norm.weight", ly.q_norm) || !takef(p + "attn_k_norm.weight", ly.k_norm))
        return -5;
      ly.kc.assign((size_t)m->hd * m->nkv * m->ctx, 0.0f);
      ly.vc.assign((size_t)m->hd * m->nkv * m->ctx, 0.0f);
    }
    if (m->nexp) {
      if (!take(p + "ffn_gate_inp.weight", ly.router, true) || !take(p + "ffn_gate_exps.weight", ly.exp_gate, false) ||
          !take(p + "ffn_up_exps.weight", ly.exp_up, false) || !take(p + "ffn_down_exps.weight", ly.exp_down, false))
        return -6;
      take(p + "ffn_gate_shexp.weight", ly.sh_gate, dq);
      take(p + "ffn_up_shexp.weight", ly.sh_up, dq);
      take(p + "ffn_down_shexp.weight", ly.sh_down, dq);
    } else {
      if (!take(p + "ffn_gate.weight", ly.gate, dq) || !take(p + "ffn_up.weight", ly.up, dq) ||
          !take(p + "ffn_down.weight", ly.down, dq))
        return -7;
    }
  }
  m->pending.clear();
  m->rd = (int)std::lround(m->hd * (double)m->prf);  // src/LoaderCPU.jl:375
  build_rope(*m);
  m->hidden.assign(m->L, std::vector<float>(m->H, 0.0f));
  return 0;
}

// src/ModelCPU.jl:525-529, 991-997 (plus clearing the KV cache, as a fresh
// init_kv_cache_cpu does)
void orc_model_reset(void* h) {
  auto* m = (Model*)h;
  for (auto& ly : m->layers) {
    std::fill(ly.conv_state.begin(), ly.conv_state.end(), 0.0f);
    std::fill(ly.S.begin(), ly.S.end(), 0.0f);
    std::fill(ly.kc.begin(), ly.kc.end(), 0.0f);
    std::fill(ly.vc.begin(), ly.vc.end(), 0.0f);
  }
}

int orc_layer_forward(void* h, int layer, float* x, int pos) {
  auto* m = (Model*)h;
  if (layer < 0 || layer >= m->L || pos < 0 || pos >= m->ctx) return -1;
  layer_forward(*m, layer, x, pos);
  return 0;
}

// src/ModelCPU.jl:945-989 + 1014-1046 + 1123-1127.  Token ids are 0-based.
// logits (vocab floats) of the last token if non-null; *argmax = first max.
int orc_forward(void* h, const int32_t* toks, int n, int pos, float* logits, int32_t* argmax) {
  auto* m = (Model*)h;
  std::vector<float> x(m->H), xn(m->H), lg(m->vocab);
  for (int t = 0; t < n; ++t) {
    if (toks[t] < 0 || toks[t] >= m->vocab || pos + t >= m->ctx) return -1;
    m->embd.row(toks[t], x.data());
    for (int i = 0; i < m->L; ++i) {
      layer_forward(*m, i, x.data(), pos + t);
      m->hidden[i] = x;
    }
  }
  rmsnorm(xn.data(), x.data(), m->out_norm.data(), m->H, m->eps);
  m->lm_head.gemv(xn.data(), lg.data());
  int best = 0;
  for (int i = 1; i < m->vocab; ++i)
    if (lg[i] > lg[best]) best = i;
  if (argmax) *argmax = best;
  if (logits) memcpy(logits, lg.data(), lg.size() * 4);
  return 0;
}

int orc_get_hidden(void* h, int layer, float* out) {
  auto* m = (Model*)h;
  if (layer < 0 || layer >= m->L) return -1;
  memcpy(out, m->hidden[layer].data(), m->H * 4);
  return 0;
}

// token embedding row (bit-exact dequant of token_embd row `tok`)
int orc_embed(void* h, int tok, float* out) {
  auto* m = (Model*)h;
  if (tok < 0 || tok >= m->vocab) return -1;
  m->embd.row(tok, out);
  return 0;
}

int orc_num_threads() {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}

}  // extern "C"
