"""Independent numpy restatement of the reference CPU forward (test helper).

A second, vectorised statement of src/ModelCPU.jl (rmsnorm_cpu! :110-122,
RoPE :134-231, GatedDeltaNetCPU :531-700, FullAttentionCPU :756-856 with an
exact softmax, mlp_forward :447-473, DecoderLayerCPU :870-891, forward_cpu!
:945-989) used to cross-check the C++ oracle on small models.  Weights are
dequantized by gguf-py (ggml semantics, identical to Inferno.jl for the
K-quants used here).
"""
import numpy as np


def dequant(t):
    import gguf
    from gguf import quants
    if t.ggml_type == 0:
        return t.data.view(np.float32).reshape(tuple(reversed(t.ne)))
    return quants.dequantize(t.data, gguf.GGMLQuantizationType(t.ggml_type)).reshape(tuple(reversed(t.ne)))


class NumpyModel:
    def __init__(self, spec, T):
        self.s = spec
        self.W = {k: dequant(v).astype(np.float64) for k, v in T.items()}
        s = spec
        self.rd = int(round(s.head_dim * s.partial_rotary))
        half = self.rd // 2
        inv = (1.0 / (np.float64(np.float32(s.rope_theta)) ** (2.0 * np.arange(half) / self.rd))).astype(np.float32)
        ang = (inv[None, :] * np.arange(s.ctx, dtype=np.float32)[:, None]).astype(np.float32)
        self.cos = np.cos(ang.astype(np.float64))
        self.sin = np.sin(ang.astype(np.float64))
        self.reset()

    def reset(self):
        s = self.s
        self.conv, self.S, self.kc, self.vc = {}, {}, {}, {}
        for i in range(s.layers):
            if f"blk.{i}.ssm_a" in self.W:
                self.conv[i] = np.zeros((s.conv_k, s.conv_channels))
                self.S[i] = np.zeros((s.ssm_nv, s.ssm_dv, s.ssm_dk))
            else:
                self.kc[i] = np.zeros((s.ctx, s.n_kv, s.head_dim))
                self.vc[i] = np.zeros((s.ctx, s.n_kv, s.head_dim))

    def rms(self, x, w):
        return x / np.sqrt(np.mean(x * x) + self.s.eps) * w

    def rope(self, v, pos):
        half = self.rd // 2
        c, sn = self.cos[pos], self.sin[pos]
        x1, x2 = v[..., :half].copy(), v[..., half:2 * half].copy()
        v[..., :half] = x1 * c - x2 * sn
        v[..., half:2 * half] = x1 * sn + x2 * c
        return v

    def gdn(self, i, x):
        s, W, p = self.s, self.W, f"blk.{i}."
        qkv = W[p + "attn_qkv.weight"] @ x
        z = W[p + "attn_gate.weight"] @ x
        self.conv[i] = np.roll(self.conv[i], -1, axis=0)
        self.conv[i][-1] = qkv
        cw = W[p + "ssm_conv1d.weight"]                      # (C, K)
        v = (self.conv[i].T * cw).sum(1)
        xc = v / (1 + np.exp(-v))
        nk, nv, dk, dv = s.ssm_nk, s.ssm_nv, s.ssm_dk, s.ssm_dv
        q = xc[:nk * dk].reshape(nk, dk)
        k = xc[nk * dk:2 * nk * dk].reshape(nk, dk)
        vv = xc[2 * nk * dk:].reshape(nv, dv)
        al = W[p + "ssm_alpha.weight"] @ x
        be = W[p + "ssm_beta.weight"] @ x
        y = np.zeros((nv, dv))
        for h in range(nv):
            g = h % nk
            qn = q[g] / (np.linalg.norm(q[g]) + 1e-6) / np.sqrt(dk)
            kn = k[g] / (np.linalg.norm(k[g]) + 1e-6)
            a = np.clip(al[h] + W[p + "ssm_dt.bias"][h], -20, 20)
            decay = np.exp(W[p + "ssm_a"][h] * np.log1p(np.exp(a)))
            b = 1 / (1 + np.exp(-np.clip(be[h], -20, 20)))
            S = self.S[i][h] * decay
            d = b * (vv[h] - S @ kn)
            S = S + np.outer(d, kn)
            self.S[i][h] = S
            y[h] = self.rms(S @ qn, W[p + "ssm_norm.weight"])
        y = y.reshape(-1) * z / (1 + np.exp(-z))
        return W[p + "ssm_out.weight"] @ y

    def attn(self, i, x, pos):
        s, W, p = self.s, self.W, f"blk.{i}."
        hd = s.head_dim
        qg = (W[p + "attn_q.weight"] @ x).reshape(s.n_heads, 2, hd)
        q, gate = qg[:, 0].copy(), qg[:, 1]
        k = (W[p + "attn_k.weight"] @ x).reshape(s.n_kv, hd)
        v = (W[p + "attn_v.weight"] @ x).reshape(s.n_kv, hd)
        q = np.stack([self.rope(self.rms(q[h], W[p + "attn_q_norm.weight"]), pos) for h in range(s.n_heads)])
        k = np.stack([self.rope(self.rms(k[h], W[p + "attn_k_norm.weight"]), pos) for h in range(s.n_kv)])
        self.kc[i][pos] = k
        self.vc[i][pos] = v
        o = np.zeros((s.n_heads, hd))
        g = s.n_heads // s.n_kv
        for h in range(s.n_heads):
            K = self.kc[i][:pos + 1, h // g]
            V = self.vc[i][:pos + 1, h // g]
            sc = K @ q[h] / np.sqrt(hd)
            pr = np.exp(sc - sc.max())
            o[h] = (pr / pr.sum()) @ V
        o = o * (1 / (1 + np.exp(-gate)))
        return W[p + "attn_output.weight"] @ o.reshape(-1)

    def layer(self, i, x, pos):
        W, p = self.W, f"blk.{i}."
        xn = self.rms(x, W[p + "attn_norm.weight"])
        r = self.gdn(i, xn) if f"blk.{i}.ssm_a" in W else self.attn(i, xn, pos)
        x = x + r
        xn = self.rms(x, W[p + "post_attention_norm.weight"])
        g = W[p + "ffn_gate.weight"] @ xn
        u = W[p + "ffn_up.weight"] @ xn
        return x + W[p + "ffn_down.weight"] @ (g / (1 + np.exp(-g)) * u)

    def forward(self, toks, pos):
        for t, tok in enumerate(toks):
            x = self.W["token_embd.weight"][tok].copy()
            for i in range(self.s.layers):
                x = self.layer(i, x, pos + t)
        xn = self.rms(x, self.W["output_norm.weight"])
        logits = self.W["token_embd.weight"] @ xn
        return int(np.argmax(logits)), logits
