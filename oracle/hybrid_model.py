"""CPU restatement of the hybrid decoder -- TEST INFRASTRUCTURE.

Only tests/ (and bench.py's CPU leg) may use this module.  It is the checker
for exl3_b200.hybrid.HybridEngine, never part of the product path.

The reference tree does not contain the model graph (upstream llama.cpp runs
attention and the gated delta net; patches/llama-exl3.patch:175-183 only
routes them), so this restates the published math in numpy, one sequence at
a time, token by token:

  * gated delta rule (Yang et al., "Gated Delta Networks", ICLR 2025):
    S_t = a_t S_{t-1} (I - b_t k_t k_t^T) + b_t v_t k_t^T, o_t = S_t q_t, with
    a_t = exp(-exp(A_log) softplus(x.W_a + dt_bias)), b_t = sigmoid(x.W_b);
    causal depthwise conv (width 4) + SiLU on q, k, v; L2-normalised q, k,
    q scaled by 1/sqrt(d); per-head RMSNorm of o times SiLU(z);
  * full attention: per-head RMSNorm of q, k; rotary embedding on the halves
    (i, i+64) of each head; softmax(q k^T / sqrt(d)) v over the causal prefix;
    grouped queries (4 per kv head);
  * RMSNorm residual blocks, SwiGLU feed-forward, tied fp16 head.

EXL3 weights enter as the dense fp16 matrices the reference codec
reconstructs (oracle C library, bit-exact to exl3::reconstruct), so the only
model-level differences from the GPU are the packed operator's own rounding
(activations quantised inside the GEMV / fp16 in the GEMM, fp32 sums) and
summation order.  Rounding points mirror the engine: the KV cache is fp16,
everything else float32/float64 (activations enter the packed matmuls as f32).
Parity of this model with the reference's own graph is unpinned: that graph
is not in the reference tree.
"""
from __future__ import annotations

import numpy as np


def _rms(x, w, eps):
    x = np.asarray(x, np.float64)
    return x / np.sqrt(np.mean(x * x, axis=-1, keepdims=True) + eps) * w


def _silu(x):
    return x / (1.0 + np.exp(-x))


def _softplus(x):
    return x if x > 20.0 else np.log1p(np.exp(x))


class OracleHybrid:
    """Token-by-token reference of exl3_b200.hybrid for one sequence at a time."""

    def __init__(self, weights, oracle):
        self.w = weights
        self.cfg = cfg = weights.cfg
        self.dense = []
        for lw in weights.layers:
            mats = {}
            for name, m in lw.mats.items():
                W = oracle.reconstruct(m.trellis, m.suh, m.svh, m.k, m.n, m.bits).view(np.float16)
                mats[name] = W.astype(np.float64)
            if lw.kind == "gdn":
                mats["qkvz"] = np.concatenate([mats["q"], mats["k"], mats["v"], mats["z"]], axis=1)
            mats["gu"] = np.concatenate([mats["gate"], mats["up"]], axis=1)
            self.dense.append(mats)
        self.E = weights.embed.astype(np.float64)
        self.inv_freq = cfg.inv_freq  # float32

    def new_sequence(self):
        cfg = self.cfg
        D = cfg.heads * cfg.head_dim
        st = []
        for lw in self.w.layers:
            if lw.kind == "full":
                st.append({"K": [], "V": []})
            else:
                st.append({"S": np.zeros((cfg.heads, cfg.head_dim, cfg.head_dim), np.float64),
                           "conv": np.zeros((3 * D, 3), np.float64)})
        return st

    def _mm(self, x, W):
        return (np.asarray(x, np.float64) @ W).astype(np.float32)

    def step(self, seq, token: int, pos: int):
        """Feed one token at position pos; returns the f32 logits of the next token."""
        cfg = self.cfg
        H, D, HD = cfg.hidden, cfg.heads * cfg.head_dim, cfg.head_dim
        KVD = cfg.kv_heads * HD
        h = self.E[token].astype(np.float32)  # exact: fp16 values
        delta = None
        for li, lw in enumerate(self.w.layers):
            W = self.dense[li]
            if delta is not None:
                h = (h + delta).astype(np.float32)
            xn = _rms(h, lw.in_norm, cfg.eps).astype(np.float32)
            if lw.kind == "full":
                q = self._mm(xn, W["q"]).reshape(cfg.heads, HD)
                k = self._mm(xn, W["k"]).reshape(cfg.kv_heads, HD)
                v = self._mm(xn, W["v"]).reshape(cfg.kv_heads, HD)
                q = _rms(q, lw.extra["q_norm"], cfg.eps)
                k = _rms(k, lw.extra["k_norm"], cfg.eps)
                ang = (np.float32(pos) * self.inv_freq).astype(np.float64)
                cs, sn = np.cos(ang), np.sin(ang)

                def rope(x):
                    a, b = x[..., :HD // 2], x[..., HD // 2:]
                    return np.concatenate([a * cs - b * sn, b * cs + a * sn], axis=-1)

                q = rope(q).astype(np.float32)
                k = rope(k).astype(np.float16)
                seq[li]["K"].append(k)
                seq[li]["V"].append(v.astype(np.float16))
                K = np.stack(seq[li]["K"]).astype(np.float64)  # [T, kvh, HD]
                V = np.stack(seq[li]["V"]).astype(np.float64)
                out = np.empty((cfg.heads, HD))
                g = cfg.heads // cfg.kv_heads
                for hq in range(cfg.heads):
                    s = K[:, hq // g, :] @ q[hq].astype(np.float64) / np.sqrt(HD)
                    p = np.exp(s - s.max())
                    out[hq] = (p / p.sum()) @ V[:, hq // g, :]
                mix = out.reshape(D).astype(np.float32)
            else:
                ex = lw.extra
                proj = self._mm(xn, W["qkvz"])
                x_qkv = proj[:3 * D].astype(np.float64)
                z = proj[3 * D:].astype(np.float64).reshape(cfg.heads, HD)
                cw = ex["conv_w"].astype(np.float64)
                cst = seq[li]["conv"]
                conv = cst[:, 0] * cw[:, 0] + cst[:, 1] * cw[:, 1] + cst[:, 2] * cw[:, 2] + x_qkv * cw[:, 3]
                cst[:, 0], cst[:, 1], cst[:, 2] = cst[:, 1].copy(), cst[:, 2].copy(), x_qkv
                c = _silu(conv)
                qh = c[:D].reshape(cfg.heads, HD)
                kh = c[D:2 * D].reshape(cfg.heads, HD)
                vh = c[2 * D:].reshape(cfg.heads, HD)
                qh = qh / np.sqrt(np.sum(qh * qh, axis=1, keepdims=True) + 1e-6) / np.sqrt(HD)
                kh = kh / np.sqrt(np.sum(kh * kh, axis=1, keepdims=True) + 1e-6)
                ab = ex["wab"].astype(np.float64) @ xn.astype(np.float64)
                out = np.empty((cfg.heads, HD))
                S = seq[li]["S"]
                for hh in range(cfg.heads):
                    alpha = np.exp(-np.exp(float(ex["A_log"][hh])) * _softplus(ab[hh] + float(ex["dt_bias"][hh])))
                    beta = 1.0 / (1.0 + np.exp(-ab[cfg.heads + hh]))
                    Sh = S[hh]  # [k, v]
                    a_v = kh[hh] @ Sh
                    c_v = qh[hh] @ Sh
                    u = beta * (vh[hh] - alpha * a_v)
                    o = alpha * c_v + (kh[hh] @ qh[hh]) * u
                    S[hh] = alpha * Sh + np.outer(kh[hh], u)
                    on = o / np.sqrt(np.mean(o * o) + cfg.eps)
                    out[hh] = on * ex["gnorm"] * _silu(z[hh])
                mix = out.reshape(D).astype(np.float32)
            o = self._mm(mix, W["o"])
            h = (h + o).astype(np.float32)
            xn = _rms(h, lw.post_norm, cfg.eps).astype(np.float32)
            gu = self._mm(xn, W["gu"]).astype(np.float64)
            act = (_silu(gu[:cfg.ffn]) * gu[cfg.ffn:]).astype(np.float32)
            delta = self._mm(act, W["down"])
        h = (h + delta).astype(np.float32)
        xn = _rms(h, self.w.final_norm, cfg.eps).astype(np.float32)
        return (self.E @ xn.astype(np.float64)).astype(np.float32)


class StreamingOracleHybrid:
    """The same model for a whole token sequence at once (teacher forcing), layer by layer, with
    nothing dense kept: every EXL3 product runs through the oracle's restatement of the reference
    operator (ggml_exl3_mul_mat, src/exl3-ggml.cpp:51-92) on the matrix's runtime records, so the
    memory stays at one layer's records however large the model.  Mixers advance position by
    position exactly as OracleHybrid.step does.  Returns every layer's residual stream and the
    logits of every position (float32)."""

    def __init__(self, weights, oracle, nth: int = 8):
        self.w = weights
        self.cfg = weights.cfg
        self.orc = oracle
        self.nth = nth

    def _mm(self, x, m):
        from exl3_b200.format import pack_records

        rec = pack_records(m.trellis, m.suh, m.svh, m.bits)
        return self.orc.mul_mat(rec, m.bits, m.k, m.n, np.ascontiguousarray(x, np.float32), nth=self.nth)

    def run(self, tokens):
        cfg = self.cfg
        H, D, HD = cfg.hidden, cfg.heads * cfg.head_dim, cfg.head_dim
        T = len(tokens)
        E = self.w.embed
        h = E[np.asarray(tokens)].astype(np.float32)
        residuals = []
        inv_freq = cfg.inv_freq
        for lw in self.w.layers:
            M = lw.mats
            xn = _rms(h, lw.in_norm, cfg.eps).astype(np.float32)
            mix = np.empty((T, D), np.float32)
            if lw.kind == "full":
                q = self._mm(xn, M["q"]).reshape(T, cfg.heads, HD)
                k = self._mm(xn, M["k"]).reshape(T, cfg.kv_heads, HD)
                v = self._mm(xn, M["v"]).reshape(T, cfg.kv_heads, HD)
                q = _rms(q, lw.extra["q_norm"], cfg.eps)
                k = _rms(k, lw.extra["k_norm"], cfg.eps)
                ang = (np.arange(T, dtype=np.float32)[:, None] * inv_freq[None, :]).astype(np.float64)
                cs, sn = np.cos(ang)[:, None, :], np.sin(ang)[:, None, :]

                def rope(x):
                    a, b = x[..., :HD // 2], x[..., HD // 2:]
                    return np.concatenate([a * cs - b * sn, b * cs + a * sn], axis=-1)

                q = rope(q).astype(np.float32).astype(np.float64)
                K = rope(k).astype(np.float16).astype(np.float64)
                V = v.astype(np.float16).astype(np.float64)
                g = cfg.heads // cfg.kv_heads
                for t in range(T):
                    out = np.empty((cfg.heads, HD))
                    for hq in range(cfg.heads):
                        sc = K[:t + 1, hq // g, :] @ q[t, hq] / np.sqrt(HD)
                        pr = np.exp(sc - sc.max())
                        out[hq] = (pr / pr.sum()) @ V[:t + 1, hq // g, :]
                    mix[t] = out.reshape(D).astype(np.float32)
            else:
                ex = lw.extra
                proj = np.concatenate([self._mm(xn, M[nm]) for nm in ("q", "k", "v", "z")], axis=1)
                cw = ex["conv_w"].astype(np.float64)
                cst = np.zeros((3 * D, 3), np.float64)
                S = np.zeros((cfg.heads, HD, HD), np.float64)
                ab_all = (ex["wab"].astype(np.float64) @ xn.astype(np.float64).T).T  # [T, 2 heads]
                for t in range(T):
                    x_qkv = proj[t, :3 * D].astype(np.float64)
                    z = proj[t, 3 * D:].astype(np.float64).reshape(cfg.heads, HD)
                    conv = cst[:, 0] * cw[:, 0] + cst[:, 1] * cw[:, 1] + cst[:, 2] * cw[:, 2] + x_qkv * cw[:, 3]
                    cst[:, 0], cst[:, 1], cst[:, 2] = cst[:, 1].copy(), cst[:, 2].copy(), x_qkv
                    c = _silu(conv)
                    qh = c[:D].reshape(cfg.heads, HD)
                    kh = c[D:2 * D].reshape(cfg.heads, HD)
                    vh = c[2 * D:].reshape(cfg.heads, HD)
                    qh = qh / np.sqrt(np.sum(qh * qh, axis=1, keepdims=True) + 1e-6) / np.sqrt(HD)
                    kh = kh / np.sqrt(np.sum(kh * kh, axis=1, keepdims=True) + 1e-6)
                    ab = ab_all[t]
                    out = np.empty((cfg.heads, HD))
                    for hh in range(cfg.heads):
                        alpha = np.exp(-np.exp(float(ex["A_log"][hh])) * _softplus(ab[hh] + float(ex["dt_bias"][hh])))
                        beta = 1.0 / (1.0 + np.exp(-ab[cfg.heads + hh]))
                        Sh = S[hh]
                        a_v = kh[hh] @ Sh
                        c_v = qh[hh] @ Sh
                        u = beta * (vh[hh] - alpha * a_v)
                        o = alpha * c_v + (kh[hh] @ qh[hh]) * u
                        S[hh] = alpha * Sh + np.outer(kh[hh], u)
                        on = o / np.sqrt(np.mean(o * o) + cfg.eps)
                        out[hh] = on * ex["gnorm"] * _silu(z[hh])
                    mix[t] = out.reshape(D).astype(np.float32)
            h = (h + self._mm(mix, M["o"])).astype(np.float32)
            xn = _rms(h, lw.post_norm, cfg.eps).astype(np.float32)
            gu = np.concatenate([self._mm(xn, M["gate"]), self._mm(xn, M["up"])], axis=1).astype(np.float64)
            act = (_silu(gu[:, :cfg.ffn]) * gu[:, cfg.ffn:]).astype(np.float32)
            h = (h + self._mm(act, M["down"])).astype(np.float32)
            residuals.append(h.copy())
        xn = _rms(h, self.w.final_norm, cfg.eps).astype(np.float32).astype(np.float64)
        logits = np.empty((T, cfg.vocab), np.float32)
        for r0 in range(0, cfg.vocab, 16384):  # bounded temporaries over the tied head
            r1 = min(cfg.vocab, r0 + 16384)
            logits[:, r0:r1] = (xn @ E[r0:r1].astype(np.float64).T).astype(np.float32)
        return residuals, logits

