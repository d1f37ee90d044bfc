"""Hybrid decoder on the EXL3 operator: a Qwen3.5-style 3:1 gated-delta-rule /
full-attention stack whose linear layers are packed EXL3 weights.

What runs on the GPU, per scheduler step of R packed rows (ragged: decode
tokens and prefill chunks of several sequences together):

    h = embed(tokens)                                     exl3cu_hyb_embed
    per layer:
        xn = rmsnorm(h += previous delta)                 exl3cu_hyb_rmsnorm
        full attention:  [q|k|v] = xn . W_{q,k,v}         exl3cu_mul_mat_batch (EXL3)
                         q/k norm, RoPE, KV append        exl3cu_hyb_attn_prep
                         a = attn(q, K, V)                exl3cu_hyb_attn
                         (decode steps: both in one launch, exl3cu_hyb_attn_decode)
        delta rule:      [q|k|v|z] = xn . W_{q,k,v,z}     exl3cu_mul_mat_batch (EXL3)
                         a = gdn(...)                     exl3cu_hyb_gdn (conv, gates, state update, gated norm)
        o = a . W_o                                       exl3cu_mul_mat (EXL3)
        xn = rmsnorm(h += o)
        [g|u] = xn . W_{gate,up}; d = swiglu . W_down     exl3cu_mul_mat_batch, exl3cu_hyb_swiglu, exl3cu_mul_mat
    xn = rmsnorm(h += d); token = argmax(xn . E^T)        exl3cu_hyb_head (tied fp16 embedding)

Steps of <= 8 rows fold the glue into the operator (exl3cu_mul_mat_batch_ex:
RMSNorm and SwiGLU on load, residual adds in the epilogue) and the final
RMSNorm into the head, which then is one launch; a layer is 4 operator
launches plus its mixer.

The model is synthetic (no checkpoints offline): random-init parameters with
the stated shapes; each linear layer is an EXL3 matrix with a seeded random
trellis bitstream, +-1 input signs and U(0.01, 0.03) output scales (the same
recipe as the operator benchmarks), i.e. random weights in EXL3 form.
"""
from __future__ import annotations

import ctypes
import os
from dataclasses import dataclass, field

import numpy as np

from ._lib import check, lib


@dataclass
class HybridConfig:
    layers: int = 28
    hidden: int = 2048
    ffn: int = 6144
    vocab: int = 151936
    heads: int = 16          # q heads and delta-rule heads, dim 128
    kv_heads: int = 4
    head_dim: int = 128
    full_every: int = 4      # layer i is full attention when i % full_every == full_every - 1 (3:1)
    rope_theta: float = 10_000_000.0
    eps: float = 1e-6
    bits: int = 4

    def is_full(self, i: int) -> bool:
        return i % self.full_every == self.full_every - 1

    @property
    def inv_freq(self) -> np.ndarray:
        i = np.arange(self.head_dim // 2, dtype=np.float64)
        return (1.0 / self.rope_theta ** (2.0 * i / self.head_dim)).astype(np.float32)

    def matrix_shapes(self, i: int) -> dict:
        H, F, D = self.hidden, self.ffn, self.heads * self.head_dim
        KV = self.kv_heads * self.head_dim
        if self.is_full(i):
            mats = {"q": (H, D), "k": (H, KV), "v": (H, KV), "o": (D, H)}
        else:
            mats = {"q": (H, D), "k": (H, D), "v": (H, D), "z": (H, D), "o": (D, H)}
        mats.update({"gate": (H, F), "up": (H, F), "down": (F, H)})
        return mats


@dataclass
class EXL3Matrix:
    k: int
    n: int
    bits: int
    trellis: np.ndarray  # uint16 [k/16, n/16, 16*bits]
    suh: np.ndarray      # fp16 bits [k]
    svh: np.ndarray      # fp16 bits [n]


@dataclass
class LayerWeights:
    kind: str                      # "full" or "gdn"
    mats: dict
    in_norm: np.ndarray            # f32 [H]
    post_norm: np.ndarray          # f32 [H]
    extra: dict = field(default_factory=dict)


@dataclass
class HybridWeights:
    cfg: HybridConfig
    embed: np.ndarray              # fp16 [V, H] (tied head)
    final_norm: np.ndarray         # f32 [H]
    layers: list


def _exl3(rng, k, n, bits) -> EXL3Matrix:
    trellis = rng.integers(0, 65536, size=(k // 16, n // 16, 16 * bits), dtype=np.uint16)
    suh = rng.choice(np.array([-1.0, 1.0], np.float32), size=k).astype(np.float16).view(np.uint16)
    sign = rng.choice(np.array([-1.0, 1.0], np.float32), size=n)
    svh = (sign * rng.uniform(0.01, 0.03, size=n)).astype(np.float16).view(np.uint16)
    return EXL3Matrix(k, n, bits, trellis, suh, svh)


def synthetic_weights(cfg: HybridConfig, seed: int = 1234) -> HybridWeights:
    """Seeded random-init parameters (numpy PCG64), EXL3 matrices as random trellis streams."""
    rng = np.random.Generator(np.random.PCG64(seed))
    H = cfg.hidden
    emb = np.empty((cfg.vocab, H), np.float16)
    for r0 in range(0, cfg.vocab, 8192):  # bounded temporaries
        r1 = min(cfg.vocab, r0 + 8192)
        emb[r0:r1] = (rng.standard_normal((r1 - r0, H), dtype=np.float32) * 0.05).astype(np.float16)
    layers = []
    for i in range(cfg.layers):
        mats = {name: _exl3(rng, k, n, cfg.bits) for name, (k, n) in cfg.matrix_shapes(i).items()}
        in_norm = (1.0 + 0.1 * rng.standard_normal(H)).astype(np.float32)
        post_norm = (1.0 + 0.1 * rng.standard_normal(H)).astype(np.float32)
        if cfg.is_full(i):
            extra = {"q_norm": (1.0 + 0.1 * rng.standard_normal(cfg.head_dim)).astype(np.float32),
                     "k_norm": (1.0 + 0.1 * rng.standard_normal(cfg.head_dim)).astype(np.float32)}
            layers.append(LayerWeights("full", mats, in_norm, post_norm, extra))
        else:
            nh, D = cfg.heads, cfg.heads * cfg.head_dim
            extra = {"wab": (rng.standard_normal((2 * nh, H), dtype=np.float32) * 0.02).astype(np.float16),
                     "conv_w": (rng.standard_normal((3 * D, 4), dtype=np.float32) * 0.5).astype(np.float32),
                     "A_log": rng.uniform(-1.0, 1.0, nh).astype(np.float32),
                     "dt_bias": (0.5 * rng.standard_normal(nh)).astype(np.float32),
                     "gnorm": (1.0 + 0.1 * rng.standard_normal(cfg.head_dim)).astype(np.float32)}
            layers.append(LayerWeights("gdn", mats, in_norm, post_norm, extra))
    final_norm = (1.0 + 0.1 * rng.standard_normal(H)).astype(np.float32)
    return HybridWeights(cfg, emb, final_norm, layers)


# ---------------------------------------------------------------------------------------------

def _vp(t) -> ctypes.c_void_p:
    return ctypes.c_void_p(t.data_ptr())


def _declare(L):
    if getattr(L, "_hyb_declared", False):
        return
    I, F, S, P = ctypes.c_int, ctypes.c_float, ctypes.c_size_t, ctypes.c_void_p
    L.exl3cu_hyb_embed.argtypes = [P, I, P, I, I, P, P, P]
    L.exl3cu_hyb_rmsnorm.argtypes = [P, P, I, P, F, I, I, P, P]
    L.exl3cu_hyb_swiglu.argtypes = [P, I, I, P, P]
    L.exl3cu_hyb_attn_prep.argtypes = [P, I, P, P, P, P, P, P, F, P, P, I, I, P, P]
    L.exl3cu_hyb_attn.argtypes = [P, I, P, P, P, P, P, I, I, F, I, P, S, P, P, P]
    L.exl3cu_hyb_attn_decode.argtypes = [P, I, P, P, P, P, P, P, F, P, P, I, I, F, I, P, S, P, P, P]
    L.exl3cu_hyb_attn_scratch_bytes.restype = S
    L.exl3cu_hyb_attn_scratch_bytes.argtypes = [I, I]
    L.exl3cu_hyb_status.argtypes = [I, ctypes.POINTER(ctypes.c_uint)]
    L.exl3cu_hyb_gdn_smem_bytes.restype = S
    L.exl3cu_hyb_gdn.argtypes = [P, P, P, P, I, P, P, P, P, P, F, P, P, P, I, I, P, P]
    L.exl3cu_hyb_head.argtypes = [P, P, I, I, P, F, P, I, P, P, P, P]
    L.exl3cu_hyb_head_feedback.argtypes = [P, P, I, I, P, F, P, I, P, P, P, P, P, P, S, P]
    for n in ("exl3cu_hyb_embed", "exl3cu_hyb_rmsnorm", "exl3cu_hyb_swiglu", "exl3cu_hyb_attn_prep",
              "exl3cu_hyb_attn", "exl3cu_hyb_attn_decode", "exl3cu_hyb_gdn", "exl3cu_hyb_head",
              "exl3cu_hyb_head_feedback", "exl3cu_hyb_status"):
        getattr(L, n).restype = ctypes.c_int
    L._hyb_declared = True


def attn_splits(rows: int) -> int:
    """Position splits per (row, head) of the attention kernel: many for decode steps (few rows, long
    contexts), one when the rows alone fill the GPU."""
    return 32 if rows <= 1 else (16 if rows <= 2 else (8 if rows <= 8 else (2 if rows <= 64 else 1)))


def one_row_each(row_offsets) -> bool:
    """True when every sequence of a step has exactly one row (a decode step): then a row attends only
    to cached positions and its own, and the fused attention (exl3cu_hyb_attn_decode) is valid."""
    offs = np.asarray(row_offsets, np.int64)
    return offs.size > 1 and bool(np.all(np.diff(offs) == 1))


class StepMeta:
    """Device int32 row metadata of one step, filled from one pinned host buffer by one copy:
    [tokens R | row_seq R | row_pos R | row_offsets n_seq+1 | seq_slot n_seq | logit_rows nout]."""

    def __init__(self, torch, device, max_rows: int, max_seq: int, max_out: int):
        self.cap = (max_rows, max_seq, max_out)
        n = 3 * max_rows + 2 * max_seq + 1 + max_out
        self.host = torch.zeros(n, dtype=torch.int32, pin_memory=True)
        self.dev = torch.zeros(n, dtype=torch.int32, device=device)
        R, Q, O = max_rows, max_seq, max_out
        self.off = {"tokens": 0, "row_seq": R, "row_pos": 2 * R, "row_offsets": 3 * R, "seq_slot": 3 * R + Q + 1,
                    "logit_rows": 3 * R + 2 * Q + 1}
        self.len = {"tokens": R, "row_seq": R, "row_pos": R, "row_offsets": Q + 1, "seq_slot": Q, "logit_rows": O}
        self.one_row_each = False  # every sequence of the filled step has exactly one row (a decode step)

    def view(self, name):
        o = self.off[name]
        return self.dev[o:o + self.len[name]]

    def fill(self, tokens, row_seq, row_pos, row_offsets, seq_slot, logit_rows):
        h = self.host.numpy()
        for name, arr in (("tokens", tokens), ("row_seq", row_seq), ("row_pos", row_pos),
                          ("row_offsets", row_offsets), ("seq_slot", seq_slot), ("logit_rows", logit_rows)):
            a = np.asarray(arr, np.int32)
            if a.size > self.len[name]:
                raise ValueError(f"{name}: {a.size} entries, capacity {self.len[name]}")
            h[self.off[name]:self.off[name] + a.size] = a
        self.one_row_each = one_row_each(row_offsets)

    def upload(self, stream):
        self.dev.copy_(self.host, non_blocking=True)


class HybridEngine:
    """The hybrid decoder resident on one GPU: EXL3 weights, fp16 embedding/head, fp16 KV caches and
    fp32 delta-rule states for `slots` concurrent sequences of up to `max_len` positions."""

    def __init__(self, weights: HybridWeights, device: int = 0, slots: int = 8, max_len: int = 1536,
                 max_rows: int = 512):
        import torch

        from .ops import Exl3Weight

        self.torch = torch
        self.cfg = cfg = weights.cfg
        self.device = device
        dev = f"cuda:{device}"
        self.dev = dev
        self.slots, self.max_len, self.max_rows = slots, max_len, max_rows
        L = lib()
        _declare(L)
        self.L = L
        t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)  # noqa: E731
        self.embed = t(weights.embed)
        self.final_norm = t(weights.final_norm)
        self.inv_freq = t(cfg.inv_freq)
        self.layers = []
        for lw in weights.layers:
            mats = {name: Exl3Weight.from_trellis(m.trellis, m.suh, m.svh, device=device)
                    for name, m in lw.mats.items()}
            d = {"kind": lw.kind, "mats": mats, "in_norm": t(lw.in_norm), "post_norm": t(lw.post_norm)}
            d.update({k: t(v) for k, v in lw.extra.items()})
            self.layers.append(d)
        H, F, D = cfg.hidden, cfg.ffn, cfg.heads * cfg.head_dim
        KV = cfg.kv_heads * cfg.head_dim
        R = max_rows
        f32, f16 = torch.float32, torch.float16
        self.h = torch.zeros((R, H), dtype=f32, device=dev)
        self.h_ss = torch.zeros((R, H // 128), dtype=f32, device=dev)  # h's sums of squares per 128-block
        self.xn = torch.zeros((R, H), dtype=f32, device=dev)
        self.proj = torch.zeros((R, 4 * D), dtype=f32, device=dev)      # [q|k|v|z] or [q|k|v]
        self.q = torch.zeros((R, D), dtype=f32, device=dev)
        self.mix = torch.zeros((R, D), dtype=f32, device=dev)           # attention / delta-rule output
        self.o = torch.zeros((R, H), dtype=f32, device=dev)
        self.gu = torch.zeros((R, 2 * F), dtype=f32, device=dev)
        self.act = torch.zeros((R, F), dtype=f32, device=dev)
        self.down = torch.zeros((R, H), dtype=f32, device=dev)
        n_full = sum(1 for d in self.layers if d["kind"] == "full")
        n_gdn = len(self.layers) - n_full
        self.kc = torch.zeros((max(n_full, 1), slots, cfg.kv_heads, max_len, cfg.head_dim), dtype=f16, device=dev)
        self.vc = torch.zeros_like(self.kc)
        self.state = torch.zeros((max(n_gdn, 1), slots, cfg.heads, cfg.head_dim, cfg.head_dim), dtype=f32,
                                 device=dev)
        self.conv = torch.zeros((max(n_gdn, 1), slots, 3 * D, 3), dtype=f32, device=dev)
        fi = gi = 0
        for d in self.layers:
            if d["kind"] == "full":
                d["cache"] = fi
                fi += 1
            else:
                d["cache"] = gi
                gi += 1
        self.meta = StepMeta(torch, dev, R, slots, 8)
        part_bytes = max(L.exl3cu_hyb_attn_scratch_bytes(r, attn_splits(r)) for r in range(1, R + 1))
        self.attn_part = torch.zeros(max(1, part_bytes // 4), dtype=f32, device=dev)
        self.attn_tickets = torch.zeros(R * cfg.heads, dtype=torch.int32, device=dev)
        self.best = torch.zeros(9, dtype=torch.int64, device=dev)  # head scratch: 8 maxima + a ticket, left zero
        self.out_tokens = torch.zeros(8, dtype=torch.int32, device=dev)
        self.KV = KV
        self._batch_args = {}
        self.fused = os.environ.get("EXL3_HYB_FUSED", "1") != "0"  # layer glue folded into the operator
        if os.environ.get("EXL3_GEMM_MIN_ROWS"):  # tuning: rows at which the operator switches to the GEMM
            check(L.exl3cu_gemm_config(int(os.environ["EXL3_GEMM_MIN_ROWS"]), 0, 0))

    # -- slot management --------------------------------------------------------------------------
    def reset_slot(self, slot: int):
        self.state[:, slot].zero_()
        self.conv[:, slot].zero_()

    # -- one step ---------------------------------------------------------------------------------
    def _mm_batch(self, names, mats, x, out_cols, rows, st, form: int = 0, nw=None, accum: bool = False,
                  x_ss=None, y_ss=None):
        """Projections sharing input x (form 0: f32 rows; 2: [gate | up] rows, SwiGLU on load; 3: residual
        rows, RMSNorm with weights nw on load, the rows' mean squares from the block sums x_ss) into
        column ranges of the given outputs, stored or (accum) added; y_ss receives the block sums of
        squares of a full-row output.

        Steps of 5..8 rows (batched decode) go to the operator as two problems of <= 4 rows per
        matrix in one grouped call: the grouped integer-tensor-core GEMV then decodes the weights of
        every matrix in one launch, which measured faster for these grouped decode shapes than one
        tensor-core GEMM launch per matrix."""
        key = (tuple(mats[nm].handle.value for nm in names), x.data_ptr(), tuple(o.data_ptr() for o in out_cols),
               rows, form, nw.data_ptr() if nw is not None else 0, accum,
               x_ss.data_ptr() if x_ss is not None else 0, y_ss.data_ptr() if y_ss is not None else 0)
        args = self._batch_args.get(key)
        if args is None:
            pieces = [(0, rows)] if not 5 <= rows <= 8 else [(0, 4), (4, rows - 4)]
            ws, xs, rs, ys, yst, xss, yss = [], [], [], [], [], [], []
            for nm, o in zip(names, out_cols):
                for r0, nr in pieces:
                    ws.append(mats[nm].handle.value)
                    xs.append(x.data_ptr() + r0 * x.stride(0) * x.element_size())
                    rs.append(nr)
                    ys.append(o.data_ptr() + r0 * o.stride(0) * o.element_size())
                    yst.append(o.stride(0))
                    xss.append(x_ss[r0:].data_ptr() if x_ss is not None else 0)
                    yss.append(y_ss[r0:].data_ptr() if y_ss is not None else 0)
            n = len(ws)
            VP, SZ, IN = ctypes.c_void_p * n, ctypes.c_size_t * n, ctypes.c_int * n
            nws = VP(*[nw.data_ptr() if nw is not None else 0] * n)
            args = (n, VP(*ws), VP(*xs), IN(*[form] * n), SZ(*rs), SZ(*[x.stride(0)] * n), nws,
                    ctypes.c_float(self.cfg.eps), VP(*ys), SZ(*yst), IN(*[1 if accum else 0] * n),
                    VP(*xss), VP(*yss))
            self._batch_args[key] = args
        check(self.L.exl3cu_mul_mat_batch_ex(*args, st))

    def _mm(self, w, x, out, rows, st, form: int = 0, nw=None, accum: bool = False, x_ss=None, y_ss=None):
        self._mm_batch(("_one",), {"_one": w}, x, [out], rows, st, form, nw, accum, x_ss, y_ss)

    def forward(self, rows: int, n_seq: int, nout: int, stream=None, feedback=None, trace=None) -> bool:
        """Run the step whose metadata is in self.meta.dev; next tokens land in self.out_tokens[:nout].
        feedback = (next_tokens, next_pos, log, counter) asks the head to feed the tokens back on the
        device (exl3cu_hyb_head_feedback); returns whether it did (steps of <= 8 rows only).
        trace (a list, steps of more than 8 rows): receives every layer's residual stream [rows, H] as
        f32 copies, for layer-by-layer comparisons with a reference."""
        torch, cfg, L = self.torch, self.cfg, self.L
        st = ctypes.c_void_p((stream or torch.cuda.current_stream()).cuda_stream)
        H, F, D, KV = cfg.hidden, cfg.ffn, cfg.heads * cfg.head_dim, self.KV
        m = self.meta
        tokens, row_seq, row_pos = m.view("tokens"), m.view("row_seq"), m.view("row_pos")
        row_offsets, seq_slot, logit_rows = m.view("row_offsets"), m.view("seq_slot"), m.view("logit_rows")
        main = stream or torch.cuda.current_stream()
        fused = rows <= 8 and self.fused and trace is None
        check(L.exl3cu_hyb_embed(_vp(self.embed), cfg.vocab, _vp(tokens), rows, H, _vp(self.h),
                                 _vp(self.h_ss) if fused else None, st))
        scale = 1.0 / float(np.sqrt(cfg.head_dim))
        if fused:
            self._forward_fused(rows, n_seq, nout, st, scale, row_seq, row_pos, row_offsets, seq_slot, logit_rows,
                                feedback)
            return feedback is not None
        delta = None
        for li, d in enumerate(self.layers):
            mats = d["mats"]
            check(L.exl3cu_hyb_rmsnorm(_vp(self.h), _vp(delta) if delta is not None else None, H, _vp(d["in_norm"]),
                                       cfg.eps, rows, H, _vp(self.xn), st))
            if d["kind"] == "full":
                p = self.proj
                # the prep kernel reads [q|k|v] rows packed (D + 2 KV wide): a packed view of self.proj
                qkv = p.view(-1)[: self.max_rows * (D + 2 * KV)].view(self.max_rows, D + 2 * KV)
                outs = [qkv[:, 0:D], qkv[:, D:D + KV], qkv[:, D + KV:D + 2 * KV]]
                self._mm_batch(("q", "k", "v"), mats, self.xn, outs, rows, st)
                c = d["cache"]
                kc, vc = self.kc[c], self.vc[c]
                check(L.exl3cu_hyb_attn_prep(_vp(qkv), rows, _vp(row_seq), _vp(row_pos), _vp(seq_slot),
                                             _vp(d["q_norm"]), _vp(d["k_norm"]), _vp(self.inv_freq), cfg.eps,
                                             _vp(kc), _vp(vc), self.max_len, self.slots, _vp(self.q), st))
                sp = attn_splits(rows)
                check(L.exl3cu_hyb_attn(_vp(self.q), rows, _vp(row_seq), _vp(row_pos), _vp(seq_slot), _vp(kc),
                                        _vp(vc), self.max_len, self.slots, scale, sp, _vp(self.attn_part),
                                        self.attn_part.numel() * 4, _vp(self.attn_tickets), _vp(self.mix), st))
            else:
                p = self.proj
                outs = [p[:, 0:D], p[:, D:2 * D], p[:, 2 * D:3 * D], p[:, 3 * D:4 * D]]
                self._mm_batch(("q", "k", "v", "z"), mats, self.xn, outs, rows, st)
                c = d["cache"]
                check(L.exl3cu_hyb_gdn(_vp(p), _vp(self.xn), None, _vp(d["wab"]), H, _vp(d["conv_w"]), _vp(self.conv[c]),
                                       _vp(d["A_log"]), _vp(d["dt_bias"]), _vp(d["gnorm"]), cfg.eps,
                                       _vp(self.state[c]), _vp(row_offsets), _vp(seq_slot), n_seq, self.slots,
                                       _vp(self.mix), st))
            self._mm(mats["o"], self.mix, self.o, rows, st)
            check(L.exl3cu_hyb_rmsnorm(_vp(self.h), _vp(self.o), H, _vp(d["post_norm"]), cfg.eps, rows, H,
                                       _vp(self.xn), st))
            self._mm_batch(("gate", "up"), mats, self.xn, [self.gu[:, 0:F], self.gu[:, F:2 * F]], rows, st)
            check(L.exl3cu_hyb_swiglu(_vp(self.gu), rows, F, _vp(self.act), st))
            self._mm(mats["down"], self.act, self.down, rows, st)
            delta = self.down
            if trace is not None:
                with torch.cuda.stream(main):
                    trace.append((self.h[:rows] + self.down[:rows]).float().clone())
        check(L.exl3cu_hyb_rmsnorm(_vp(self.h), _vp(delta), H, _vp(self.final_norm), cfg.eps, rows, H, _vp(self.xn),
                                   st))
        check(L.exl3cu_hyb_head(_vp(self.xn), _vp(logit_rows), nout, H, None, cfg.eps, _vp(self.embed), cfg.vocab,
                                None, _vp(self.best), _vp(self.out_tokens), st))

    def _forward_fused(self, rows, n_seq, nout, st, scale, row_seq, row_pos, row_offsets, seq_slot, logit_rows,
                       feedback=None):
        """Steps of <= 8 rows: the layer glue folded into the packed operator -- RMSNorm on load for the
        projections (and inside the delta-rule gates), SwiGLU on load for the down projection, the o and
        down products added into the residual stream h -- so a layer is 4 operator launches plus its
        mixer (attention or delta rule).  The kernels that write h (the embedding, the o and down
        products) also write its sums of squares per 128-block (h_ss), from which the RMSNorm-on-load
        projections take the rows' mean squares without reading h in full."""
        cfg, L = self.cfg, self.L
        H, F, D, KV = cfg.hidden, cfg.ffn, cfg.heads * cfg.head_dim, self.KV
        for li, d in enumerate(self.layers):
            mats = d["mats"]
            if d["kind"] == "full":
                qkv = self.proj.view(-1)[: self.max_rows * (D + 2 * KV)].view(self.max_rows, D + 2 * KV)
                outs = [qkv[:, 0:D], qkv[:, D:D + KV], qkv[:, D + KV:D + 2 * KV]]
                self._mm_batch(("q", "k", "v"), mats, self.h, outs, rows, st, 3, d["in_norm"], x_ss=self.h_ss)
                c = d["cache"]
                kc, vc = self.kc[c], self.vc[c]
                sp = attn_splits(rows)
                if rows == n_seq and self.meta.one_row_each:  # decode: prep + attention in one launch
                    check(L.exl3cu_hyb_attn_decode(_vp(qkv), rows, _vp(row_seq), _vp(row_pos), _vp(seq_slot),
                                                   _vp(d["q_norm"]), _vp(d["k_norm"]), _vp(self.inv_freq), cfg.eps,
                                                   _vp(kc), _vp(vc), self.max_len, self.slots, scale, sp,
                                                   _vp(self.attn_part), self.attn_part.numel() * 4,
                                                   _vp(self.attn_tickets), _vp(self.mix), st))
                else:
                    check(L.exl3cu_hyb_attn_prep(_vp(qkv), rows, _vp(row_seq), _vp(row_pos), _vp(seq_slot),
                                                 _vp(d["q_norm"]), _vp(d["k_norm"]), _vp(self.inv_freq), cfg.eps,
                                                 _vp(kc), _vp(vc), self.max_len, self.slots, _vp(self.q), st))
                    check(L.exl3cu_hyb_attn(_vp(self.q), rows, _vp(row_seq), _vp(row_pos), _vp(seq_slot), _vp(kc),
                                            _vp(vc), self.max_len, self.slots, scale, sp, _vp(self.attn_part),
                                            self.attn_part.numel() * 4, _vp(self.attn_tickets), _vp(self.mix), st))
            else:
                p = self.proj
                outs = [p[:, 0:D], p[:, D:2 * D], p[:, 2 * D:3 * D], p[:, 3 * D:4 * D]]
                self._mm_batch(("q", "k", "v", "z"), mats, self.h, outs, rows, st, 3, d["in_norm"],
                               x_ss=self.h_ss)
                c = d["cache"]
                check(L.exl3cu_hyb_gdn(_vp(p), _vp(self.h), _vp(d["in_norm"]), _vp(d["wab"]), H, _vp(d["conv_w"]),
                                       _vp(self.conv[c]), _vp(d["A_log"]), _vp(d["dt_bias"]), _vp(d["gnorm"]),
                                       cfg.eps, _vp(self.state[c]), _vp(row_offsets), _vp(seq_slot), n_seq,
                                       self.slots, _vp(self.mix), st))
            self._mm(mats["o"], self.mix, self.h, rows, st, 0, None, True, y_ss=self.h_ss)    # h += o
            self._mm_batch(("gate", "up"), mats, self.h, [self.gu[:, 0:F], self.gu[:, F:2 * F]], rows, st, 3,
                           d["post_norm"], x_ss=self.h_ss)
            self._mm(mats["down"], self.gu, self.h, rows, st, 2, None, True, y_ss=self.h_ss)  # h += down(swiglu)
        # the final RMSNorm is applied by the head as it loads h
        if feedback is not None:
            nt, npos, log, counter = feedback
            check(L.exl3cu_hyb_head_feedback(_vp(self.h), _vp(logit_rows), nout, H, _vp(self.final_norm), cfg.eps,
                                             _vp(self.embed), cfg.vocab, _vp(self.best), _vp(self.out_tokens),
                                             _vp(nt), _vp(npos), _vp(log), _vp(counter), log.numel(), st))
        else:
            check(L.exl3cu_hyb_head(_vp(self.h), _vp(logit_rows), nout, H, _vp(self.final_norm), cfg.eps,
                                    _vp(self.embed), cfg.vocab, None, _vp(self.best), _vp(self.out_tokens), st))

    def head_logits(self, nout: int, stream=None):
        """Logits of the last step's logit rows (f32 [nout, vocab]); recomputes the head only."""
        torch, cfg = self.torch, self.cfg
        st = ctypes.c_void_p((stream or torch.cuda.current_stream()).cuda_stream)
        out = torch.empty((nout, cfg.vocab), dtype=torch.float32, device=self.dev)
        # h holds the last step's final residual stream on both forward paths
        check(self.L.exl3cu_hyb_head(_vp(self.h), _vp(self.meta.view("logit_rows")), nout, cfg.hidden,
                                     _vp(self.final_norm), cfg.eps, _vp(self.embed), cfg.vocab, _vp(out),
                                     _vp(self.best), _vp(self.out_tokens), st))
        return out

    def free(self):
        for d in self.layers:
            for w in d["mats"].values():
                w.free()
        self.layers = []


# ---------------------------------------------------------------------------------------------
# Continuous-admission scheduler

@dataclass
class Request:
    prompt: np.ndarray        # int32 token ids
    max_new: int
    slot: int = -1
    pos: int = 0              # tokens already in the caches
    generated: list = field(default_factory=list)

    @property
    def done(self) -> bool:
        return len(self.generated) >= self.max_new


def plan_step(active, waiting, slots_free, max_rows: int, chunk: int):
    """Rows of one step: every decoding request contributes its last token; the oldest prefilling
    request (admitted into a free slot when needed) contributes a chunk of its prompt.
    Returns (seqs, tokens, row_seq, row_pos, row_offsets, seq_slot, logit_rows, logit_seq)."""
    seqs, tokens, row_seq, row_pos, offsets, slots_, logit_rows, logit_seq = [], [], [], [], [0], [], [], []
    budget = max_rows
    for rq in active:
        if rq.pos >= len(rq.prompt) and not rq.done and budget > 0 and len(logit_rows) < 8:
            s = len(seqs)
            seqs.append(rq)
            tokens.append(rq.generated[-1])
            row_seq.append(s)
            row_pos.append(rq.pos)
            offsets.append(offsets[-1] + 1)
            slots_.append(rq.slot)
            logit_rows.append(len(tokens) - 1)
            logit_seq.append(rq)
            budget -= 1
    prefilling = [rq for rq in active if rq.pos < len(rq.prompt)]
    if not prefilling and waiting and slots_free:
        rq = waiting.pop(0)
        rq.slot = slots_free.pop(0)
        active.append(rq)
        prefilling = [rq]
    if prefilling and budget > 0 and len(logit_rows) < 8:
        rq = prefilling[0]
        n = min(chunk, budget, len(rq.prompt) - rq.pos)
        s = len(seqs)
        seqs.append(rq)
        for j in range(n):
            tokens.append(int(rq.prompt[rq.pos + j]))
            row_seq.append(s)
            row_pos.append(rq.pos + j)
        offsets.append(offsets[-1] + n)
        slots_.append(rq.slot)
        if rq.pos + n == len(rq.prompt):
            logit_rows.append(len(tokens) - 1)
            logit_seq.append(rq)
    return seqs, tokens, row_seq, row_pos, offsets, slots_, logit_rows, logit_seq


def run_requests(engine: HybridEngine, requests, chunk: int = 512, stream=None, graphs: dict | None = None,
                 stats: dict | None = None, multi_step: bool = True):
    """Serve `requests` to completion with continuous admission; returns (steps, rows_total).

    Pure decode steps of n sequences replay a captured step (one per n, kept in `graphs` when given,
    captured after the first eager step of that shape); steps with prefill rows run eagerly.  Every
    step copies its metadata in and its next tokens out (the host schedules the next step), except
    with multi_step, where runs of pure decode steps with no admission possible go to the device
    as one block (see below) and come back as one copy of their tokens."""
    torch = engine.torch
    stream = stream or torch.cuda.Stream(device=engine.dev)
    graphs = {} if graphs is None else graphs
    waiting = list(requests)
    active = []
    free = list(range(engine.slots))
    steps = rows_total = 0
    import time

    seen = graphs.setdefault("seen", set())
    while waiting or active:
        t0 = time.perf_counter()
        # Multi-step decoding: when every running request is decoding and nothing can be admitted,
        # replay a captured step with device-side token feedback K times (K = the fewest tokens a
        # running request still needs) and read the K x n tokens back in one copy.
        # With requests waiting, K is the fewest tokens a running request still needs (its slot frees
        # at the block's end); with none waiting, the block runs to the longest one, the finished
        # requests' extra rows computed and discarded, so the batch keeps its shape and graph.
        n_act = len(active)
        if (multi_step and active and not (waiting and free) and n_act <= 8 and n_act in seen
                and all(rq.pos >= len(rq.prompt) and not rq.done for rq in active)):
            rem = [rq.max_new - len(rq.generated) for rq in active]
            K = min(rem) if waiting else max(rem)
            K = min(K, 256, engine.max_len - 1 - max(rq.pos for rq in active))
            if K >= 2:
                engine.meta.fill([rq.generated[-1] for rq in active], list(range(n_act)),
                                 [rq.pos for rq in active], list(range(n_act + 1)), [rq.slot for rq in active],
                                 list(range(n_act)))
                with torch.cuda.stream(stream):
                    engine.meta.upload(stream)
                dg = graphs.get(("decode", n_act))
                if dg is None:
                    stream.synchronize()
                    dg = graphs[("decode", n_act)] = DecodeGraph(engine, n_act, 256, stream, warm=False)
                with torch.cuda.stream(stream):
                    dg.reset()
                    for _ in range(K):
                        dg.replay()
                    log = dg.log[:K * n_act].to("cpu", non_blocking=False).numpy().reshape(K, n_act)
                for i, rq in enumerate(active):
                    need = rq.max_new - len(rq.generated)
                    rq.generated.extend(int(x) for x in log[:min(K, need), i])
                    rq.pos += K
                for rq in list(active):
                    if rq.done:
                        active.remove(rq)
                        free.append(rq.slot)
                steps += K
                rows_total += K * n_act
                if stats is not None:
                    stats["multistep_blocks"] = stats.get("multistep_blocks", 0) + 1
                    stats["decode_steps"] = stats.get("decode_steps", 0) + K
                    stats["decode_rows"] = stats.get("decode_rows", 0) + K * n_act
                    stats["decode_ms"] = stats.get("decode_ms", 0.0) + 1e3 * (time.perf_counter() - t0)
                continue
        seqs, tokens, row_seq, row_pos, offsets, slots_, logit_rows, logit_seq = plan_step(
            active, waiting, free, engine.max_rows, chunk)
        for s, rq in enumerate(seqs):
            if rq.pos == 0:
                engine.reset_slot(rq.slot)
        engine.meta.fill(tokens, row_seq, row_pos, offsets, slots_, logit_rows)
        n = len(tokens)
        pure_decode = n == len(seqs) == len(logit_rows)
        g = graphs.get(n) if pure_decode else None
        with torch.cuda.stream(stream):
            if g is not None:  # metadata in, step, tokens out: one captured graph
                g.replay()
                stream.synchronize()
                out = g.out_host[:len(logit_rows)]
            else:
                engine.meta.upload(stream)
                engine.forward(n, len(seqs), len(logit_rows), stream)
                out = engine.out_tokens[:len(logit_rows)].to("cpu", non_blocking=False)
        if pure_decode and n not in graphs:
            if n in seen:
                graphs[n] = _StepGraph(engine, n, stream)
            seen.add(n)
        # advance positions
        for s, rq in enumerate(seqs):
            rq.pos += offsets[s + 1] - offsets[s]
        for o, rq in enumerate(logit_seq):
            rq.generated.append(int(out[o]))
        for rq in list(active):
            if rq.done:
                active.remove(rq)
                free.append(rq.slot)
        steps += 1
        rows_total += len(tokens)
        if stats is not None:
            kind = "decode" if pure_decode else "prefill"
            stats[kind + "_steps"] = stats.get(kind + "_steps", 0) + 1
            stats[kind + "_rows"] = stats.get(kind + "_rows", 0) + n
            stats[kind + "_ms"] = stats.get(kind + "_ms", 0.0) + 1e3 * (time.perf_counter() - t0)
    return steps, rows_total


class _StepGraph:
    """A captured pure decode step of n sequences, its host I/O included: the step metadata is copied
    in from the engine's pinned host buffer and the n next tokens out into `out_host` (pinned), so a
    host-scheduled step is one graph launch and one synchronisation.  Fill engine.meta on the host,
    replay(), synchronise the stream, read out_host[:n]."""

    def __init__(self, engine, n, stream):
        torch = engine.torch
        self.out_host = torch.zeros(8, dtype=torch.int32, pin_memory=True)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph, stream=stream):
            engine.meta.upload(stream)
            engine.forward(n, n, n, stream)
            self.out_host[:n].copy_(engine.out_tokens[:n], non_blocking=True)

    def replay(self):
        self.graph.replay()


class DecodeGraph:
    """One captured decode step for `n` sequences (one row each, rows 0..n-1 in the step metadata):
    the step, then on the device: tokens[:n] <- next tokens, row_pos[:n] += 1, and the tokens appended
    to a log.  Replaying it runs greedy decoding with no host round trip; the metadata must hold a
    pure decode step for n sequences before the first replay."""

    def __init__(self, engine: HybridEngine, n: int, max_steps: int, stream=None, warm: bool = True):
        """warm=True runs the step once eagerly before capturing (one real decode step, logged first);
        warm=False requires an earlier eager step of n rows on this engine (buffers, kernel attributes)."""
        torch = engine.torch
        self.engine, self.n = engine, n
        self.stream = stream or torch.cuda.Stream(device=engine.dev)
        self.log = torch.zeros(max_steps * n, dtype=torch.int32, device=engine.dev)
        self.counter = torch.zeros(1, dtype=torch.int64, device=engine.dev)
        self.ar = torch.arange(n, dtype=torch.int64, device=engine.dev)
        self.max_steps = max_steps
        m = engine.meta
        self._tok, self._pos = m.view("tokens")[:n], m.view("row_pos")[:n]
        if warm:
            with torch.cuda.stream(self.stream):
                self._body()
        self.stream.synchronize()
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph, stream=self.stream):
            self._body()

    def _body(self):
        e, n = self.engine, self.n
        if e.forward(n, n, n, self.stream, feedback=(self._tok, self._pos, self.log, self.counter)):
            return  # the head kernel fed the tokens back (same effect as the steps below)
        self._tok.copy_(e.out_tokens[:n])
        self._pos.add_(1)
        idx = (self.counter * n + self.ar).clamp_(max=self.log.numel() - 1)
        self.log.scatter_(0, idx, e.out_tokens[:n])
        self.counter.add_(1)

    def reset(self):
        self.counter.zero_()

    def replay(self):
        self.graph.replay()


def main(argv=None) -> int:
    """Run the synthetic decoder for a few eager steps: `requests` sequences prefilled with seeded
    random prompts of `prompt` tokens, then `steps` greedy decode steps of one row per sequence.
    Prints the tokens and the host-timed milliseconds per decode step.  Eager launches (no CUDA
    graph) keep every kernel visible to a profiler's launch list."""
    import argparse
    import time

    import torch

    ap = argparse.ArgumentParser(prog="python -m exl3_b200.hybrid")
    ap.add_argument("--layers", type=int, default=28)
    ap.add_argument("--requests", type=int, default=1)
    ap.add_argument("--prompt", type=int, default=64)
    ap.add_argument("--steps", type=int, default=4)
    ap.add_argument("--seed", type=int, default=7)
    args = ap.parse_args(argv)
    if not 1 <= args.requests <= 8:
        ap.error("--requests must be 1..8 (one step's logit rows)")
    cfg = HybridConfig(layers=args.layers)
    eng = HybridEngine(synthetic_weights(cfg, seed=args.seed), device=0, slots=args.requests,
                       max_len=args.prompt + args.steps + 1, max_rows=max(64, args.requests))
    rng = np.random.default_rng(args.seed)
    tok = []
    for sq in range(args.requests):
        eng.reset_slot(sq)
        prompt = rng.integers(0, cfg.vocab, args.prompt).astype(np.int32)
        for c0 in range(0, args.prompt, 64):
            c = min(64, args.prompt - c0)
            eng.meta.fill(prompt[c0:c0 + c], np.zeros(c), np.arange(c0, c0 + c), [0, c], [sq], [c - 1])
            eng.meta.upload(None)
            eng.forward(c, 1, 1)
        tok.append(int(eng.out_tokens[0]))
    n, pos, out = args.requests, args.prompt, []
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        eng.meta.fill(tok, np.arange(n), [pos] * n, np.arange(n + 1), np.arange(n), np.arange(n))
        eng.meta.upload(None)
        eng.forward(n, n, n)
        tok = [int(v) for v in eng.out_tokens[:n].cpu().numpy()]
        out.append(tok)
        pos += 1
    ms = (time.perf_counter() - t0) * 1000 / max(1, args.steps)
    print(f"tokens {out}\n{ms:.3f} ms per eager decode step ({n} rows, {args.layers} layers)")
    eng.free()
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
