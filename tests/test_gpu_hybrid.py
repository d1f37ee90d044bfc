"""The hybrid decoder (exl3_b200.hybrid) against its CPU restatement
(oracle/hybrid_model.py) on a reduced configuration: 4 layers (3 delta-rule,
1 full attention), hidden 2048, 16 heads of 128, vocab 2048, EXL3 4 bpw.

Tolerances (written here): next-token logits within max|dl| / max|l| <= 5e-3
of the oracle at every step; greedy tokens identical at every step, except
where the oracle's top two logits are closer than 2e-3 of max|l| (a tie at the
operator's rounding level), where either choice passes and both continue from
the GPU's token (teacher forcing).
"""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

LOGIT_TOL = 5e-3
TIE_TOL = 2e-3


@pytest.fixture(scope="module")
def model(cuda_lib, oracle):
    from exl3_b200.hybrid import HybridConfig, HybridEngine, synthetic_weights
    from oracle.hybrid_model import OracleHybrid

    cfg = HybridConfig(layers=4, hidden=2048, ffn=1024, vocab=2048)
    w = synthetic_weights(cfg, seed=99)
    eng = HybridEngine(w, device=0, slots=3, max_len=160, max_rows=64)
    return eng, OracleHybrid(w, oracle)


def _check_step(gpu_logits, gpu_token, ref_logits, where, stats):
    scale = float(np.max(np.abs(ref_logits)))
    err = float(np.max(np.abs(gpu_logits - ref_logits))) / scale
    stats["max_err"] = max(stats.get("max_err", 0.0), err)
    assert err <= LOGIT_TOL, (where, err)
    ref_tok = int(np.argmax(ref_logits))
    if gpu_token != ref_tok:
        gap = float(ref_logits[ref_tok] - ref_logits[gpu_token]) / scale
        assert gap <= TIE_TOL, (where, gpu_token, ref_tok, gap)
        stats["ties"] = stats.get("ties", 0) + 1
    assert gpu_token == int(np.argmax(gpu_logits)), where  # fused argmax = argmax of the logits


def test_single_sequence_64_greedy_steps(model):
    eng, ref = model
    rng = np.random.default_rng(3)
    prompt = rng.integers(0, eng.cfg.vocab, 12).astype(np.int32)
    slot = 0
    eng.reset_slot(slot)
    seq = ref.new_sequence()
    for p, t in enumerate(prompt):
        ref_logits = ref.step(seq, int(t), p)
    n = len(prompt)
    eng.meta.fill(prompt, np.zeros(n), np.arange(n), [0, n], [slot], [n - 1])
    eng.meta.upload(None)
    eng.forward(n, 1, 1)
    stats = {}
    pos = n
    for step in range(64):
        gl = eng.head_logits(1)[0].cpu().numpy()
        tok = int(eng.out_tokens[0].item())
        _check_step(gl, tok, ref_logits, step, stats)
        ref_logits = ref.step(seq, tok, pos)
        eng.meta.fill([tok], [0], [pos], [0, 1], [slot], [0])
        eng.meta.upload(None)
        eng.forward(1, 1, 1)
        pos += 1
    print("single sequence:", stats)


def test_ragged_continuous_admission_matches_per_sequence_oracle(model):
    """Three requests through the scheduler (prefill chunks of 5 rows interleaved with decode rows);
    each request's tokens are replayed through the oracle on its own."""
    from exl3_b200.hybrid import Request, run_requests

    eng, ref = model
    rng = np.random.default_rng(4)
    reqs = [Request(rng.integers(0, eng.cfg.vocab, n).astype(np.int32), max_new=m)
            for n, m in ((7, 12), (13, 9), (3, 15))]
    steps, rows = run_requests(eng, reqs, chunk=5)
    assert steps > 0 and all(r.done for r in reqs)
    stats = {}
    for ri, rq in enumerate(reqs):
        seq = ref.new_sequence()
        for p, t in enumerate(rq.prompt):
            logits = ref.step(seq, int(t), p)
        pos = len(rq.prompt)
        for j, tok in enumerate(rq.generated):
            ref_tok = int(np.argmax(logits))
            if tok != ref_tok:
                scale = float(np.max(np.abs(logits)))
                gap = float(logits[ref_tok] - logits[tok]) / scale
                assert gap <= TIE_TOL, (ri, j, tok, ref_tok, gap)
                stats["ties"] = stats.get("ties", 0) + 1
            logits = ref.step(seq, tok, pos)
            pos += 1
    print("ragged:", steps, rows, stats)


def test_head_argmax_and_embedding(model):
    """The fused head: the final RMSNorm of the residual rows on load, then argmax over fp32 logits of
    the tied fp16 embedding, lowest index on ties."""
    eng, _ = model
    E = eng.embed.float().cpu().numpy()
    x = (np.random.default_rng(5).standard_normal((3, eng.cfg.hidden)) * 0.5).astype(np.float32)
    eng.h[:3].copy_(torch.from_numpy(x).cuda())
    eng.meta.fill([0], [0], [0], [0, 1], [0], [0, 1, 2])
    eng.meta.upload(None)
    lg = eng.head_logits(3).cpu().numpy()
    x64 = x.astype(np.float64)
    xn = x64 / np.sqrt(np.mean(x64 * x64, axis=1, keepdims=True) + eng.cfg.eps) * eng.final_norm.cpu().numpy()
    ref = xn @ E.T.astype(np.float64)
    assert np.max(np.abs(lg - ref)) / np.max(np.abs(ref)) < 1e-5
    assert list(eng.out_tokens[:3].cpu().numpy()) == list(np.argmax(lg, axis=1))


def test_attention_splits_agree(model):
    """The split (flash-decoding) attention against the single-CTA form on the same cache, rows at
    several positions; then the split scratch's tickets are back at zero."""
    import ctypes

    from exl3_b200.hybrid import _vp

    eng, _ = model
    L = eng.L
    c = 0
    g = torch.Generator(device="cuda").manual_seed(11)
    eng.kc[c].copy_(torch.randn(eng.kc[c].shape, generator=g, device="cuda").half())
    eng.vc[c].copy_(torch.randn(eng.vc[c].shape, generator=g, device="cuda").half())
    rows = 5
    q = torch.randn((rows, 16 * 128), generator=g, device="cuda")
    pos = [0, 3, 31, 100, 159]
    eng.meta.fill([0] * rows, [0, 1, 2, 0, 1], pos, [0, 1, 2, 3], [0, 1, 2], [0])
    eng.meta.upload(None)
    m = eng.meta
    outs = []
    for sp in (1, 2, 8, 16):
        o = torch.zeros((rows, 16 * 128), dtype=torch.float32, device="cuda")
        st = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
        rc = L.exl3cu_hyb_attn(_vp(q), rows, _vp(m.view("row_seq")), _vp(m.view("row_pos")), _vp(m.view("seq_slot")),
                               _vp(eng.kc[c]), _vp(eng.vc[c]), eng.max_len, eng.slots, 0.088388, sp,
                               _vp(eng.attn_part), eng.attn_part.numel() * 4, _vp(eng.attn_tickets), _vp(o), st)
        assert rc == 0
        outs.append(o.cpu().numpy())
    # fp32 reference on the host
    K = eng.kc[c].float().cpu().numpy()
    V = eng.vc[c].float().cpu().numpy()
    qq = q.cpu().numpy().reshape(rows, 16, 128)
    slots = [0, 1, 2, 0, 1]
    ref = np.zeros((rows, 16, 128))
    for r in range(rows):
        for h in range(16):
            k = K[slots[r], h // 4, :pos[r] + 1]
            s = k @ qq[r, h] * 0.088388
            p = np.exp(s - s.max())
            ref[r, h] = (p / p.sum()) @ V[slots[r], h // 4, :pos[r] + 1]
    ref = ref.reshape(rows, -1)
    for o in outs:
        assert np.max(np.abs(o - ref)) < 1e-4
    assert int(eng.attn_tickets.abs().sum()) == 0
    st = ctypes.c_uint(0)
    assert L.exl3cu_hyb_status(1, ctypes.byref(st)) == 0 and st.value == 0


def test_fused_decode_attention_matches_prep_plus_attention(model):
    """exl3cu_hyb_attn_decode (q/k norm, RoPE, KV append and attention in one launch, one row per
    sequence) against exl3cu_hyb_attn_prep + exl3cu_hyb_attn on the same inputs: outputs and both
    caches bit for bit, at positions 0, inside and at the end of the cache, for 1, 2 and 8 splits."""
    import ctypes

    from exl3_b200.hybrid import _vp

    eng, _ = model
    L = eng.L
    c = 0
    full = next(d for d in eng.layers if d["kind"] == "full")
    g = torch.Generator(device="cuda").manual_seed(12)
    k0 = torch.randn(eng.kc[c].shape, generator=g, device="cuda").half()
    v0 = torch.randn(eng.vc[c].shape, generator=g, device="cuda").half()
    rows = 3
    qkv = torch.randn((rows, (16 + 2 * 4) * 128), generator=g, device="cuda")
    pos = [0, 57, eng.max_len - 1]
    eng.meta.fill([0] * rows, [0, 1, 2], pos, [0, 1, 2, 3], [2, 0, 1], [0])
    eng.meta.upload(None)
    assert eng.meta.one_row_each
    m = eng.meta
    st = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    args_meta = (_vp(m.view("row_seq")), _vp(m.view("row_pos")), _vp(m.view("seq_slot")))
    norms = (_vp(full["q_norm"]), _vp(full["k_norm"]), _vp(eng.inv_freq), eng.cfg.eps)
    for sp in (1, 2, 8, 32):
        eng.kc[c].copy_(k0)
        eng.vc[c].copy_(v0)
        q = torch.zeros((rows, 16 * 128), dtype=torch.float32, device="cuda")
        oa = torch.zeros((rows, 16 * 128), dtype=torch.float32, device="cuda")
        assert L.exl3cu_hyb_attn_prep(_vp(qkv), rows, *args_meta, *norms, _vp(eng.kc[c]), _vp(eng.vc[c]),
                                      eng.max_len, eng.slots, _vp(q), st) == 0
        assert L.exl3cu_hyb_attn(_vp(q), rows, *args_meta, _vp(eng.kc[c]), _vp(eng.vc[c]), eng.max_len, eng.slots,
                                 0.088388, sp, _vp(eng.attn_part), eng.attn_part.numel() * 4,
                                 _vp(eng.attn_tickets), _vp(oa), st) == 0
        ka, va = eng.kc[c].clone(), eng.vc[c].clone()
        eng.kc[c].copy_(k0)
        eng.vc[c].copy_(v0)
        ob = torch.zeros((rows, 16 * 128), dtype=torch.float32, device="cuda")
        assert L.exl3cu_hyb_attn_decode(_vp(qkv), rows, *args_meta, *norms, _vp(eng.kc[c]), _vp(eng.vc[c]),
                                        eng.max_len, eng.slots, 0.088388, sp, _vp(eng.attn_part),
                                        eng.attn_part.numel() * 4, _vp(eng.attn_tickets), _vp(ob), st) == 0
        torch.cuda.synchronize()
        assert torch.equal(oa, ob), sp
        assert torch.equal(ka.view(torch.int16), eng.kc[c].view(torch.int16)), sp
        assert torch.equal(va.view(torch.int16), eng.vc[c].view(torch.int16)), sp
        assert not torch.equal(ka.view(torch.int16), k0.view(torch.int16))  # the append happened
    assert int(eng.attn_tickets.abs().sum()) == 0
