"""CPU tests of the hybrid decoder's host side: the continuous-admission step
planner and the synthetic model's shapes (no GPU)."""
import numpy as np

from exl3_b200.hybrid import HybridConfig, Request, plan_step


def test_config_is_3_to_1_with_the_stated_shapes():
    cfg = HybridConfig()
    kinds = ["full" if cfg.is_full(i) else "gdn" for i in range(cfg.layers)]
    assert kinds.count("gdn") == 21 and kinds.count("full") == 7
    assert cfg.matrix_shapes(3) == {"q": (2048, 2048), "k": (2048, 512), "v": (2048, 512), "o": (2048, 2048),
                                    "gate": (2048, 6144), "up": (2048, 6144), "down": (6144, 2048)}
    assert set(cfg.matrix_shapes(0)) == {"q", "k", "v", "z", "o", "gate", "up", "down"}


def test_plan_step_admits_one_prefill_and_packs_decode_rows():
    a = Request(np.arange(5, dtype=np.int32), max_new=3)
    b = Request(np.arange(9, dtype=np.int32), max_new=3)
    waiting, active, free = [a, b], [], [0, 1]
    seqs, tok, rs, rp, off, sl, lr, ls = plan_step(active, waiting, free, max_rows=64, chunk=4)
    assert seqs == [a] and tok == [0, 1, 2, 3] and rp == [0, 1, 2, 3] and off == [0, 4] and sl == [0]
    assert lr == [] and a.slot == 0 and free == [1] and waiting == [b]
    a.pos = 4
    seqs, tok, rs, rp, off, sl, lr, ls = plan_step(active, waiting, free, max_rows=64, chunk=4)
    assert seqs == [a] and tok == [4] and lr == [0] and ls == [a]  # last prompt row gives a token
    a.pos = 5
    a.generated.append(77)
    seqs, tok, rs, rp, off, sl, lr, ls = plan_step(active, waiting, free, max_rows=64, chunk=4)
    # a decodes (token 77 at position 5); b is admitted and prefills 4 rows in the same step
    assert seqs == [a, b] and tok == [77, 0, 1, 2, 3] and rs == [0, 1, 1, 1, 1]
    assert rp == [5, 0, 1, 2, 3] and off == [0, 1, 5] and sl == [0, 1] and lr == [0] and ls == [a]


def test_plan_step_respects_row_budget():
    reqs = [Request(np.arange(3, dtype=np.int32), max_new=2) for _ in range(3)]
    active = []
    for i, r in enumerate(reqs):
        r.slot, r.pos = i, 3
        r.generated.append(i)
        active.append(r)
    seqs, tok, rs, rp, off, sl, lr, ls = plan_step(active, [], [], max_rows=2, chunk=4)
    assert len(tok) == 2 and lr == [0, 1]


def test_hybrid_c_abi_exports_every_declared_symbol():
    import re
    from pathlib import Path

    from exl3_b200 import _lib

    lib = _lib.lib()
    text = (Path(__file__).resolve().parents[1] / "include" / "exl3cu_hybrid.h").read_text()
    names = sorted(set(re.findall(r"\b(exl3cu_hyb_\w+)\s*\(", text)))
    assert len(names) >= 10
    for n in names:
        assert hasattr(lib, n), n


def test_attention_split_policy():
    from exl3_b200.hybrid import attn_splits

    assert attn_splits(1) == 32 and attn_splits(2) == 16 and attn_splits(8) == 8 and attn_splits(9) == 2
    assert attn_splits(512) == 1


def test_decode_step_detection():
    """The fused attention runs only when every sequence of the step has exactly one row."""
    from exl3_b200.hybrid import one_row_each

    assert one_row_each([0, 1, 2, 3])
    assert one_row_each([0, 1])
    assert not one_row_each([0, 2])           # a 2-row chunk: its rows attend to each other
    assert not one_row_each([0, 1, 1, 2])     # a sequence granted no row
    assert not one_row_each([0, 1, 5])        # a decode row beside a prefill chunk
    assert not one_row_each([0])              # no sequence


def test_streaming_oracle_agrees_with_token_by_token_oracle(oracle):
    """The teacher-forced, layer-by-layer oracle (packed products through the restated reference
    operator, nothing dense kept) against the token-by-token oracle on dense reconstructed weights:
    the same logits up to the operator's activation rounding (2e-3 of max|l|), on a 4-layer model
    with both mixers."""
    import numpy as np

    from exl3_b200.hybrid import HybridConfig, synthetic_weights
    from oracle.hybrid_model import OracleHybrid, StreamingOracleHybrid

    cfg = HybridConfig(layers=4, hidden=256, ffn=512, vocab=512, heads=2, kv_heads=1)
    w = synthetic_weights(cfg, seed=7)
    tokens = np.random.default_rng(8).integers(0, cfg.vocab, 6)
    dense = OracleHybrid(w, oracle)
    seq = dense.new_sequence()
    want = np.stack([dense.step(seq, int(t), p) for p, t in enumerate(tokens)])
    residuals, got = StreamingOracleHybrid(w, oracle, nth=2).run(tokens)
    assert len(residuals) == cfg.layers and residuals[-1].shape == (len(tokens), cfg.hidden)
    assert got.shape == want.shape
    assert np.max(np.abs(got - want)) / np.max(np.abs(want)) <= 2e-3
