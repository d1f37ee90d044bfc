"""Pins the CPU oracle (oracle/exl3_oracle.c) before anything is compared with it.

1. The reference's own known-answer tests (tests/test_codec.cpp:14-89 of the
   reference), restated against the oracle.
2. The golden vectors in tests/golden/exl3_golden.npz, produced by the
   reference's own compiled sources (tests/golden/make_golden.py).
3. When oracle/_ref is present: live agreement with the reference on seeded
   random shapes.
"""
import hashlib
import math

import numpy as np
import pytest

import kat


def sha(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


# ---- (1) the reference's own KATs -------------------------------------------------------

def test_mul1_closed_form_exhaustive(oracle):
    """All 65536 mul1 states equal (1774*s - 905216)/2^18 rounded once (test_codec.cpp:16-32)."""
    table = oracle.codebook_table(2)
    states = np.arange(65536, dtype=np.uint64)
    p = (states * 0x83DCD12D) & 0xFFFFFFFF
    s = (p & 255) + ((p >> 8) & 255) + ((p >> 16) & 255) + (p >> 24)
    exact = ((1774 * s.astype(np.int64) - 905216) / 262144.0).astype(np.float32)
    assert np.all(np.abs(exact) >= 2.0 ** -14) and np.all(np.abs(exact) < 65504.0)
    assert np.array_equal(exact.astype(np.float16).view(np.uint16), table)
    # the packed-rounding integer form (test_codec.cpp:22-31)
    fb = exact.view(np.uint32).astype(np.uint64)
    mag = fb & 0x7FFFFFFF
    tie = (mag >> 13) & 1
    code = mag - 0x38000001 + tie
    assert np.all(code <= 0x7FFFFFFF - 4096)
    rounded = (code + 4096) >> 13
    assert np.all(rounded <= 32767)
    packed_half = (rounded | ((fb >> 16) & 0x8000)).astype(np.uint16)
    assert np.array_equal(packed_half, table)


def test_fp16_roundtrip_and_rounding(oracle):
    for h in range(0, 65536, 7):
        if (h & 0x7C00) != 0x7C00:
            assert oracle.float_to_half(oracle.half_to_float(h)) == h
    assert oracle.float_to_half(1.00048828125) == 0x3C00   # tie to even
    assert oracle.float_to_half(1.00146484375) == 0x3C02   # odd tie upward
    assert oracle.float_to_half(65520.0) == 0x7C00         # overflow rounding
    assert oracle.float_to_half(float("nan")) & 0x7FFF == 0x7E00
    assert oracle.float_to_half(-float("inf")) == 0xFC00
    assert oracle.float_to_half(2.0 ** -25) == 0            # exact half-ulp tie below min subnormal
    assert oracle.float_to_half(2.0 ** -24) == 1


def test_fp16_matches_numpy_everywhere(oracle):
    """numpy's float32->float16 is IEEE RNE too; compare on every fp16 plus midpoints."""
    h = np.arange(65536, dtype=np.uint16)
    f = h.view(np.float16).astype(np.float32)
    back = np.array([oracle.half_to_float(int(v)) for v in h[::97]], np.float32)
    assert np.array_equal(back.view(np.uint32)[~np.isnan(back)], f[::97].view(np.uint32)[~np.isnan(back)])
    rng = np.random.default_rng(1)
    samples = rng.standard_normal(5000).astype(np.float32) * np.float32(2.0) ** rng.integers(-26, 17, 5000)
    mine = np.array([oracle.float_to_half(float(v)) for v in samples], np.uint16)
    assert np.array_equal(mine, samples.astype(np.float16).view(np.uint16))


def test_h128_involution(oracle):
    values = np.array([(i % 19 - 9) / 17 for i in range(256)], np.float32)
    twice = oracle.hadamard128(oracle.hadamard128(values))
    assert np.max(np.abs(twice - values)) < 1e-6
    with pytest.raises(ValueError):
        oracle.hadamard128(np.zeros(100, np.float32))


def test_zero_ring_decode(oracle):
    packed = np.zeros(128, np.uint16)
    for bits in range(1, 9):
        for cb in range(3):
            tile = oracle.decode_tile(packed, bits, cb)
            assert np.all(tile == oracle.decode_codebook(np.array([0]), cb)[0])


def test_invalid_arguments_rejected(oracle):
    packed = np.zeros(128, np.uint16)
    with pytest.raises(ValueError):
        oracle.decode_tile(packed, 0, 2)
    with pytest.raises(ValueError):
        oracle.decode_tile(packed, 9, 2)
    with pytest.raises(ValueError):
        oracle.decode_tile(packed, 4, 3)
    with pytest.raises(ValueError):  # slice past the end (test_codec.cpp:86)
        oracle.decode_inner(packed, 16, 16, 4, 2, first_column=16, column_count=16)
    with pytest.raises(ValueError):
        oracle.decode_inner(packed, 16, 16, 4, 2, first_column=8, column_count=8)


# ---- (2) golden vectors from the reference -----------------------------------------------

def test_golden_codebooks(oracle, golden):
    _, meta = golden
    for cb in range(3):
        assert sha(oracle.codebook_table(cb)) == meta[f"cb_sha256_{cb}"], cb


@pytest.mark.parametrize("bits", range(1, 9))
def test_golden_inner_and_reconstruct(oracle, golden, bits):
    data, meta = golden
    packed = kat.kat_packed(bits)
    assert sha(packed) == meta[f"packed_sha256_{bits}"]
    suh, svh = kat.kat_scales()
    for cb in range(3):
        inner = oracle.decode_inner(packed, kat.KAT_K, kat.KAT_N, bits, cb)
        assert np.array_equal(inner[:2], data[f"inner_head_{bits}_{cb}"])
        assert sha(inner) == meta[f"inner_sha256_{bits}_{cb}"], (bits, cb)
        rec = oracle.reconstruct(packed, suh, svh, kat.KAT_K, kat.KAT_N, bits, cb)
        assert sha(rec) == meta[f"recon_sha256_{bits}_{cb}"], (bits, cb)


def _max_abs_rel(y, ref):
    return float(np.max(np.abs(y - ref)) / max(np.max(np.abs(ref)), 1e-30))


@pytest.mark.parametrize("bits", range(1, 9))
def test_golden_mul_mat(oracle, golden, bits):
    data, _ = golden
    k, n = kat.KAT_K, kat.KAT_N
    suh, svh = kat.kat_scales()
    records = oracle.pack_records(kat.kat_packed(bits), suh, svh, k, n, bits)
    for rows in ((1, 4, 8) if bits in (4, 6, 8) else (1, 4)):
        y = oracle.mul_mat(records, bits, k, n, kat.kat_input(rows))
        assert _max_abs_rel(y, data[f"mm_y_b{bits}_r{rows}"]) < 1e-6
    y16 = oracle.mul_mat(records, bits, k, n, kat.kat_input(1).astype(np.float16))
    assert _max_abs_rel(y16, data[f"mm_y16_b{bits}_r1"]) < 1e-6
    for nth in (2, 3):  # thread-count invariance: the reference gives the same y for any ith/nth split
        assert np.array_equal(oracle.mul_mat(records, bits, k, n, kat.kat_input(1), nth=nth),
                              oracle.mul_mat(records, bits, k, n, kat.kat_input(1), nth=1))


def test_golden_mul_mat_codebooks(oracle, golden):
    data, _ = golden
    k, n = kat.KAT_K, kat.KAT_N
    suh, svh = kat.kat_scales()
    records = oracle.pack_records(kat.kat_packed(4), suh, svh, k, n, 4)
    for cb in (0, 1):
        y = oracle.mul_mat(records, 4, k, n, kat.kat_input(1), codebook=cb)
        assert _max_abs_rel(y, data[f"mm_cb{cb}_b4_r1"]) < 1e-6


@pytest.mark.parametrize("bits", (4, 6, 8))
def test_golden_get_rows(oracle, golden, bits):
    data, _ = golden
    k, n = kat.KAT_K, kat.KAT_N
    suh, svh = kat.kat_scales()
    records = oracle.pack_records(kat.kat_packed(bits), suh, svh, k, n, bits)
    for count in (1, 3, 17):
        out = oracle.get_rows(records, bits, k, n, kat.rows_ids(count, n))
        assert np.array_equal(out, data[f"rows_b{bits}_c{count}"])


def test_golden_h128(oracle, golden):
    data, meta = golden
    h = oracle.hadamard128(kat.kat_h128_blocks())
    assert sha(h) == meta["h128_sha256"]
    assert np.array_equal(h[5], data["h128_block5"])


# ---- (3) live agreement with the reference build -----------------------------------------

@pytest.mark.parametrize("seed", range(3))
def test_live_vs_reference(oracle, reference, seed):
    rng = np.random.default_rng(seed)
    bits = int(rng.integers(1, 9))
    k, n = 128 * int(rng.integers(1, 4)), 128 * int(rng.integers(1, 4))
    packed = rng.integers(0, 65536, (k // 16, n // 16, 16 * bits), dtype=np.uint16)
    suh = rng.choice([-1.0, 1.0], k).astype(np.float16).view(np.uint16)
    svh = (rng.choice([-1.0, 1.0], n) * rng.uniform(0.01, 0.03, n)).astype(np.float16).view(np.uint16)
    for cb in range(3):
        assert np.array_equal(oracle.decode_inner(packed, k, n, bits, cb), reference.decode_inner(packed, k, n, bits, cb))
        assert np.array_equal(oracle.reconstruct(packed, suh, svh, k, n, bits, cb),
                              reference.reconstruct(packed, suh, svh, k, n, bits, cb))
    records = oracle.pack_records(packed, suh, svh, k, n, bits)
    x = rng.standard_normal((3, k)).astype(np.float16)
    y_ref = reference.mul_mat(records, bits, k, n, x, nth=2)
    y = oracle.mul_mat(records, bits, k, n, x)
    assert _max_abs_rel(y, y_ref) < 1e-6


def test_reference_ggml_thread_invariance(reference, oracle):
    k, n, bits = 256, 384, 4
    suh, svh = kat.kat_scales()
    records = oracle.pack_records(kat.kat_packed(bits), suh, svh, k, n, bits)
    x = kat.kat_input(2)
    base = reference.mul_mat(records, bits, k, n, x, nth=1)
    for nth in (2, 4, 8):
        assert np.array_equal(reference.mul_mat(records, bits, k, n, x, nth=nth), base)
    assert math.isfinite(float(base.sum()))
