"""GPU get_rows (the tied-embedding lookup, src/exl3-ggml.cpp:19-49) against the
reference operator's golden outputs and the oracle.

Bar: bit-exact.  Every output value is an fp16 that exl3::reconstruct produces
(src/exl3_codec.cpp:169-204: decode, row H128, column H128, x suh x svh, round),
widened to f32; the kernel performs the same fp32 operations in the same order.
"""
import ctypes

import numpy as np
import pytest
import torch

import kat

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ops(cuda_lib):
    from exl3_b200 import ops as _ops

    return _ops


def _rows(w, ids):
    t = torch.from_numpy(np.ascontiguousarray(ids, np.int32)).cuda()
    out = w.get_rows(t)
    torch.cuda.synchronize()
    return out.cpu().numpy()


@pytest.mark.parametrize("bits", (4, 6, 8))
def test_get_rows_golden(ops, golden, bits):
    """The reference operator's own outputs for its graph test's ids (tests/test-exl3-graph.cpp:112)."""
    from exl3_b200 import format as fmt

    data, _ = golden
    k, n = kat.KAT_K, kat.KAT_N
    suh, svh = kat.kat_scales()
    w = ops.Exl3Weight.from_records(fmt.pack_records(kat.kat_packed(bits), suh, svh, bits), k, n, bits)
    for count in (1, 3, 17):
        ids = kat.rows_ids(count, n)
        ref = data[f"rows_b{bits}_c{count}"]
        assert np.array_equal(_rows(w, ids), ref), (bits, count)
        assert np.array_equal(w.get_rows_host(ids), ref), (bits, count)


@pytest.mark.parametrize("bits", range(1, 9))
@pytest.mark.parametrize("codebook", (0, 1, 2))
def test_get_rows_oracle_every_bitrate_and_codebook(ops, oracle, bits, codebook):
    from exl3_b200 import synthetic

    k, n = 512, 384
    m = synthetic.matrix(k, n, bits, seed=900 + bits)
    rec = m.records()
    w = ops.Exl3Weight.from_records(rec, k, n, bits, codebook=codebook)
    rng = np.random.default_rng(bits * 10 + codebook)
    ids = np.concatenate([[0, n - 1, 127, 128], rng.integers(0, n, 20)]).astype(np.int32)
    got = _rows(w, ids)
    ref = oracle.get_rows(rec, bits, k, n, ids, codebook=codebook)
    assert np.array_equal(got, ref)


def test_get_rows_column_range_handle(ops, oracle):
    """A handle over blocks [1, 3) answers local ids 0..255 with columns 128..383."""
    from exl3_b200 import synthetic

    k, n, bits = 256, 512, 4
    rec = synthetic.matrix(k, n, bits, seed=31).records()
    w = ops.Exl3Weight.from_records(rec, k, n, bits, first_block=1, block_count=2)
    ids = np.array([0, 5, 127, 128, 255], np.int32)
    ref = oracle.get_rows(rec, bits, k, n, ids + 128)
    assert np.array_equal(_rows(w, ids), ref)


def test_get_rows_many_ids_and_strided_out(ops, oracle):
    from exl3_b200 import synthetic

    k, n, bits = 1024, 1024, 5
    rec = synthetic.matrix(k, n, bits, seed=32).records()
    w = ops.Exl3Weight.from_records(rec, k, n, bits)
    ids = np.random.default_rng(4).integers(0, n, 300).astype(np.int32)
    out = torch.full((300, k + 64), 7.0, dtype=torch.float32, device="cuda")
    w.get_rows(torch.from_numpy(ids).cuda(), out=out)
    torch.cuda.synchronize()
    o = out.cpu().numpy()
    assert np.array_equal(o[:, :k], oracle.get_rows(rec, bits, k, n, ids))
    assert np.all(o[:, k:] == 7.0)  # the stride gap is not written


def test_get_rows_bad_id_is_reported_not_faulted(ops):
    """An id outside the columns read on the device: NaN row + status bit 1; valid rows unaffected.
    The host form rejects it before any device work."""
    from exl3_b200 import _lib, synthetic

    k, n, bits = 256, 256, 4
    rec = synthetic.matrix(k, n, bits, seed=33).records()
    w = ops.Exl3Weight.from_records(rec, k, n, bits)
    ops.device_status(0, clear=True)
    got = _rows(w, np.array([3, n, -1, 4], np.int32))
    assert np.all(np.isnan(got[1])) and np.all(np.isnan(got[2]))
    assert np.all(np.isfinite(got[0])) and np.all(np.isfinite(got[3]))
    assert ops.device_status(0, clear=True) & 2
    assert ops.device_status(0, clear=True) == 0
    with pytest.raises(Exception):
        w.get_rows_host(np.array([0, n], np.int32))
    assert b"outside" in _lib.lib().exl3cu_last_error()


def test_get_rows_equals_reconstructed_columns(ops):
    """Cross-check inside the library: get_rows(id) == column id of the reconstructed matrix."""
    from exl3_b200 import synthetic

    k, n, bits = 256, 256, 3
    m = synthetic.matrix(k, n, bits, seed=34)
    w = ops.Exl3Weight.from_records(m.records(), k, n, bits)
    ids = np.arange(n, dtype=np.int32)
    rows = _rows(w, ids)
    full = ops.reconstruct(m.trellis, m.suh, m.svh, k, n, bits).view(np.float16)
    assert np.array_equal(rows, full.astype(np.float32).T)


class GgmlTensor(ctypes.Structure):
    _fields_ = [("type", ctypes.c_int), ("ne", ctypes.c_int64 * 4), ("nb", ctypes.c_size_t * 4),
                ("src", ctypes.c_void_p * 10), ("data", ctypes.c_void_p)]


class GgmlParams(ctypes.Structure):
    _fields_ = [("ith", ctypes.c_int), ("nth", ctypes.c_int), ("wsize", ctypes.c_size_t), ("wdata", ctypes.c_void_p)]


def _tensor(typ, ne, nb, data):
    t = GgmlTensor()
    t.type = typ
    for i in range(4):
        t.ne[i] = ne[i]
        t.nb[i] = nb[i]
    t.data = data
    return t


def _ggml_get_rows(glib, records, bits, k, n, ids2d, row_pitch, nth=4):
    """ids as ggml's [ne0, ne1] I32 tensor; dst rows `row_pitch` floats apart."""
    from exl3_b200.format import BITS_GGML_TYPE

    ne0, ne1 = ids2d.shape[1], ids2d.shape[0]
    count = ne0 * ne1
    dst_buf = np.full((count, row_pitch), 5.0, np.float32)
    w = _tensor(BITS_GGML_TYPE[bits], (k, n, 1, 1), (1, 1, 1, 1), records.ctypes.data)
    idt = _tensor(26, (ne0, ne1, 1, 1), (4, 4 * ne0, 4 * count, 4 * count), ids2d.ctypes.data)
    dst = _tensor(0, (k, ne0, ne1, 1), (4, 4 * row_pitch, 4 * row_pitch * ne0, 4 * row_pitch * count),
                  dst_buf.ctypes.data)
    dst.src[0] = ctypes.addressof(w)
    dst.src[1] = ctypes.addressof(idt)
    fn = glib.ggml_exl3_get_rows
    fn.argtypes = [ctypes.POINTER(GgmlParams), ctypes.POINTER(GgmlTensor)]
    for ith in reversed(range(nth)):
        p = GgmlParams(ith, nth, 0, None)
        fn(ctypes.byref(p), ctypes.byref(dst))
    return dst_buf


@pytest.mark.parametrize("bits", (4, 6, 8))
def test_ggml_get_rows_matches_reference_operator(cuda_lib, golden, bits):
    from exl3_b200 import _lib
    from exl3_b200 import format as fmt

    glib = ctypes.CDLL(str(_lib.GGML_LIB_PATH))
    data, _ = golden
    k, n = kat.KAT_K, kat.KAT_N
    suh, svh = kat.kat_scales()
    rec = fmt.pack_records(kat.kat_packed(bits), suh, svh, bits)
    ids = np.ascontiguousarray(kat.rows_ids(17, n)[:16].reshape(4, 4))
    ref = data[f"rows_b{bits}_c17"][:16]
    for pitch in (k, k + 32):  # contiguous dst, then rows with a gap
        out = _ggml_get_rows(glib, rec, bits, k, n, ids, pitch)
        assert np.array_equal(out[:, :k], ref), (bits, pitch)
        if pitch > k:
            assert np.all(out[:, k:] == 5.0)


def test_ggml_get_rows_live_reference(cuda_lib, reference):
    from exl3_b200 import _lib, synthetic

    glib = ctypes.CDLL(str(_lib.GGML_LIB_PATH))
    k, n, bits = 1024, 2048, 4
    rec = synthetic.matrix(k, n, bits, seed=35).records()
    ids = np.random.default_rng(5).integers(0, n, (3, 7)).astype(np.int32)
    out = _ggml_get_rows(glib, rec, bits, k, n, ids, k)
    assert np.array_equal(out, reference.get_rows(rec, bits, k, n, ids.reshape(-1), nth=4))
