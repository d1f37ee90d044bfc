"""The ggml-facing drop-in: ggml_exl3_mul_mat called exactly as ggml's CPU backend
calls the reference's (params->ith/nth, ggml_tensor src[0]/src[1]/dst with byte
strides), checked against the reference operator's own outputs (golden) and,
when oracle/_ref is present, against the reference operator run live."""
import ctypes

import numpy as np
import pytest

import kat

pytestmark = pytest.mark.gpu


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


def ggml_mul_mat(lib, records, bits, k, n, x, nth=4):
    from exl3_b200.format import BITS_GGML_TYPE

    es = x.itemsize
    rows = x.shape[0]
    y = np.full((rows, n), np.nan, np.float32)
    w = _tensor(BITS_GGML_TYPE[bits], (k, n, 1, 1), (1, 1, 1, 1), records.ctypes.data)
    xin = _tensor(0 if x.dtype == np.float32 else 1, (k, rows, 1, 1), (es, es * k, es * k * rows, es * k * rows),
                  x.ctypes.data)
    dst = _tensor(0, (n, rows, 1, 1), (4, 4 * n, 4 * n * rows, 4 * n * rows), y.ctypes.data)
    dst.src[0] = ctypes.addressof(w)
    dst.src[1] = ctypes.addressof(xin)
    fn = lib.ggml_exl3_mul_mat
    fn.argtypes = [ctypes.POINTER(GgmlParams), ctypes.POINTER(GgmlTensor)]
    for ith in reversed(range(nth)):  # every thread index, as ggml's workers would call it
        p = GgmlParams(ith, nth, 0, None)
        fn(ctypes.byref(p), ctypes.byref(dst))
    return y


@pytest.fixture(scope="module")
def ggml_lib(cuda_lib):
    from exl3_b200 import _lib

    return ctypes.CDLL(str(_lib.GGML_LIB_PATH))


@pytest.mark.parametrize("bits", (4, 6, 8))
def test_ggml_mul_mat_matches_reference_operator(ggml_lib, golden, bits):
    from exl3_b200 import format as fmt

    data, _ = golden
    k, n = kat.KAT_K, kat.KAT_N
    suh, svh = kat.kat_scales()
    rec = fmt.pack_records(kat.kat_packed(bits), suh, svh, bits)
    for rows in (1, 4, 8):
        y = ggml_mul_mat(ggml_lib, rec, bits, k, n, kat.kat_input(rows))
        ref = data[f"mm_y_b{bits}_r{rows}"]
        rel = np.max(np.abs(y - ref)) / np.max(np.abs(ref))
        nmse = np.sum((y.astype(np.float64) - ref) ** 2) / np.sum(ref.astype(np.float64) ** 2)
        assert rel <= 2e-3 and nmse < 1e-5, (bits, rows, rel, nmse)
    y16 = ggml_mul_mat(ggml_lib, rec, bits, k, n, kat.kat_input(1).astype(np.float16))
    ref16 = data[f"mm_y16_b{bits}_r1"]
    assert np.max(np.abs(y16 - ref16)) / np.max(np.abs(ref16)) <= 2e-3


def test_ggml_mul_mat_live_reference(ggml_lib, reference):
    from exl3_b200 import synthetic

    k, n, bits = 2048, 1024, 4
    m = synthetic.matrix(k, n, bits, seed=77)
    rec = m.records()
    x = synthetic.activations(37, k, seed=78)  # a ragged batch, as the reference's graph test uses
    y = ggml_mul_mat(ggml_lib, rec, bits, k, n, x)
    ref = reference.mul_mat(rec, bits, k, n, x, nth=8)
    assert np.max(np.abs(y - ref)) / np.max(np.abs(ref)) <= 2e-3


def test_ggml_weight_cache_follows_buffer_contents(ggml_lib, oracle):
    """A model reloaded into the same host buffer (same address, type and shape) must be served its
    own weights, not the device copy of the previous ones; ggml_exl3_release_weights drops every
    cached upload and the next call uploads again."""
    from exl3_b200 import synthetic

    k, n, bits = 1024, 512, 4
    a = synthetic.matrix(k, n, bits, seed=91).records()
    b = synthetic.matrix(k, n, bits, seed=92).records()
    buf = a.copy()
    x = synthetic.activations(2, k, seed=93)
    ya = ggml_mul_mat(ggml_lib, buf, bits, k, n, x)
    buf[:] = b  # a second model at the same address
    yb = ggml_mul_mat(ggml_lib, buf, bits, k, n, x)
    ref_a = oracle.mul_mat(a, bits, k, n, x)
    ref_b = oracle.mul_mat(b, bits, k, n, x)
    assert np.max(np.abs(ya - ref_a)) / np.max(np.abs(ref_a)) <= 2e-3
    assert np.max(np.abs(yb - ref_b)) / np.max(np.abs(ref_b)) <= 2e-3
    ggml_lib.ggml_exl3_release_weights.restype = None
    ggml_lib.ggml_exl3_release_weights()
    yb2 = ggml_mul_mat(ggml_lib, buf, bits, k, n, x)
    assert np.array_equal(yb2, yb)
