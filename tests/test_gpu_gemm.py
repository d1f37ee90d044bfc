"""GPU parity of the tensor-core GEMM path (operands of 5 rows or more) against the oracle.

Rows of a call go to the tcgen05 GEMM from 5 upwards: decoded weights in TMEM
as the A operand, up to 256 tokens per CTA as N, K split over a cluster when
the column blocks alone do not fill the device, ragged last token groups,
launches of at most 2048 rows.  Same
tolerance as the GEMV path: max|y - y_ref| / max|y_ref| <= 2e-3 and NMSE < 1e-5
(tests/test-exl3-graph.cpp:100); decoded weights are bit-exact, activations
enter the tensor cores rotated and rounded to fp16, products accumulate in fp32.
"""
import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

TOL_MAX_ABS_REL = 2e-3
TOL_NMSE = 1e-5


def errs(y, ref):
    y = np.asarray(y, np.float64)
    ref = np.asarray(ref, np.float64)
    rel = np.max(np.abs(y - ref)) / max(np.max(np.abs(ref)), 1e-30)
    nmse = np.sum((y - ref) ** 2) / max(np.sum(ref ** 2), 1e-300)
    return rel, nmse


def assert_close(y, ref, what=""):
    assert np.all(np.isfinite(y)), what
    rel, nmse = errs(y, ref)
    assert rel <= TOL_MAX_ABS_REL and nmse < TOL_NMSE, f"{what}: max_abs_rel={rel:.3e} nmse={nmse:.3e}"


@pytest.fixture(scope="module")
def ops(cuda_lib):
    from exl3_b200 import ops as _ops

    return _ops


def _status(cuda_lib):
    st = ctypes.c_uint(0)
    assert cuda_lib.exl3cu_device_status(torch.cuda.current_device(), ctypes.byref(st), 1) == 0
    return st.value


def _mm(w, x):
    y = w.mul_mat(torch.from_numpy(np.ascontiguousarray(x)).cuda())
    torch.cuda.synchronize()
    return y.cpu().numpy()


# (k, n): S = 8 cluster split (few column blocks), S = 1 (enough blocks to fill the device), in between
SHAPES = [(2048, 256), (512, 128 * 80), (1024, 768)]


@pytest.mark.parametrize("k,n", SHAPES)
@pytest.mark.parametrize("rows", (5, 9, 16, 100, 128, 129, 300, 512, 600))
def test_gemm_rows(ops, oracle, cuda_lib, k, n, rows):
    from exl3_b200 import synthetic

    bits = 4
    m = synthetic.matrix(k, n, bits, seed=rows + k)
    rec = m.records()
    w = ops.Exl3Weight.from_records(rec, k, n, bits)
    x = synthetic.activations(rows, k, seed=rows * 3 + 1)
    assert_close(_mm(w, x), oracle.mul_mat(rec, bits, k, n, x, nth=16), f"{k}x{n} rows={rows}")
    assert _status(cuda_lib) == 0
    w.free()


@pytest.mark.parametrize("bits", range(1, 9))
def test_gemm_bits(ops, oracle, bits):
    from exl3_b200 import synthetic

    k, n, rows = 1024, 512, 40
    m = synthetic.matrix(k, n, bits, seed=50 + bits)
    rec = m.records()
    w = ops.Exl3Weight.from_records(rec, k, n, bits)
    x = synthetic.activations(rows, k, seed=60 + bits)
    assert_close(_mm(w, x), oracle.mul_mat(rec, bits, k, n, x, nth=16), f"bits={bits}")
    w.free()


@pytest.mark.parametrize("cb", (0, 1))
def test_gemm_codebooks(ops, oracle, cb):
    from exl3_b200 import synthetic

    k, n, bits, rows = 768, 384, 3, 33
    m = synthetic.matrix(k, n, bits, seed=70 + cb)
    rec = m.records()
    w = ops.Exl3Weight.from_records(rec, k, n, bits, codebook=cb)
    x = synthetic.activations(rows, k, seed=71)
    assert_close(_mm(w, x), oracle.mul_mat(rec, bits, k, n, x, codebook=cb, nth=16), f"cb={cb}")
    w.free()


def test_gemm_f32_input_strides_and_slices(ops, oracle):
    from exl3_b200 import synthetic

    k, n, bits, rows = 1280, 640, 4, 70
    m = synthetic.matrix(k, n, bits, seed=81)
    rec = m.records()
    x = synthetic.activations(rows, k, seed=82).astype(np.float32)
    ref = oracle.mul_mat(rec, bits, k, n, x, nth=16)
    w = ops.Exl3Weight.from_records(rec, k, n, bits)
    xpad = torch.zeros((rows, k + 32), dtype=torch.float32, device="cuda")
    xpad[:, :k] = torch.from_numpy(x).cuda()
    ypad = torch.full((rows, n + 64), float("nan"), dtype=torch.float32, device="cuda")
    w.mul_mat(xpad[:, :k], out=ypad[:, :n])
    torch.cuda.synchronize()
    yp = ypad.cpu().numpy()
    assert_close(yp[:, :n], ref, "f32 strided")
    assert np.all(np.isnan(yp[:, n:])), "wrote outside y rows"
    w.free()
    ws = ops.Exl3Weight.from_records(rec, k, n, bits, first_block=1, block_count=3)
    assert_close(_mm(ws, x), ref[:, 128:512], "column slice")
    ws.free()


def test_gemm_beyond_one_launch(ops, oracle):
    """More rows than one launch pair takes (2048): the call splits its rows."""
    from exl3_b200 import synthetic

    k, n, bits, rows = 256, 256, 4, 2100
    m = synthetic.matrix(k, n, bits, seed=91)
    rec = m.records()
    w = ops.Exl3Weight.from_records(rec, k, n, bits)
    x = synthetic.activations(rows, k, seed=92)
    assert_close(_mm(w, x), oracle.mul_mat(rec, bits, k, n, x, nth=16), "rows=2100")
    w.free()


def test_gemm_deterministic(ops):
    from exl3_b200 import synthetic

    k, n, bits, rows = 4096, 1024, 4, 64
    m = synthetic.matrix(k, n, bits, seed=93)
    w = ops.Exl3Weight.from_records(m.records(), k, n, bits)
    x = torch.from_numpy(synthetic.activations(rows, k, seed=94)).cuda()
    first = w.mul_mat(x).clone()
    outs = [w.mul_mat(x) for _ in range(10)]
    torch.cuda.synchronize()
    for o in outs:
        assert torch.equal(o, first)
    w.free()


def test_gemm_rows_independent(ops):
    """A row's output does not depend on the other rows of the batch (ragged admission)."""
    from exl3_b200 import synthetic

    k, n, bits = 1024, 512, 4
    m = synthetic.matrix(k, n, bits, seed=95)
    w = ops.Exl3Weight.from_records(m.records(), k, n, bits)
    x = synthetic.activations(200, k, seed=96)
    full = _mm(w, x)
    part = _mm(w, x[37:37 + 90])
    np.testing.assert_array_equal(part, full[37:37 + 90])
    w.free()


def test_gemm_batch_mixed_with_gemv(ops, oracle):
    """A grouped call whose operands split between the GEMV (<= 4 rows) and the GEMM."""
    from exl3_b200 import synthetic

    k, n, bits = 1024, 384, 4
    mats = [synthetic.matrix(k, n, bits, seed=100 + i) for i in range(3)]
    recs = [m.records() for m in mats]
    ws = [ops.Exl3Weight.from_records(r, k, n, bits) for r in recs]
    xs_np = [synthetic.activations(r, k, seed=110 + r) for r in (3, 20, 130)]
    xs = [torch.from_numpy(x).cuda() for x in xs_np]
    outs = ops.mul_mat_batch(ws, xs)
    torch.cuda.synchronize()
    for w, r, x, y in zip(ws, recs, xs_np, outs):
        assert_close(y.cpu().numpy(), oracle.mul_mat(r, bits, k, n, x, nth=16), f"rows={x.shape[0]}")
        w.free()
