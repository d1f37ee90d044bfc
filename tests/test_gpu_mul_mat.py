"""GPU parity of the EXL3 operator (the GEMV hot path) against the oracle.

Tolerance (north star): max|y - y_ref| / max|y_ref| <= 2e-3 with fp32
accumulation, plus the reference graph test's NMSE < 1e-5
(tests/test-exl3-graph.cpp:100).  The GEMV path rotates activations in fp32
and holds them as fixed point with one scale per warp (22 bits for one or two
rows, 15 bits for three or four); the GEMM path feeds them to the tensor cores
as fp16.  Heavy-tailed inputs (outlier channels, one loud 128-group) are
checked separately because they stress exactly that scaling.
"""
import numpy as np
import pytest
import torch

import kat

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


def _mm(ops, w, x):
    xt = torch.from_numpy(np.ascontiguousarray(x)).cuda()
    y = w.mul_mat(xt)
    torch.cuda.synchronize()
    return y.cpu().numpy()


@pytest.mark.parametrize("bits", range(1, 9))
def test_mul_mat_golden(ops, golden, bits):
    """Against ggml_exl3_mul_mat's own output (4/6/8-bit) or the reference-codec loop."""
    from exl3_b200 import format as fmt

    data, _ = golden
    k, n = kat.KAT_K, kat.KAT_N
    suh, svh = kat.kat_scales()
    rec = fmt.pack_records(kat.kat_packed(bits), suh, svh, bits)
    w = ops.Exl3Weight.from_records(rec, k, n, bits)
    for rows in ((1, 4, 8) if bits in (4, 6, 8) else (1, 4)):
        x = kat.kat_input(rows)
        assert_close(_mm(ops, w, x), data[f"mm_y_b{bits}_r{rows}"], f"bits={bits} rows={rows}")
    x16 = kat.kat_input(1).astype(np.float16)
    assert_close(_mm(ops, w, x16), data[f"mm_y16_b{bits}_r1"], f"bits={bits} f16")
    w.free()


def test_mul_mat_golden_codebooks(ops, golden):
    from exl3_b200 import format as fmt

    data, _ = golden
    k, n = kat.KAT_K, kat.KAT_N
    suh, svh = kat.kat_scales()
    rec = fmt.pack_records(kat.kat_packed(4), suh, svh, 4)
    for cb in (0, 1):
        w = ops.Exl3Weight.from_records(rec, k, n, 4, codebook=cb)
        assert_close(_mm(ops, w, kat.kat_input(1)), data[f"mm_cb{cb}_b4_r1"], f"cb={cb}")
        w.free()


def test_config0_single_layer(ops, oracle):
    """2048 x 6144, 4 bpw, mul1, fp16 N(0,1) batch 1."""
    from exl3_b200 import synthetic

    m = synthetic.matrix(2048, 6144, 4, seed=0)
    rec = m.records()
    w = ops.Exl3Weight.from_records(rec, 2048, 6144, 4)
    inner = w.decode_inner()
    assert np.array_equal(inner, oracle.decode_inner(m.trellis, 2048, 6144, 4, 2))
    x = synthetic.activations(1, 2048, seed=1)
    ref = oracle.mul_mat(rec, 4, 2048, 6144, x, nth=8)
    assert_close(_mm(ops, w, x), ref, "config0")
    w.free()


@pytest.mark.parametrize("bits", (2, 3, 4, 5, 6))
def test_config1_layer_sweep(ops, oracle, bits):
    """every per-layer shape of the 2B decoder at 2..6 bpw, batch 1."""
    from exl3_b200 import synthetic

    for i, (name, (k, n)) in enumerate(synthetic.LAYER_SHAPES.items()):
        m = synthetic.matrix(k, n, bits, seed=1000 * bits + i)
        rec = m.records()
        w = ops.Exl3Weight.from_records(rec, k, n, bits)
        x = synthetic.activations(1, k, seed=7 + i)
        assert_close(_mm(ops, w, x), oracle.mul_mat(rec, bits, k, n, x, nth=8), f"{name} {k}x{n} @{bits}")
        w.free()


@pytest.mark.parametrize("rows", (2, 3, 7, 8, 9, 13, 37))
def test_batches(ops, oracle, rows):
    from exl3_b200 import synthetic

    k, n, bits = 1024, 768, 4
    m = synthetic.matrix(k, n, bits, seed=rows)
    rec = m.records()
    w = ops.Exl3Weight.from_records(rec, k, n, bits)
    x = synthetic.activations(rows, k, seed=rows + 1)
    assert_close(_mm(ops, w, x), oracle.mul_mat(rec, bits, k, n, x, nth=8), f"rows={rows}")
    xf = x.astype(np.float32)
    assert_close(_mm(ops, w, xf), oracle.mul_mat(rec, bits, k, n, xf, nth=8), f"rows={rows} f32")
    w.free()


def test_strided_rows_and_column_slices(ops, oracle):
    from exl3_b200 import synthetic

    k, n, bits = 768, 1024, 3
    m = synthetic.matrix(k, n, bits, seed=11)
    rec = m.records()
    x = synthetic.activations(5, k, seed=12)
    ref = oracle.mul_mat(rec, bits, k, n, x, nth=8)
    w = ops.Exl3Weight.from_records(rec, k, n, bits)
    xpad = torch.zeros((5, k + 64), dtype=torch.float16, device="cuda")
    xpad[:, :k] = torch.from_numpy(x).cuda()
    ypad = torch.full((5, n + 128), float("nan"), dtype=torch.float32, device="cuda")
    w.mul_mat(xpad[:, :k], out=ypad[:, :n])
    torch.cuda.synchronize()
    yp = ypad.cpu().numpy()
    assert_close(yp[:, :n], ref, "strided")
    assert np.all(np.isnan(yp[:, n:])), "wrote outside y rows"
    w.free()
    # a handle holding column blocks [2, 5) computes exactly those columns
    ws = ops.Exl3Weight.from_records(rec, k, n, bits, first_block=2, block_count=3)
    assert_close(_mm(ops, ws, x), ref[:, 256:640], "column slice")
    ws.free()


def test_deterministic_and_workspace_reuse(ops):
    from exl3_b200 import synthetic

    k, n, bits = 4096, 1024, 4
    m = synthetic.matrix(k, n, bits, seed=3)
    w = ops.Exl3Weight.from_records(m.records(), k, n, bits)
    assert w.workspace_bytes > 0  # this shape splits K
    x = torch.from_numpy(synthetic.activations(1, k, seed=4)).cuda()
    first = w.mul_mat(x).clone()
    outs = [w.mul_mat(x) for _ in range(20)]
    torch.cuda.synchronize()
    for o in outs:
        assert torch.equal(o, first)
    ws = torch.zeros(w.workspace_bytes // 4 + 4, dtype=torch.float32, device="cuda")
    via_ws = [w.mul_mat(x, workspace=ws) for _ in range(3)]  # global-workspace split-K variant
    torch.cuda.synchronize()
    for o in via_ws:
        assert torch.equal(o, via_ws[0])
        # fp16-activation variant vs the fixed-point mul1 path: both within the operator tolerance
        assert errs(o.cpu().numpy(), first.cpu().numpy())[0] < TOL_MAX_ABS_REL
    w.free()


def test_host_buffer_path(ops, oracle):
    from exl3_b200 import synthetic

    k, n, bits = 2048, 2048, 4
    m = synthetic.matrix(k, n, bits, seed=21)
    rec = m.records()
    w = ops.Exl3Weight.from_records(rec, k, n, bits)
    x = synthetic.activations(3, k, seed=22)
    y_host = w.mul_mat_host(x)
    assert np.array_equal(y_host, _mm(ops, w, x))
    assert_close(y_host, oracle.mul_mat(rec, bits, k, n, x, nth=8), "host path")
    w.free()


def test_large_matrix_config4(ops, oracle):
    """configs[4] shape: [4096, 14336] weight (k=14336, n=4096) at 4 bpw, batch 1 and 8."""
    from exl3_b200 import synthetic

    k, n, bits = 14336, 4096, 4
    m = synthetic.matrix(k, n, bits, seed=44)
    rec = m.records()
    w = ops.Exl3Weight.from_records(rec, k, n, bits)
    for rows in (1, 8):
        x = synthetic.activations(rows, k, seed=45 + rows)
        assert_close(_mm(ops, w, x), oracle.mul_mat(rec, bits, k, n, x, nth=16), f"config4 rows={rows}")
    w.free()


@pytest.mark.parametrize("bits", (2, 5, 8))
def test_long_k_wide_build(ops, oracle, bits):
    """k >= 8192 runs the GEMV's wide build (two CTAs per SM, tile-pair decode): 1..4 rows at the
    configs[4] depth and several bit widths, against the oracle, and so does the default build
    forced on the same call (its own cluster split, so not bit for bit the same)."""
    import os

    from exl3_b200 import synthetic

    k, n = 14336, 512
    m = synthetic.matrix(k, n, bits, seed=60 + bits)
    rec = m.records()
    w = ops.Exl3Weight.from_records(rec, k, n, bits)
    for rows in (1, 2, 3, 4):
        x = synthetic.activations(rows, k, seed=61 + rows)
        ref = oracle.mul_mat(rec, bits, k, n, x, nth=16)
        assert_close(_mm(ops, w, x), ref, f"wide bits={bits} rows={rows}")
        os.environ["EXL3CU_MUL1_WIDE"] = "0"
        try:
            y_default = _mm(ops, w, x)
        finally:
            del os.environ["EXL3CU_MUL1_WIDE"]
        assert_close(y_default, ref, f"default bits={bits} rows={rows}")
    w.free()


def test_linearity_full_size(ops):
    """Size-independent property at a full BASELINE size: y(a x1 + b x2) = a y(x1) + b y(x2)."""
    from exl3_b200 import synthetic

    k, n, bits = 6144, 2048, 4
    m = synthetic.matrix(k, n, bits, seed=9)
    w = ops.Exl3Weight.from_records(m.records(), k, n, bits)
    x1 = torch.from_numpy(synthetic.activations(1, k, seed=1).astype(np.float32)).cuda()
    x2 = torch.from_numpy(synthetic.activations(1, k, seed=2).astype(np.float32)).cuda()
    y = w.mul_mat(0.5 * x1 + 0.25 * x2)
    y12 = 0.5 * w.mul_mat(x1) + 0.25 * w.mul_mat(x2)
    torch.cuda.synchronize()
    rel, _ = errs(y.cpu().numpy(), y12.cpu().numpy())
    assert rel < 2e-3
    w.free()


def test_invalid_mul_mat_arguments(ops):
    from exl3_b200 import Exl3InvalidArgument, synthetic

    m = synthetic.matrix(256, 256, 4, seed=1)
    w = ops.Exl3Weight.from_records(m.records(), 256, 256, 4)
    with pytest.raises(Exl3InvalidArgument):
        w.mul_mat(torch.zeros((1, 255), dtype=torch.float16, device="cuda"))
    with pytest.raises(Exl3InvalidArgument):  # host memory handed to the device entry point
        from exl3_b200 import _lib
        import ctypes

        x = np.zeros((1, 256), np.float16)
        y = np.zeros((1, 256), np.float32)
        _lib.check(_lib.lib().exl3cu_mul_mat(w.handle, ctypes.c_void_p(x.ctypes.data), 1, 1, 256,
                                             ctypes.c_void_p(y.ctypes.data), 256, None))
    w.free()


def test_grouped_batch_matches_single_calls(ops, oracle):
    """exl3cu_mul_mat_batch: mixed shapes, bitrates, dtypes and row counts (> 8 rows split into
    sub-problems) give what one exl3cu_mul_mat call per item gives, and match the oracle."""
    from exl3_b200 import synthetic

    specs = [(2048, 2048, 4, 1), (2048, 512, 4, 1), (2048, 512, 6, 3), (6144, 2048, 4, 1), (1024, 768, 3, 11),
             (2048, 6144, 4, 2), (512, 256, 5, 1), (4096, 1024, 4, 9), (2048, 2048, 4, 4),
             (256, 128, 2, 1)]
    ws, xs, refs = [], [], []
    for i, (k, n, bits, rows) in enumerate(specs):
        m = synthetic.matrix(k, n, bits, seed=300 + i)
        rec = m.records()
        ws.append(ops.Exl3Weight.from_records(rec, k, n, bits))
        x = synthetic.activations(rows, k, seed=400 + i)
        if i % 3 == 1:
            x = x.astype(np.float32)
        xs.append(torch.from_numpy(x).cuda())
        refs.append(oracle.mul_mat(rec, bits, k, n, x, nth=8))
    outs = ops.mul_mat_batch(ws, xs)
    singles = [w.mul_mat(x) for w, x in zip(ws, xs)]
    torch.cuda.synchronize()
    for i, (o, s1, ref) in enumerate(zip(outs, singles, refs)):
        # a grouped launch may pick another K split than a single one (other summation order and
        # per-CTA activation scale): equal within the operator tolerance, not bit for bit
        assert errs(o.cpu().numpy(), s1.cpu().numpy())[0] < TOL_MAX_ABS_REL, f"item {i}: grouped vs single"
        assert_close(o.cpu().numpy(), ref, f"item {i} {specs[i]}")
    for w in ws:
        w.free()


def test_global_workspace_variant_matches(ops, oracle):
    """exl3cu_mul_mat_ws (split-K through a caller's workspace, the k_gemv kernel) agrees with the
    default operator and, directly, with the CPU restatement of the reference operator."""
    from exl3_b200 import synthetic

    k, n, bits = 6144, 2048, 4
    m = synthetic.matrix(k, n, bits, seed=13)
    rec = m.records()
    w = ops.Exl3Weight.from_records(rec, k, n, bits)
    xh = synthetic.activations(3, k, seed=14)
    x = torch.from_numpy(xh).cuda()
    ws = torch.zeros(w.workspace_bytes // 4 + 4, dtype=torch.float32, device="cuda")
    a = w.mul_mat(x)
    b = w.mul_mat(x, workspace=ws)
    torch.cuda.synchronize()
    rel, _ = errs(a.cpu().numpy(), b.cpu().numpy())
    assert rel < TOL_MAX_ABS_REL
    assert_close(b.cpu().numpy(), oracle.mul_mat(rec, bits, k, n, xh), "workspace kernel vs oracle")
    w.free()


def test_fused_input_forms_and_accumulate(ops):
    """exl3cu_mul_mat_batch_ex: SwiGLU-on-load and RMSNorm-on-load inputs and the accumulating
    epilogue against the plain operator on inputs formed in fp32 on the host (same values up to
    the order of the RMS sum)."""
    import ctypes

    from exl3_b200 import _lib, synthetic

    L = _lib.lib()
    k, n, bits = 1024, 512, 4
    m = synthetic.matrix(k, n, bits, seed=61)
    w = ops.Exl3Weight.from_records(m.records(), k, n, bits)
    rng = np.random.default_rng(7)
    for rows in (1, 3, 4):
        gu = torch.from_numpy(rng.standard_normal((rows, 2 * k)).astype(np.float32)).cuda()
        h = torch.from_numpy((rng.standard_normal((rows, k)) * 3).astype(np.float32)).cuda()
        nw = torch.from_numpy((1 + 0.1 * rng.standard_normal(k)).astype(np.float32)).cuda()
        base = torch.from_numpy(rng.standard_normal((rows, n)).astype(np.float32)).cuda()
        g, u = gu[:, :k], gu[:, k:]
        x_glu = (g / (1 + torch.exp(-g)) * u).contiguous()
        x_rms = (h * torch.rsqrt((h * h).mean(dim=1, keepdim=True) + 1e-6) * nw).contiguous()
        y_glu = base.clone()
        y_rms = torch.empty((rows, n), dtype=torch.float32, device="cuda")
        VP, SZ, IN = ctypes.c_void_p * 2, ctypes.c_size_t * 2, ctypes.c_int * 2
        y_ss = torch.full((rows, n // 128), -1.0, dtype=torch.float32, device="cuda")
        rc = L.exl3cu_mul_mat_batch_ex(
            2, VP(w.handle.value, w.handle.value), VP(gu.data_ptr(), h.data_ptr()), IN(_lib.X_GLU, _lib.X_RMSNORM),
            SZ(rows, rows), SZ(2 * k, k), VP(0, nw.data_ptr()), ctypes.c_float(1e-6),
            VP(y_glu.data_ptr(), y_rms.data_ptr()), SZ(n, n), IN(1, 0), None, VP(y_ss.data_ptr(), 0), None)
        assert rc == 0, L.exl3cu_last_error()
        ref_glu = base + w.mul_mat(x_glu)
        ref_rms = w.mul_mat(x_rms)
        torch.cuda.synchronize()
        assert_close(y_glu.cpu().numpy(), ref_glu.cpu().numpy(), f"glu rows={rows}")
        assert_close(y_rms.cpu().numpy(), ref_rms.cpu().numpy(), f"rmsnorm rows={rows}")
        # the accumulated output's sums of squares per 128-block
        ss_ref = (y_glu.double() ** 2).view(rows, n // 128, 128).sum(dim=2)
        assert torch.allclose(y_ss.double(), ss_ref, rtol=1e-5, atol=0), f"y sums of squares rows={rows}"
        # RMSNorm input with the mean square taken from block sums of squares: same result as from the rows
        h_ss = (h.double() ** 2).view(rows, k // 128, 128).sum(dim=2).float().contiguous()
        y_rms2 = torch.empty((rows, n), dtype=torch.float32, device="cuda")
        VP1, SZ1, IN1 = ctypes.c_void_p * 1, ctypes.c_size_t * 1, ctypes.c_int * 1
        rc = L.exl3cu_mul_mat_batch_ex(1, VP1(w.handle.value), VP1(h.data_ptr()), IN1(_lib.X_RMSNORM), SZ1(rows),
                                       SZ1(k), VP1(nw.data_ptr()), ctypes.c_float(1e-6), VP1(y_rms2.data_ptr()),
                                       SZ1(n), None, VP1(h_ss.data_ptr()), None, None)
        assert rc == 0, L.exl3cu_last_error()
        torch.cuda.synchronize()
        assert_close(y_rms2.cpu().numpy(), ref_rms.cpu().numpy(), f"rmsnorm from block sums rows={rows}")
    # the fused forms are GEMV-only: an 8-row item goes to the GEMM and is refused
    h8 = torch.zeros((8, k), dtype=torch.float32, device="cuda")
    y8 = torch.zeros((8, n), dtype=torch.float32, device="cuda")
    VP1, SZ1, IN1 = ctypes.c_void_p * 1, ctypes.c_size_t * 1, ctypes.c_int * 1
    rc = L.exl3cu_mul_mat_batch_ex(1, VP1(w.handle.value), VP1(h8.data_ptr()), IN1(_lib.X_RMSNORM), SZ1(8), SZ1(k),
                                   VP1(nw.data_ptr()), ctypes.c_float(1e-6), VP1(y8.data_ptr()), SZ1(n), None, None,
                                   None, None)
    assert rc == _lib.NO_SUPPORT
    w.free()


def _heavy_tail(rows, k, seed, mode):
    """N(0,1) activations with 1% of the channels scaled x300 ('channels'), or one whole 128-group
    scaled x1000 ('group'); fp16 like the other operator inputs."""
    from exl3_b200 import synthetic

    x = synthetic.activations(rows, k, seed=seed).astype(np.float32)
    rng = np.random.default_rng(seed + 1)
    if mode == "channels":
        hot = rng.choice(k, size=max(1, k // 100), replace=False)
        x[:, hot] *= 300.0
    else:
        g = int(rng.integers(0, k // 128))
        x[:, g * 128:(g + 1) * 128] *= 1000.0
    return x.astype(np.float16)


@pytest.mark.parametrize("mode", ["channels", "group"])
@pytest.mark.parametrize("rows", [1, 4, 8, 37])
@pytest.mark.parametrize("name", ["q", "gate", "down"])
def test_heavy_tailed_activations(ops, oracle, name, rows, mode):
    """configs[1] shapes with outlier channels or a loud 128-group, within the operator bars (2e-3,
    NMSE 1e-5).  1 and 4 rows run the GEMV, whose fixed-point scale (one per row over a CTA's K range)
    must keep the ordinary channels' resolution; 8 and 37 rows run the tensor-core GEMM, whose fp16
    rotated activations must hold the loud values without overflow or lost resolution."""
    from exl3_b200 import synthetic

    k, n = synthetic.LAYER_SHAPES[name]
    m = synthetic.matrix(k, n, 4, seed=k + 3 * n + rows)
    rec = m.records()
    w = ops.Exl3Weight.from_records(rec, k, n, 4)
    x = _heavy_tail(rows, k, seed=100 + rows, mode=mode)
    y = _mm(ops, w, x)
    assert_close(y, oracle.mul_mat(rec, 4, k, n, x, nth=8), f"{name} rows={rows} {mode}")
    w.free()

