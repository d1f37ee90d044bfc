"""The persistent sequence operator (exl3cu_mul_mat_sequence): many problems in one launch,
grouped, a later group reading an earlier group's output.  Same tolerance as the operator:
max|y - y_ref| / max|y_ref| <= 2e-3, NMSE < 1e-5."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

TOL_MAX_ABS_REL = 2e-3
TOL_NMSE = 1e-5


def assert_close(y, ref, what=""):
    y = np.asarray(y, np.float64)
    ref = np.asarray(ref, np.float64)
    assert np.all(np.isfinite(y)), what
    rel = np.max(np.abs(y - ref)) / max(np.max(np.abs(ref)), 1e-30)
    nmse = np.sum((y - ref) ** 2) / max(np.sum(ref ** 2), 1e-300)
    assert rel <= TOL_MAX_ABS_REL and nmse < TOL_NMSE, f"{what}: max_abs_rel={rel:.3e} nmse={nmse:.3e}"


@pytest.fixture(scope="module")
def ops(cuda_lib):
    from exl3_b200 import ops as _ops

    return _ops


def _mat(ops, k, n, bits, seed):
    from exl3_b200 import synthetic

    m = synthetic.matrix(k, n, bits, seed=seed)
    rec = m.records()
    return ops.Exl3Weight.from_records(rec, k, n, bits), rec


@pytest.mark.parametrize("bits", (2, 4, 6))
def test_sequence_matches_oracle(ops, oracle, bits):
    """A decoder-like layer: {q, k, v} | {o} | {gate, up} | {down}, rows 1..4, independent inputs."""
    from exl3_b200 import synthetic

    shapes = [(1024, 1024), (1024, 256), (1024, 256), (1024, 1024), (1024, 2048), (1024, 2048), (2048, 1024)]
    groups = [0, 0, 0, 1, 2, 2, 3]
    rows = [1, 2, 3, 4, 1, 3, 2]
    mats = [_mat(ops, k, n, bits, 300 + i) for i, (k, n) in enumerate(shapes)]
    xs_np = [synthetic.activations(r, k, seed=400 + i) for i, ((k, _), r) in enumerate(zip(shapes, rows))]
    xs = [torch.from_numpy(x).cuda() for x in xs_np]
    outs = ops.mul_mat_sequence([w for w, _ in mats], xs, groups=groups)
    torch.cuda.synchronize()
    for i, ((w, rec), (k, n), x, y) in enumerate(zip(mats, shapes, xs_np, outs)):
        assert_close(y.cpu().numpy(), oracle.mul_mat(rec, bits, k, n, x, nth=16), f"problem {i}")
    assert ops.device_status(0) == 0
    for w, _ in mats:
        w.free()


def test_sequence_dependency_chain(ops, oracle):
    """Group g+1's input is group g's output (f32): the wait and the L2-coherent reads are exercised."""
    from exl3_b200 import synthetic

    bits, rows, depth = 4, 3, 6
    dims = [1024, 2048, 512, 1536, 1024, 2048, 768]
    mats = [_mat(ops, dims[i], dims[i + 1], bits, 500 + i) for i in range(depth)]
    x0 = synthetic.activations(rows, dims[0], seed=600).astype(np.float32)
    bufs = [torch.from_numpy(x0).cuda()] + [torch.full((rows, dims[i + 1]), float("nan"), device="cuda")
                                            for i in range(depth)]
    for _ in range(3):  # repeated launches reuse the counters and slots
        for b in bufs[1:]:
            b.fill_(float("nan"))
        ops.mul_mat_sequence([w for w, _ in mats], bufs[:depth], outs=bufs[1:], groups=list(range(depth)))
        torch.cuda.synchronize()
        ref = x0
        for i, (w, rec) in enumerate(mats):
            # the reference consumes the GPU's own previous output, so errors do not compound
            x_in = bufs[i].cpu().numpy()
            ref = oracle.mul_mat(rec, bits, dims[i], dims[i + 1], x_in, nth=16)
            assert_close(bufs[i + 1].cpu().numpy(), ref, f"stage {i}")
    assert ops.device_status(0) == 0
    for w, _ in mats:
        w.free()


def test_sequence_deterministic_and_matches_mul_mat(ops):
    from exl3_b200 import synthetic

    bits = 4
    mats = [_mat(ops, 2048, 2048, bits, 700 + i)[0] for i in range(4)]
    xs = [torch.from_numpy(synthetic.activations(2, 2048, seed=710 + i)).cuda() for i in range(4)]
    a = [o.clone() for o in ops.mul_mat_sequence(mats, xs, groups=[0, 0, 1, 1])]
    b = ops.mul_mat_sequence(mats, xs, groups=[0, 0, 1, 1])
    singles = [w.mul_mat(x) for w, x in zip(mats, xs)]
    torch.cuda.synchronize()
    for i in range(4):
        assert torch.equal(a[i], b[i])
        # same math as the standalone operator; the K split differs, so compare within tolerance
        assert_close(a[i].cpu().numpy(), singles[i].cpu().numpy(), f"problem {i} vs mul_mat")
    for w in mats:
        w.free()


def test_sequence_rejects_unsupported(ops):
    from exl3_b200 import _lib, synthetic

    w4, _ = _mat(ops, 256, 256, 4, 801)
    w3, _ = _mat(ops, 256, 256, 3, 802)
    x = torch.from_numpy(synthetic.activations(2, 256, seed=803)).cuda()
    with pytest.raises(_lib.Exl3Error):
        ops.mul_mat_sequence([w4, w3], [x, x])  # mixed bit widths
    x5 = torch.from_numpy(synthetic.activations(5, 256, seed=804)).cuda()
    with pytest.raises(_lib.Exl3Error):
        ops.mul_mat_sequence([w4], [x5])  # more than 4 rows
    with pytest.raises(_lib.Exl3Error):
        ops.mul_mat_sequence([w4, w4], [x, x], groups=[1, 0])  # decreasing groups
    w4.free()
    w3.free()
