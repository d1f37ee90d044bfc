"""Ragged continuous-admission batches on the GPU: the packer (exl3cu_pack_ragged) against
a plain statement of its rule, and the operator over a packed batch
(exl3cu_mul_mat_ragged, row count read on the device) against the oracle.

Operator tolerance as everywhere: max|y - y_ref| / max|y_ref| <= 2e-3, NMSE < 1e-5."""
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


def pack_rule(want, pos, max_rows):
    """The packing rule: in order, sequence i gets min(max(want_i, 0), rows left)."""
    offs, left = [0], max_rows
    for w in want:
        g = min(max(int(w), 0), left)
        left -= g
        offs.append(offs[-1] + g)
    row_seq = np.full(max_rows, -1, np.int32)
    row_pos = np.full(max_rows, -1, np.int32)
    for i in range(len(want)):
        for r in range(offs[i], offs[i + 1]):
            row_seq[r] = i
            row_pos[r] = pos[i] + r - offs[i]
    return np.array(offs, np.int32), row_seq, row_pos


@pytest.fixture(scope="module")
def ops(cuda_lib):
    from exl3_b200 import ops as _ops

    return _ops


@pytest.mark.parametrize("n_seq,max_rows,seed", [(1, 8, 0), (8, 512, 1), (64, 512, 2), (3000, 4096, 3), (17, 64, 4)])
def test_pack_matches_rule(ops, n_seq, max_rows, seed):
    rng = np.random.default_rng(seed)
    decode = rng.random(n_seq) < 0.5
    want = np.where(decode, 1, rng.integers(16, 513, n_seq)).astype(np.int32)
    want[rng.random(n_seq) < 0.05] = 0
    want[rng.random(n_seq) < 0.02] = -3  # nonsense requests count as zero
    pos = rng.integers(0, 4096, n_seq).astype(np.int32)
    offs, rseq, rpos = ops.pack_ragged(torch.from_numpy(want).cuda(), torch.from_numpy(pos).cuda(), max_rows)
    torch.cuda.synchronize()
    e_offs, e_seq, e_pos = pack_rule(want, pos, max_rows)
    np.testing.assert_array_equal(offs.cpu().numpy(), e_offs)
    np.testing.assert_array_equal(rseq.cpu().numpy(), e_seq)
    np.testing.assert_array_equal(rpos.cpu().numpy(), e_pos)


def _weight(ops, k, n, bits, seed):
    from exl3_b200 import synthetic

    m = synthetic.matrix(k, n, bits, seed=seed)
    rec = m.records()
    return ops.Exl3Weight.from_records(rec, k, n, bits), rec


@pytest.mark.parametrize("want", [[1, 1, 300, 1, 40], [0, 0, 0], [700], [5], [1] * 37 + [60]])
def test_mul_mat_ragged_matches_oracle(ops, oracle, want):
    from exl3_b200 import synthetic

    k, n, bits, max_rows = 1024, 512, 4, 512
    w, rec = _weight(ops, k, n, bits, 7)
    x = synthetic.activations(max_rows, k, seed=8)
    want_t = torch.tensor(want, dtype=torch.int32, device="cuda")
    offs, _, _ = ops.pack_ragged(want_t, torch.zeros_like(want_t), max_rows)
    y = torch.full((max_rows, n), float("nan"), dtype=torch.float32, device="cuda")
    w.mul_mat_ragged(torch.from_numpy(x).cuda(), offs, out=y)
    torch.cuda.synchronize()
    rows = min(sum(max(v, 0) for v in want), max_rows)
    yn = y.cpu().numpy()
    if rows:
        assert_close(yn[:rows], oracle.mul_mat(rec, bits, k, n, x[:rows], nth=16), f"rows={rows}")
    assert np.all(np.isnan(yn[rows:])), "wrote rows past the packed count"
    assert ops.device_status(0) == 0
    w.free()


def test_ragged_graph_replays_any_batch(ops, oracle):
    """One CUDA graph captured at capacity serves batches of every size (device-side row count)."""
    from exl3_b200 import synthetic

    k, n, bits, max_rows = 2048, 768, 4, 512
    w, rec = _weight(ops, k, n, bits, 11)
    x_np = synthetic.activations(max_rows, k, seed=12)
    x = torch.from_numpy(x_np).cuda()
    want = torch.zeros(8, dtype=torch.int32, device="cuda")
    pos = torch.zeros(8, dtype=torch.int32, device="cuda")
    packed = (torch.empty(9, dtype=torch.int32, device="cuda"), torch.empty(max_rows, dtype=torch.int32, device="cuda"),
              torch.empty(max_rows, dtype=torch.int32, device="cuda"))
    y = torch.empty((max_rows, n), dtype=torch.float32, device="cuda")
    st = torch.cuda.Stream()
    want.fill_(64)
    with torch.cuda.stream(st):  # warm-up at full size: grows the GEMM scratch before capture
        ops.pack_ragged(want, pos, max_rows, stream=st, out=packed)
        w.mul_mat_ragged(x, packed[0], out=y, stream=st)
    st.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=st):
        ops.pack_ragged(want, pos, max_rows, stream=st, out=packed)
        w.mul_mat_ragged(x, packed[0], out=y, stream=st)
    for batch in ([1, 1, 1, 1, 1, 1, 1, 1], [3, 0, 17, 1, 1, 0, 40, 2], [64] * 8, [100, 200, 300, 0, 0, 0, 0, 0]):
        want.copy_(torch.tensor(batch, dtype=torch.int32))
        y.fill_(float("nan"))
        g.replay()
        torch.cuda.synchronize()
        rows = min(sum(batch), max_rows)
        yn = y.cpu().numpy()
        assert_close(yn[:rows], oracle.mul_mat(rec, bits, k, n, x_np[:rows], nth=16), f"batch {batch}")
        assert np.all(np.isnan(yn[rows:])), f"batch {batch}: wrote rows past the count"
    del g
    w.free()


def test_ragged_beyond_one_launch(ops, oracle):
    """Capacity above one launch pair (2048 rows): the device count is split across launches."""
    from exl3_b200 import synthetic

    k, n, bits, max_rows = 256, 256, 4, 2300
    w, rec = _weight(ops, k, n, bits, 13)
    x = synthetic.activations(max_rows, k, seed=14)
    for rows in (2100, 2048, 1000):
        offs = torch.tensor([0, rows], dtype=torch.int32, device="cuda")
        y = torch.full((max_rows, n), float("nan"), dtype=torch.float32, device="cuda")
        w.mul_mat_ragged(torch.from_numpy(x).cuda(), offs, out=y)
        torch.cuda.synchronize()
        yn = y.cpu().numpy()
        assert_close(yn[:rows], oracle.mul_mat(rec, bits, k, n, x[:rows], nth=16), f"rows={rows}")
        assert np.all(np.isnan(yn[rows:]))
    w.free()


def test_graphs_survive_scratch_growth(ops, oracle):
    """Graphs captured at a small capacity stay valid after a larger call grows the stream's
    GEMM scratch (the outgrown buffer is retired, not freed)."""
    from exl3_b200 import synthetic

    k, n, bits = 1024, 384, 4
    w, rec = _weight(ops, k, n, bits, 21)
    x_np = synthetic.activations(512, k, seed=22)
    x = torch.from_numpy(x_np).cuda()
    st = torch.cuda.Stream()
    graphs, outs = [], []
    for cap in (32, 128, 512):  # each warm-up grows the scratch past the previous graph's
        offs = torch.tensor([0, cap], dtype=torch.int32, device="cuda")
        y = torch.empty((cap, n), dtype=torch.float32, device="cuda")
        with torch.cuda.stream(st):
            w.mul_mat_ragged(x[:cap], offs, out=y, stream=st)
        st.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=st):
            w.mul_mat_ragged(x[:cap], offs, out=y, stream=st)
        graphs.append(g)
        outs.append((cap, y, offs))
    for g, (cap, y, _) in zip(graphs, outs):
        y.fill_(float("nan"))
        g.replay()
        torch.cuda.synchronize()
        assert_close(y.cpu().numpy(), oracle.mul_mat(rec, bits, k, n, x_np[:cap], nth=16), f"cap={cap}")
    del graphs
    w.free()
