"""The column-split exchange's protocol on one GPU, through the C ABI.

Two ranks of a column split are emulated in one process on one GPU: each
rank's y buffer (two halves) and state words are plain device buffers, and
every rank's "peer pointers" are the same local buffers.  Per call, rank 0's
and then rank 1's exl3cu_mul_mat_peers run in stream order (each stores its
slice into both ranks' buffers and publishes its epoch), and only then do the
two exl3cu_wait_peers run.  Every word they wait for was stored by a kernel
that already finished, so no kernel waits on another kernel running at the
same time.  The calls cover the fused GEMV (1 and 4 rows: its epilogue stores to
the peers), the fused tensor-core GEMM (8 rows) and the operator followed by
exl3cu_store_peers (3 rows); consecutive calls use both halves of the
double-buffered y.  Each rank's output is checked
bit for bit against the 1-GPU operator on the same slice, and the epoch
counters and tickets are checked after the calls.
"""
import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def test_two_ranks_on_one_gpu_fused_and_fallback(cuda_lib, oracle):
    from exl3_b200 import _lib, synthetic
    from exl3_b200.ops import Exl3Weight

    L = _lib.lib()
    k, n, bits, world, max_rows = 2048, 1024, 4, 2, 8
    m = synthetic.matrix(k, n, bits, seed=71)
    trellis, suh, svh = m.trellis, m.suh, m.svh
    count = n // 128 // world
    ws = [Exl3Weight.from_trellis(trellis, suh, svh, device=0, first_block=r * count, block_count=count)
          for r in range(world)]
    half = max_rows * n
    ys = [torch.zeros(2 * half, dtype=torch.int64, device="cuda") for _ in range(world)]  # (epoch, value) words
    states = [torch.zeros(16, dtype=torch.int32, device="cuda") for _ in range(world)]
    yp = (ctypes.c_void_p * world)(*[y.data_ptr() for y in ys])
    slices = [torch.empty((max_rows, count * 128), dtype=torch.float32, device="cuda") for _ in range(world)]
    outs = [torch.empty((max_rows, n), dtype=torch.float32, device="cuda") for _ in range(world)]
    st = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    calls = 0
    for rows, fused in ((1, True), (4, True), (8, True), (3, False), (1, True)):
        x = torch.from_numpy(synthetic.activations(rows, k, seed=72 + rows)).cuda()
        for r in range(world):
            if fused:
                _lib.check(L.exl3cu_mul_mat_peers(ws[r].handle, x.data_ptr(), _lib.F16, rows, k,
                                                  slices[r].data_ptr(), count * 128, world, yp, n, half,
                                                  r * count * 128, states[r].data_ptr(), st))
            else:
                ws[r].mul_mat(x, out=slices[r][:rows])
                _lib.check(L.exl3cu_store_peers(slices[r].data_ptr(), rows, count * 128, count * 128, world, yp, n,
                                                half, r * count * 128, states[r].data_ptr(), st))
        for r in range(world):
            outs[r].fill_(float("nan"))
            _lib.check(L.exl3cu_wait_peers(states[r].data_ptr(), ys[r].data_ptr(), n, half, outs[r].data_ptr(), n,
                                           rows, n, st))
        calls += 1
        torch.cuda.synchronize()
        want = torch.cat([w.mul_mat(x) for w in ws], dim=1)
        for r in range(world):
            assert torch.equal(outs[r][:rows], want), (rows, r)
        ref = oracle.mul_mat(m.records(), bits, k, n, x.cpu().numpy())
        got = outs[0][:rows].cpu().numpy()
        assert np.max(np.abs(got - ref)) / np.max(np.abs(ref)) <= 2e-3
    st_words = [s.cpu().numpy() for s in states]
    for r in range(world):
        assert st_words[r][8] == 0      # the wait kernel's arrival ticket reset itself
        assert st_words[r][9] == calls  # this rank's epoch counter
    status = ctypes.c_uint(0)
    _lib.check(L.exl3cu_device_status(0, ctypes.byref(status), 1))
    assert status.value == 0
    for w in ws:
        w.free()


def test_peer_entries_reject_host_pointers(cuda_lib):
    """The exchange's entries validate their buffers on the host: a host pointer where device memory
    belongs is refused with EXL3CU_INVALID_ARGUMENT before anything is launched."""
    import numpy as np

    from exl3_b200 import _lib

    L = _lib.lib()
    host_state = np.zeros(16, np.uint32)
    y = torch.zeros(2 * 8 * 128, dtype=torch.int64, device="cuda")
    out = torch.zeros((8, 128), dtype=torch.float32, device="cuda")
    st = torch.cuda.current_stream().cuda_stream
    rc = L.exl3cu_wait_peers(host_state.ctypes.data, y.data_ptr(), 128, 8 * 128, out.data_ptr(), 128, 1, 128, st)
    assert rc == _lib.INVALID_ARGUMENT
    assert b"state" in L.exl3cu_last_error()
    slice_ = torch.zeros((1, 128), dtype=torch.float32, device="cuda")
    host_y = np.zeros(2 * 8 * 128, np.int64)
    yp = (ctypes.c_void_p * 1)(host_y.ctypes.data)
    state = torch.zeros(16, dtype=torch.int32, device="cuda")
    rc = L.exl3cu_store_peers(slice_.data_ptr(), 1, 128, 128, 1, yp, 128, 8 * 128, 0, state.data_ptr(), st)
    assert rc == _lib.INVALID_ARGUMENT
    assert b"peer" in L.exl3cu_last_error()
    torch.cuda.synchronize()
