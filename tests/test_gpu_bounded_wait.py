"""A bounded wait that runs out, on one GPU, without a fault.

exl3cu_wait_peers holds its stream until every word of this call's half of
the rank's y buffer carries this call's epoch (the column split's exchange
protocol: 8-byte words epoch << 32 | float bits).  Here the words carry an
older epoch and nothing will store the new one: the wait must give up after
its bound (about a second), set bit 0 (a bounded wait ran out) in
exl3cu_device_status, still finish its copy and advance the counter, and
leave the context usable -- the next call, whose words are in place, returns
at once with a clean status and the stored values.  The words are ordinary
device memory set from the host; no GPU is made to fault, trap or hang.
"""
import time

import pytest
import torch

pytestmark = pytest.mark.gpu

EPOCH_WORD = 9  # state words: [8] the wait kernel's arrival ticket, [9] this rank's epoch counter


def _words(epoch, values):
    bits = values.contiguous().view(torch.int32).to(torch.int64) & 0xFFFFFFFF
    return (epoch << 32) | bits


def _wait(L, state, y, out, rows, cols):
    return L.exl3cu_wait_peers(state.data_ptr(), y.data_ptr(), cols, rows * cols, out.data_ptr(), cols, rows, cols,
                               torch.cuda.current_stream().cuda_stream)


def test_peer_wait_times_out_sets_status_and_context_survives(cuda_lib):
    from exl3_b200 import _lib, ops

    L = _lib.lib()
    rows, cols = 2, 8
    ops.device_status(0, clear=True)
    state = torch.zeros(16, dtype=torch.int32, device="cuda")
    state[EPOCH_WORD] = 5  # five calls done: this call is epoch 6, half 0
    vals = torch.arange(2 * rows * cols, dtype=torch.float32, device="cuda").view(2, rows, cols)
    y = torch.empty((2, rows, cols), dtype=torch.int64, device="cuda")
    y[0] = _words(5, vals[0])  # an older epoch: nothing will store epoch 6
    y[1] = _words(5, vals[1])
    out = torch.full((rows, cols), -1.0, dtype=torch.float32, device="cuda")
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    _lib.check(_wait(L, state, y, out, rows, cols))
    torch.cuda.synchronize()
    waited = time.perf_counter() - t0
    assert ops.device_status(0, clear=True) & 1, "the wait ran out: bit 0 must be set"
    assert waited < 10.0, waited
    assert int(state[EPOCH_WORD]) == 6 and int(state[8]) == 0  # the call still completed
    # the context is intact: the next call (epoch 7, half 1) finds its words and returns at once
    y[1] = _words(7, vals[1])
    out.fill_(-1.0)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    _lib.check(_wait(L, state, y, out, rows, cols))
    torch.cuda.synchronize()
    assert time.perf_counter() - t0 < waited
    assert ops.device_status(0, clear=True) == 0
    assert torch.equal(out, vals[1])
    assert int(state[EPOCH_WORD]) == 7
