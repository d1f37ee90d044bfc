"""A bounded wait that runs out, on one GPU, without a fault.

exl3cu_wait_peers holds its stream until every rank's epoch flag has reached
this rank's epoch.  Here rank 1's flag is one call behind and nothing ever
raises it: the wait must give up after its bound (about a second), set bit 0
(a bounded wait ran out) in exl3cu_device_status, still finish its copy, and
leave the context usable -- the next call, with the flag raised, returns at
once with a clean status and the finished half of y.  The flag is an ordinary
device word set from the host; no GPU is made to fault, trap or hang.
"""
import ctypes
import time

import pytest
import torch

pytestmark = pytest.mark.gpu

EPOCH_WORD = 9  # the state words: [0, 8) every rank's epoch, [8] store ticket, [9] this rank's counter


def _wait(L, state, y, out, rows, cols):
    st = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    return L.exl3cu_wait_peers(ctypes.c_void_p(state.data_ptr()), 2, ctypes.c_void_p(y.data_ptr()), cols, rows * cols,
                               ctypes.c_void_p(out.data_ptr()), cols, rows, cols, st)


def test_peer_wait_times_out_sets_status_and_context_survives(cuda_lib):
    from exl3_b200 import _lib, ops

    L = _lib.lib()
    rows, cols = 2, 8
    ops.device_status(0, clear=True)
    state = torch.zeros(16, dtype=torch.int32, device="cuda")
    state[EPOCH_WORD] = 5   # this rank is at epoch 5
    state[0] = 5            # its own flag is up to date
    state[1] = 4            # rank 1 is one call behind and nothing will raise it
    y = torch.arange(2 * rows * cols, dtype=torch.float32, device="cuda").view(2, rows, cols)
    out = torch.full((rows, cols), -1.0, dtype=torch.float32, device="cuda")
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    _lib.check(_wait(L, state, y, out, rows, cols))
    torch.cuda.synchronize()
    waited = time.perf_counter() - t0
    assert ops.device_status(0, clear=True) & 1, "the wait ran out: bit 0 must be set"
    assert waited < 10.0, waited
    # the context is intact: the same call with the flag raised returns the odd (epoch 5) half at once
    state[1] = 5
    out.fill_(-1.0)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    _lib.check(_wait(L, state, y, out, rows, cols))
    torch.cuda.synchronize()
    assert time.perf_counter() - t0 < waited
    assert ops.device_status(0, clear=True) == 0
    assert torch.equal(out, y[1])
    # a rank one call ahead (flag at epoch 6) also satisfies the wait
    state[1] = 6
    _lib.check(_wait(L, state, y, out, rows, cols))
    assert ops.device_status(0, clear=True) == 0
