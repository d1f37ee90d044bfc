"""Column-split EXL3 operator on 2+ GPUs over NCCL (configs[4] shape), one process per GPU.

Each rank uploads only its column blocks, runs the CUDA operator on its slice and
rebuilds y on every rank, once through one NCCL all-gather of the fp32 slices and
once through peer memory (NVLink stores and epoch flags); every rank must hold the
same y, within the operator tolerance of the oracle, at batch 1, 8 and 512.  Skipped when fewer than two GPUs are visible."""
import ctypes
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

pytestmark = [pytest.mark.gpu, pytest.mark.multigpu]


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    import sys
    from datetime import timedelta
    from pathlib import Path

    root = Path(__file__).resolve().parents[1]
    sys.path[:0] = [str(root), str(root / "xiaomi-hexagon-exl3_b200")]
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    import torch.distributed as dist

    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60),
                            device_id=torch.device(f"cuda:{rank}"))
    try:
        from exl3_b200 import synthetic
        from exl3_b200.parallel import ColumnParallelExl3
        from oracle.oracle import Oracle

        k, n, bits = 14336, 4096, 4
        m = synthetic.matrix(k, n, bits, seed=44)
        rec = m.records()
        layer = ColumnParallelExl3(rec, k, n, bits, device=rank)
        out = []
        for rows in (1, 8, 512):  # GEMV, grouped GEMV, tcgen05 GEMM
            x = synthetic.activations(rows, k, seed=45 + rows)
            y = layer.forward(torch.from_numpy(x).cuda(rank))  # fp32 gather, as one GPU returns y
            torch.cuda.synchronize(rank)
            y = y.float().cpu().numpy()
            ref = Oracle().mul_mat(rec, bits, k, n, x, nth=8) if rank == 0 else None
            if ref is not None:
                rel = float(np.max(np.abs(y - ref)) / np.max(np.abs(ref)))
                out.append((rows, rel))
            # every rank holds the same gathered y
            t = torch.from_numpy(y).cuda(rank)
            ref0 = t.clone()
            dist.broadcast(ref0, 0)
            out.append((rows, "same", bool(torch.equal(t, ref0))))
        layer.free()
        # the same through peer memory (NVLink stores + epoch flags, no collective library); three calls
        # in a row so that both halves of the double-buffered y are used and reused
        from exl3_b200.parallel import PeerColumnParallelExl3

        peer = PeerColumnParallelExl3(rec, k, n, bits, max_rows=512, device=rank)
        for rows in (1, 8, 512, 1):
            x = synthetic.activations(rows, k, seed=45 + rows)
            y = peer.forward(torch.from_numpy(x).cuda(rank)).clone()
            torch.cuda.synchronize(rank)
            if rank == 0:
                ref = Oracle().mul_mat(rec, bits, k, n, x, nth=8)
                yn = y.cpu().numpy()
                out.append((rows, float(np.max(np.abs(yn - ref)) / np.max(np.abs(ref)))))
            ref0 = y.clone()
            dist.broadcast(ref0, 0)
            out.append((rows, "same", bool(torch.equal(y, ref0))))
        st = ctypes.c_uint(0)
        from exl3_b200 import _lib
        _lib.check(_lib.lib().exl3cu_device_status(rank, ctypes.byref(st), 1))
        out.append((0, "status", int(st.value)))
        peer.free()
        q.put((rank, out))
    finally:
        dist.destroy_process_group()


def test_column_parallel_nccl():
    world = torch.cuda.device_count() if torch.cuda.is_available() else 0
    if world < 2:
        pytest.skip("needs two or more GPUs")
    world = min(world, 8)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    for _ in range(world):
        rank, out = q.get(timeout=300)
        results[rank] = out
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    for rank, out in results.items():
        for item in out:
            if item[1] == "status":
                assert item[2] == 0, f"rank {rank}: device status {item[2]:#x} (a peer wait ran out)"
            elif item[1] == "same":
                assert item[2], f"rank {rank} rows {item[0]}: gathered y differs from rank 0"
            else:
                assert item[1] <= 2e-3, f"rows {item[0]}: max_abs_rel {item[1]}"
