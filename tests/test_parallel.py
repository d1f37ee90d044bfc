"""Multi-rank logic of the column split, on CPU: world_size 2 and 3 gloo ranks, the
oracle standing in for each rank's local EXL3 slice.  Checks the block ranges,
the padded all-gather and the reassembly against the single-process oracle
output; plus the replicas-only contract of the decode benchmark."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_column_split_ranges():
    from exl3_b200.parallel import ColumnSplit

    s = ColumnSplit(4096, 8)
    assert [s.range(r) for r in range(8)] == [(4 * r, 4) for r in range(8)]
    s = ColumnSplit(128 * 7, 3)
    assert [s.range(r) for r in range(3)] == [(0, 3), (3, 2), (5, 2)]
    assert s.max_blocks == 3
    covered = sorted(b for r in range(3) for b in range(s.range(r)[0], sum(s.range(r))))
    assert covered == list(range(7))
    with pytest.raises(ValueError):
        ColumnSplit(100, 2)
    with pytest.raises(ValueError):
        ColumnSplit(256, 3)


def _worker(rank, world, port, k, n, bits, rows, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        import sys
        from pathlib import Path

        root = Path(__file__).resolve().parents[1]
        sys.path[:0] = [str(root), str(root / "xiaomi-hexagon-exl3_b200"), str(root / "tests" / "golden")]
        from exl3_b200 import synthetic
        from exl3_b200.format import pack_records, unpack_records
        from exl3_b200.parallel import ColumnSplit, gather_columns
        from oracle.oracle import Oracle

        orc = Oracle()
        m = synthetic.matrix(k, n, bits, seed=77)
        rec = pack_records(m.trellis, m.suh, m.svh, bits)
        x = synthetic.activations(rows, k, seed=78)
        split = ColumnSplit(n, world)
        first, count = split.range(rank)
        # this rank's share of the records: column blocks [first, first+count)
        tr, su, sv = unpack_records(rec, k, n, bits)
        part = tr[:, first * 8:(first + count) * 8, :]
        rec_local = pack_records(part, su, sv[first * 128:(first + count) * 128], bits)
        y_local = orc.mul_mat(rec_local, bits, k, count * 128, x)
        full = orc.mul_mat(rec, bits, k, n, x)
        y32 = gather_columns(torch.from_numpy(y_local), split)  # fp32 by default: exact
        y16 = gather_columns(torch.from_numpy(y_local), split, dtype=torch.float16)
        e32 = float(np.max(np.abs(y32.numpy() - full)))
        e16 = float(np.max(np.abs(y16.float().numpy() - full.astype(np.float16).astype(np.float32))))
        q.put((rank, max(e32, e16), y32.dtype == torch.float32))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,n", [(2, 512), (3, 896)])
def test_column_split_gather_matches_single_process(world, n):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, 256, n, 4, 3, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    results = sorted(q.get(timeout=10) for _ in range(world))
    assert [r for r, _, _ in results] == list(range(world))
    for _, err, is32 in results:
        assert is32  # the default gather keeps the operator's fp32 output
        assert err == 0.0  # every rank rebuilds the exact fp32 (and, on request, fp16) single-process output
