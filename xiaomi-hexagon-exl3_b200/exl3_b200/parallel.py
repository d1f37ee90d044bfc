"""Multi-GPU execution of the EXL3 operator.

Two layouts, both one process per GPU over torch.distributed:

* **Replicas** (the decode sweep and the model): every rank holds all weights
  and serves its own requests; no collective on the data path.
* **Column split** (the large-matrix configuration): output column blocks of
  128 are dealt to ranks in contiguous ranges; each rank uploads only its
  blocks (``Exl3Weight.from_records(..., first_block, block_count)``) and
  computes its slice of y.  Two ways rebuild y on every rank:
  ``ColumnParallelExl3`` runs one NCCL all-gather of the fp32 slices (fp16 on
  request); ``PeerColumnParallelExl3`` stores every slice straight into every
  rank's y over NVLink (CUDA IPC mappings, P2P stores, an epoch flag per rank
  and a bounded wait on the device) -- no collective library on the path.  The epilogue's H128 and sv act inside a 128-column block, so a
  slice needs nothing from the other ranks.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.distributed as dist


@dataclass(frozen=True)
class ColumnSplit:
    """Contiguous ranges of 128-column blocks, as even as possible (the first ranks take one more)."""

    n: int
    world: int

    def __post_init__(self):
        if self.n % 128 or self.n <= 0:
            raise ValueError("n must be a positive multiple of 128")
        if self.world <= 0 or self.world > self.n // 128:
            raise ValueError("need 1 <= world <= n/128 column blocks")

    @property
    def blocks(self) -> int:
        return self.n // 128

    def range(self, rank: int) -> tuple[int, int]:
        """(first_block, block_count) of `rank`."""
        base, extra = divmod(self.blocks, self.world)
        first = rank * base + min(rank, extra)
        return first, base + (1 if rank < extra else 0)

    @property
    def max_blocks(self) -> int:
        return -(-self.blocks // self.world)


def gather_columns(y_local: torch.Tensor, split: ColumnSplit, group=None, dtype=torch.float32) -> torch.Tensor:
    """All-gather column slices [rows, 128*count_r] into y [rows, n] on every rank.

    dtype float32 (the default) keeps the operator's fp32 output bit for bit, as one GPU
    returns it; float16 halves the bytes on the wire and rounds y to fp16 (at most 2^-11
    relative, and |y| beyond 65504 overflows).  Uneven shares are padded to the largest so
    one collective moves them; on NCCL that is a single all_gather_into_tensor of
    [world, rows, 128*max_blocks].  With one rank (or no process group) the slice already
    is y."""
    rows = y_local.shape[0]
    if split.world == 1 or not dist.is_initialized():
        return y_local.to(dtype)
    width = 128 * split.max_blocks
    even = split.blocks % split.world == 0
    if even:
        send = y_local.to(dtype)
    else:
        send = torch.zeros((rows, width), dtype=dtype, device=y_local.device)
        send[:, : y_local.shape[1]] = y_local.to(dtype)
    if dist.get_backend(group) == "nccl":
        recv = torch.empty((split.world, rows, width), dtype=dtype, device=y_local.device)
        dist.all_gather_into_tensor(recv, send.contiguous(), group=group)
        if even:  # rank-major slices are y's column blocks in order
            return recv.permute(1, 0, 2).reshape(rows, split.n)
        parts = list(recv.unbind(0))
    else:
        parts = [torch.empty_like(send) for _ in range(split.world)]
        dist.all_gather(parts, send.contiguous(), group=group)
    out = torch.empty((rows, split.n), dtype=dtype, device=y_local.device)
    for r, part in enumerate(parts):
        first, count = split.range(r)
        out[:, first * 128:(first + count) * 128] = part[:, : count * 128]
    return out


class ColumnParallelExl3:
    """One rank's share of a column-split EXL3 matrix plus the gather that rebuilds y."""

    def __init__(self, records, k: int, n: int, bits: int, group=None, device: int | None = None, codebook: int = 2):
        from .ops import Exl3Weight

        self.group = group
        self.split = ColumnSplit(n, dist.get_world_size(group))
        self.rank = dist.get_rank(group)
        first, count = self.split.range(self.rank)
        dev = torch.cuda.current_device() if device is None else device
        self.weight = Exl3Weight.from_records(records, k, n, bits, codebook=codebook, device=dev, first_block=first,
                                              block_count=count)
        self.k, self.n = k, n

    def forward(self, x: torch.Tensor, stream=None, dtype=torch.float32) -> torch.Tensor:
        """y = x . W as [rows, n] on every rank (local EXL3 slice + one all-gather); fp32 like the
        single-GPU operator unless dtype=torch.float16 asks for the half-size gather."""
        y_local = self.weight.mul_mat(x, stream=stream)
        return gather_columns(y_local, self.split, self.group, dtype=dtype)

    def free(self):
        self.weight.free()


class PeerColumnParallelExl3:
    """configs[4]'s column split with the all-gather done over NVLink peer memory (no collective
    library on the data path).  Every rank owns a y buffer of (epoch << 32 | float bits) words, two
    halves of max_rows x n, which every other rank maps through CUDA IPC, and 16 state words (its epoch
    counter).  forward(): exl3cu_mul_mat_peers computes the rank's slice and stores it as (epoch,
    value) words into every rank's buffer -- for 1..4 rows inside the GEMV's epilogue, one launch --
    and exl3cu_wait_peers holds the stream until every word of this call has arrived, copies the row
    into a fixed output and advances the counter.  The epoch lives on the device, so forward() can be
    captured in a CUDA graph and replayed.  The returned tensor is a view of the fixed output, valid
    until the next call.

    The (epoch, value) words double the bytes on the wire, which is the right trade while the call
    is latency-bound: with 2 GPUs, 1 row took 18.4 us this way against 23.4 us with the NCCL
    all-gather, and 8 rows 29.7 against 40.2 us.  At 512 rows the NVLink bytes dominate (102 against
    88 us), so calls of more than `pair_words` words per rank (rows x n) gather the slices with NCCL
    instead (gather_columns)."""

    pair_words = 1 << 18  # rows x n above which forward() gathers with NCCL: 64 rows of 4096

    def __init__(self, records, k: int, n: int, bits: int, max_rows: int, group=None, device: int | None = None,
                 codebook: int = 2, weight=None):
        import ctypes

        from . import _lib
        from .ops import Exl3Weight

        self.L = _lib.lib()
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if self.world > 8:
            raise ValueError("the peer exchange serves up to 8 ranks")
        self.split = ColumnSplit(n, self.world)
        first, count = self.split.range(self.rank)
        self.first, self.count = first, count
        self.dev = torch.cuda.current_device() if device is None else device
        # `weight`: an existing handle of this rank's column blocks, used as is and not freed here
        self.owns_weight = weight is None
        self.weight = weight if weight is not None else Exl3Weight.from_records(
            records, k, n, bits, codebook=codebook, device=self.dev, first_block=first, block_count=count)
        self.k, self.n, self.max_rows = k, n, max_rows
        self.half = max_rows * n  # words between the two halves of y
        c = ctypes
        y_ptr = c.c_void_p()
        y_h = (c.c_char * 64)()
        _lib.check(self.L.exl3cu_ipc_alloc(self.dev, 2 * self.half * 8, c.byref(y_ptr), y_h))  # 8-byte words
        self.y_own = y_ptr.value
        self.state = torch.zeros(16, dtype=torch.int32, device=f"cuda:{self.dev}")  # read and advanced locally
        handles = [None] * self.world
        dist.all_gather_object(handles, bytes(y_h), group=group)
        self.y_peers, self.opened = [], []
        for r, yh in enumerate(handles):
            if r == self.rank:
                self.y_peers.append(self.y_own)
                continue
            yp = c.c_void_p()
            _lib.check(self.L.exl3cu_ipc_open(self.dev, c.create_string_buffer(yh, 64), c.byref(yp)))
            self.y_peers.append(yp.value)
            self.opened.append(yp.value)
        dist.barrier(group=group)  # every rank has mapped every buffer before any store
        self._yp = (c.c_void_p * self.world)(*self.y_peers)
        self.slice = torch.empty((max_rows, count * 128), dtype=torch.float32, device=f"cuda:{self.dev}")
        self.out = torch.empty((max_rows, n), dtype=torch.float32, device=f"cuda:{self.dev}")

    def forward(self, x: torch.Tensor, stream=None) -> torch.Tensor:
        """y = x . W as fp32 [rows, n] on every rank, the slices exchanged over peer memory."""
        import ctypes

        from . import _lib
        from .ops import _stream_handle

        rows = x.shape[0]
        if rows > self.max_rows:
            raise ValueError(f"{rows} rows > max_rows {self.max_rows}")
        if x.dtype not in (torch.float32, torch.float16):
            raise TypeError("x must be float32 or float16")
        x = x if x.stride(-1) == 1 else x.contiguous()
        if rows * self.n > self.pair_words:  # bandwidth-bound: the collective library's all-gather
            y_local = self.weight.mul_mat(x, out=self.slice[:rows], stream=stream)
            with torch.cuda.stream(stream or torch.cuda.current_stream()):
                return gather_columns(y_local, self.split, self.group)
        sh = _stream_handle(stream)
        cols = self.count * 128
        # the slice's operator and its all-gather: one launch for 1..4 rows (the GEMV stores its output
        # blocks into every rank's buffer), else the operator into self.slice plus the peer stores
        _lib.check(self.L.exl3cu_mul_mat_peers(self.weight.handle, x.data_ptr(), _lib.F32 if x.dtype == torch.float32
                                               else _lib.F16, rows, x.stride(0), self.slice.data_ptr(), cols,
                                               self.world, self._yp, self.n, self.half, self.first * 128,
                                               self.state.data_ptr(), sh))
        _lib.check(self.L.exl3cu_wait_peers(self.state.data_ptr(), ctypes.c_void_p(self.y_own), self.n, self.half,
                                            self.out.data_ptr(), self.n, rows, self.n, sh))
        return self.out[:rows]

    def free(self):
        torch.cuda.synchronize(self.dev)
        dist.barrier(group=self.group)  # no rank still stores into another's buffers
        for p in self.opened:
            self.L.exl3cu_ipc_close(self.dev, p)
        dist.barrier(group=self.group)
        self.L.exl3cu_ipc_free(self.dev, self.y_own)
        if self.owns_weight:
            self.weight.free()
