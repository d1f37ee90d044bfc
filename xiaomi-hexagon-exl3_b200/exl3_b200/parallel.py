"""Multi-GPU execution of the EXL3 operator.

Two layouts, both one process per GPU over torch.distributed:

* **Replicas** (the decode sweep and the model): every rank holds all weights
  and serves its own requests; no collective on the data path.
* **Column split** (the large-matrix configuration): output column blocks of
  128 are dealt to ranks in contiguous ranges; each rank uploads only its
  blocks (``Exl3Weight.from_records(..., first_block, block_count)``) and
  computes its slice of y; one all-gather of the fp16 slices rebuilds y on
  every rank.  The epilogue's H128 and sv act inside a 128-column block, so a
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


def gather_columns(y_local: torch.Tensor, split: ColumnSplit, group=None) -> torch.Tensor:
    """All-gather fp16 column slices [rows, 128*count_r] into y [rows, n] on every rank.

    Uneven shares are padded to the largest so one collective moves them; on NCCL that
    is a single all_gather_into_tensor of [world, rows, 128*max_blocks].  With one rank
    (or no process group) the slice already is y."""
    rows = y_local.shape[0]
    if split.world == 1 or not dist.is_initialized():
        return y_local.to(torch.float16)
    width = 128 * split.max_blocks
    even = split.blocks % split.world == 0
    if even:
        send = y_local.to(torch.float16)
    else:
        send = torch.zeros((rows, width), dtype=torch.float16, device=y_local.device)
        send[:, : y_local.shape[1]] = y_local.to(torch.float16)
    if dist.get_backend(group) == "nccl":
        recv = torch.empty((split.world, rows, width), dtype=torch.float16, device=y_local.device)
        dist.all_gather_into_tensor(recv, send.contiguous(), group=group)
        if even:  # rank-major slices are y's column blocks in order
            return recv.permute(1, 0, 2).reshape(rows, split.n)
        parts = list(recv.unbind(0))
    else:
        parts = [torch.empty_like(send) for _ in range(split.world)]
        dist.all_gather(parts, send.contiguous(), group=group)
    out = torch.empty((rows, split.n), dtype=torch.float16, device=y_local.device)
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

    def forward(self, x: torch.Tensor, stream=None) -> torch.Tensor:
        """y = x . W as fp16 [rows, n] on every rank (local EXL3 slice + one all-gather)."""
        y_local = self.weight.mul_mat(x, stream=stream)
        return gather_columns(y_local, self.split, self.group)

    def free(self):
        self.weight.free()
