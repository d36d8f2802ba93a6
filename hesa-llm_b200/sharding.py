"""Row sharding of the quantized matvec over the GPUs of one node.

Output rows of y = W x are independent: rank r holds the contiguous rows
[r0, r1) of W (packed GGUF rows, balanced to one row, the same split the strip
kernel uses between its CTAs), computes y[r0:r1], and the full y is
all-gathered so every rank holds it. NCCL's all_gather_into_tensor wants equal
sizes, so every rank contributes a slot of ceil(n_out / world) rows and the
gathered buffer is compacted back to n_out rows with one index_select (a no-op
view when world divides n_out).
"""
from __future__ import annotations


def row_range(n_out: int, rank: int, world: int) -> tuple[int, int]:
    """Rows [r0, r1) of rank `rank`: floor(rank * n_out / world) .. for rank + 1."""
    if world < 1 or not 0 <= rank < world or n_out < 0:
        raise ValueError(f"bad shard: n_out={n_out} rank={rank} world={world}")
    return rank * n_out // world, (rank + 1) * n_out // world


def slot_rows(n_out: int, world: int) -> int:
    """Rows of every rank's slot in the gathered buffer."""
    return -(-n_out // world)


class ShardedQMatvec:
    """y = scale * W x with W's rows split over the ranks of `group`.

    w_rows: this rank's packed rows [r1 - r0, row_bytes] (see row_range).
    local: optional f(w_rows, x, y_slot) computing this rank's rows into
    y_slot[: r1 - r0]; the default is this library's CUDA matvec. It exists
    so the sharding and the gather can run on CPU ranks in tests.
    """

    def __init__(self, qtype: int, w_rows, n_out: int, k: int, rank: int, world: int, group=None,
                 device=None, local=None):
        import torch
        self.qtype, self.n_out, self.k, self.rank, self.world, self.group = qtype, n_out, k, rank, world, group
        self.r0, self.r1 = row_range(n_out, rank, world)
        if w_rows.shape[0] != self.r1 - self.r0:
            raise ValueError(f"rank {rank} holds {w_rows.shape[0]} rows, its shard has {self.r1 - self.r0}")
        self.w = w_rows
        self.device = device or w_rows.device
        self.slot = slot_rows(n_out, world)
        self.y_slot = torch.zeros(self.slot, dtype=torch.float32, device=self.device)
        self.y_all = torch.empty(world * self.slot, dtype=torch.float32, device=self.device)
        if world * self.slot == n_out:
            self.index = None
        else:
            idx = [r * self.slot + i for r in range(world) for i in range(row_range(n_out, r, world)[1]
                                                                            - row_range(n_out, r, world)[0])]
            self.index = torch.tensor(idx, dtype=torch.int64, device=self.device)
        self.local = local or self._cuda_local
        self.workspace = None

    def _cuda_local(self, w_rows, x, y):
        import hesa_cuda as H
        n = w_rows.shape[0]
        if n == 0:
            return
        if self.workspace is None:
            self.workspace = H.make_workspace(self.qtype, n, self.k, device=self.device)
        H.qmatvec(self.qtype, w_rows, x, y=y[:n], workspace=self.workspace)

    def __call__(self, x, scale: float = 1.0):
        import torch.distributed as dist
        self.local(self.w, x, self.y_slot)
        if scale != 1.0:
            self.y_slot.mul_(scale)
        dist.all_gather_into_tensor(self.y_all, self.y_slot, group=self.group)
        return self.y_all if self.index is None else self.y_all.index_select(0, self.index)
