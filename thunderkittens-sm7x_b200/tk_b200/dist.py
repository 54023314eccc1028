"""Multi-GPU layer of the hot path: one process per GPU, work split with no
data-path collective, NCCL all-gather only when a gathered output is requested.

The path shards naturally:
  * GEMM by M row blocks: rank r computes rows [r0, r1) of C from the same rows of
    A and all of B (B replicated);
  * attention by (batch, head): rank r owns a contiguous range of the flattened
    B*H slices of Q, K, V and out;
  * tile row ops by tile range.
Shards are contiguous and equal up to an alignment unit (GEMM: a 256-row CTA-pair
tile), the last rank taking the remainder, so a gathered output is the rank-order
concatenation of the shards.
"""

from __future__ import annotations


def shard_range(total: int, world: int, rank: int, align: int = 1) -> tuple[int, int]:
    """[start, stop) of `rank`'s contiguous share of `total` units; every shard but the
    last starts and ends on a multiple of `align`."""
    if world <= 0 or not 0 <= rank < world or total < 0 or align <= 0:
        raise ValueError("invalid shard request")
    units = -(-total // align)            # alignment blocks
    per = -(-units // world)              # blocks per rank, last rank short
    start = min(total, rank * per * align)
    stop = min(total, (rank + 1) * per * align)
    return start, stop


def gemm_rows(m: int, world: int, rank: int) -> tuple[int, int]:
    """Row block of C (and A) computed by `rank`: 256-row aligned (CTA-pair tiles),
    16-row granular at the end as the GEMM contract requires."""
    start, stop = shard_range(m, world, rank, align=256)
    return start, stop


def attention_slices(batch: int, heads: int, world: int, rank: int) -> tuple[int, int]:
    """Range of flattened (batch * heads + head) slices owned by `rank`."""
    return shard_range(batch * heads, world, rank)


def tile_range(n_tiles: int, world: int, rank: int) -> tuple[int, int]:
    return shard_range(n_tiles, world, rank)


def gather_shards(local, total_rows: int, world: int, rank: int, rows_of, group=None):
    """All-gather rank-ordered row shards of a tensor whose first dimension is split by
    `rows_of(world, rank) -> (start, stop)`; returns the full [total_rows, ...] tensor on
    every rank. Shards may differ in length (padded to the longest for the collective)."""
    import torch
    import torch.distributed as dist
    sizes = [rows_of(world, r) for r in range(world)]
    longest = max(stop - start for start, stop in sizes)
    shape = (longest,) + tuple(local.shape[1:])
    send = torch.zeros(shape, dtype=local.dtype, device=local.device)
    send[: local.shape[0]] = local
    recv = torch.empty((world * longest,) + tuple(local.shape[1:]), dtype=local.dtype, device=local.device)
    dist.all_gather_into_tensor(recv, send, group=group)
    parts = [recv[r * longest: r * longest + (stop - start)] for r, (start, stop) in enumerate(sizes)]
    out = torch.cat(parts, dim=0)
    assert out.shape[0] == total_rows
    return out


class _DeviceArray:
    """A raw device buffer exposed through __cuda_array_interface__ (torch.as_tensor
    wraps it without copying)."""

    def __init__(self, ptr: int, shape: tuple, typestr: str = "<f4"):
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": typestr, "data": (ptr, False),
                                         "version": 3}


class GatheredBuffer:
    """Every rank's `rows x ld` FP32 gathered output, mapped into every rank's
    process, for tk_gemm_f16_f16_f32_nn_gather (the all-gather fused into the GEMM
    epilogue: each rank's kernel stores its row block straight into all ranks'
    buffers over NVLink). Collective: every rank constructs it with the same shape.
    `ptrs` lists the buffers in rank order (this rank's own allocation at `rank`);
    `tensor()` is a torch view of this rank's buffer."""

    def __init__(self, rows: int, ld: int, group=None):
        import torch.distributed as dist

        import tk_b200
        self.rows, self.ld = rows, ld
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.own, handle = tk_b200.ipc_alloc(rows * ld * 4)
        handles = [None] * self.world
        dist.all_gather_object(handles, handle, group=group)
        self.ptrs = [self.own if r == self.rank else tk_b200.ipc_open(h) for r, h in enumerate(handles)]

    def tensor(self):
        import torch
        return torch.as_tensor(_DeviceArray(self.own, (self.rows, self.ld)), device="cuda")

    def close(self, group=None):
        """Collective: unmaps the peers' buffers, waits until every rank has unmapped
        this rank's, then frees it (an exported allocation must outlive its mappings).
        Call once no rank's kernel writes into the buffers any more."""
        import torch.distributed as dist

        import tk_b200
        if not self.ptrs:
            return
        for r, ptr in enumerate(self.ptrs):
            if r != self.rank:
                tk_b200.ipc_close(ptr)
        dist.barrier(group=group)
        tk_b200.ipc_free(self.own)
        self.ptrs = []
