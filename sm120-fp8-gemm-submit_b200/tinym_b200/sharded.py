"""N-sharded (column-parallel) tiny-M FP8 GEMM over a process group.

One process per GPU.  Rank r owns W rows [start_r, stop_r) -- a contiguous
slab of N, cut at multiples of the 128-row W tile where the split allows --
and computes Y[:, start_r:stop_r] = alpha * X . W_r^T with the single-GPU
kernel.  X (at most 16 x K bytes) and alpha are replicated.  No reduction is
needed (K is not split across GPUs).  Optionally the BF16 slabs are
all-gathered over NCCL into the full Y[M, N] on every rank.

The reference has no multi-GPU code; this wrapper is new (its collective is
the only data exchange, and it moves only M*N*2 bytes).
"""

from __future__ import annotations

from dataclasses import dataclass

TILE = 128


def shard_bounds(n: int, world: int, rank: int, tile: int = TILE) -> tuple[int, int]:
    """Contiguous [start, stop) rows of an N-row W owned by `rank`.

    Whole tiles are dealt out as evenly as possible: the last N_tiles %
    world ranks get one extra tile, so the ragged last tile (if any) lands on
    a rank holding an extra tile and no two slabs differ by more than one
    tile.  If there are fewer tiles than ranks, rows are split evenly instead
    so that every rank gets work.
    """
    if world < 1 or not 0 <= rank < world:
        raise ValueError("bad rank / world size")
    tiles = -(-n // tile)
    if tiles >= world:
        base, extra = divmod(tiles, world)
        first_big = world - extra
        t0 = rank * base + max(0, rank - first_big)
        t1 = t0 + base + (1 if rank >= first_big else 0)
        return min(n, t0 * tile), min(n, t1 * tile)
    base, extra = divmod(n, world)
    r0 = rank * base + min(rank, extra)
    return r0, r0 + base + (1 if rank < extra else 0)


@dataclass
class ShardedFp8Gemm:
    """Holds this rank's W slab and runs the sharded GEMM.

    ``local_gemm(x, w_local, alpha, out)`` computes the local slab; by
    default it is the CUDA kernel through the C ABI (``tinym_b200.gemm``).
    Tests substitute a CPU function to exercise the host logic on gloo.
    """

    w_local: object
    n: int
    start: int
    stop: int
    group: object = None
    local_gemm: object = None

    @classmethod
    def from_full_weight(cls, w_full, group=None, local_gemm=None):
        """Slice this rank's rows out of the full [N, K] weight (model-load
        time, outside any timed region)."""
        import torch.distributed as dist

        world = dist.get_world_size(group) if dist.is_initialized() else 1
        rank = dist.get_rank(group) if dist.is_initialized() else 0
        n = int(w_full.shape[0])
        start, stop = shard_bounds(n, world, rank)
        w_local = w_full[start:stop].contiguous()
        return cls(w_local, n, start, stop, group, local_gemm)

    def _gemm(self, x, alpha, out):
        if self.local_gemm is not None:
            return self.local_gemm(x, self.w_local, alpha, out)
        from . import gemm

        return gemm(x, self.w_local, alpha, out=out)

    def local(self, x, alpha):
        """This rank's Y[:, start:stop] (no communication)."""
        import torch

        m = int(x.shape[0])
        out = torch.empty((m, self.stop - self.start), dtype=torch.bfloat16, device=x.device)
        if self.stop > self.start:
            self._gemm(x, alpha, out)
        return out

    def __call__(self, x, alpha, gather: bool = True):
        """Y[M, N] on every rank (gather=True) or this rank's slab."""
        import torch
        import torch.distributed as dist

        y_loc = self.local(x, alpha)
        if not gather or not dist.is_initialized() or dist.get_world_size(self.group) == 1:
            return y_loc
        world = dist.get_world_size(self.group)
        m = int(x.shape[0])
        bounds = [shard_bounds(self.n, world, r) for r in range(world)]
        width = max(b - a for a, b in bounds)
        # equal-size padded slabs so one all-gather moves everything
        send = torch.zeros((m, width), dtype=torch.bfloat16, device=x.device)
        send[:, : y_loc.shape[1]] = y_loc
        recv = torch.empty((world, m, width), dtype=torch.bfloat16, device=x.device)
        if dist.get_backend(self.group) == "nccl":
            dist.all_gather_into_tensor(recv.view(-1), send.view(-1).contiguous(), group=self.group)
        else:
            dist.all_gather(list(recv.unbind(0)), send, group=self.group)
        y = torch.empty((m, self.n), dtype=torch.bfloat16, device=x.device)
        for r, (a, b) in enumerate(bounds):
            y[:, a:b] = recv[r, :, : b - a]
        return y
