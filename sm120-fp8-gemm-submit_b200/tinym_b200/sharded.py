"""N-sharded (column-parallel) tiny-M FP8 GEMM over a process group.

One process per GPU.  Rank r owns W rows [start_r, stop_r) -- a contiguous
slab of N, cut at multiples of the 128-row W tile where the split allows --
and computes Y[:, start_r:stop_r] = alpha * X . W_r^T with the single-GPU
kernel.  X (at most 16 x K bytes) and alpha are replicated.  No reduction is
needed (K is not split across GPUs).  Optionally the BF16 slabs are
all-gathered into the full Y[M, N] on every rank: over NCCL, or fused into
the GEMM (``enable_fused_gather``): each rank's epilogue stores its rows
straight into every rank's Y through CUDA IPC peer mappings over NVLink and
signals per-rank arrival counters (tinym_fp8_gemm_allgather).

The reference has no multi-GPU code; this wrapper is new (its gather is the
only data exchange, and it moves only M*N*2 bytes).
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

    # ---------------------------------------------------------------- fused gather
    def enable_fused_gather(self, m_max: int = 16, device=None):
        """Set up the fused all-gather: two [m_max, N] BF16 buffers (used
        alternately) and an arrival counter on this rank, exported to and
        mapped by every rank (collective: call on all ranks)."""
        import torch
        import torch.distributed as dist

        from . import GatherDesc, ipc_export, ipc_open

        device = device or torch.device("cuda", torch.cuda.current_device())
        world = dist.get_world_size(self.group)
        rank = dist.get_rank(self.group)
        # Both checks see the same values on every rank, so all ranks refuse
        # together, before the first collective.
        if world > 8:
            raise ValueError("the fused all-gather supports up to 8 ranks")
        if self.n < world:
            raise ValueError(f"the fused all-gather needs N >= world size (N={self.n}, world={world})")
        if not 1 <= m_max <= 16:
            raise ValueError(f"m_max must be in 1..16 (got {m_max})")
        self._ybuf = torch.empty((2, m_max, self.n), dtype=torch.bfloat16, device=device)
        self._counter = torch.zeros(1, dtype=torch.int64, device=device)
        torch.cuda.synchronize(device)
        mine = (ipc_export(self._ybuf.data_ptr()), ipc_export(self._counter.data_ptr()))
        allh = [None] * world
        dist.all_gather_object(allh, mine, group=self.group)
        self._opened = []
        y_ptr, c_ptr = [], []
        for r, ((hy, oy), (hc, oc)) in enumerate(allh):
            if r == rank:
                y_ptr.append(self._ybuf.data_ptr())
                c_ptr.append(self._counter.data_ptr())
                continue
            by = ipc_open(hy)
            self._opened.append(by)
            bc = by if hc == hy else ipc_open(hc)
            if bc != by:
                self._opened.append(bc)
            y_ptr.append(by + oy)
            c_ptr.append(bc + oc)
        self._m_max, self._y_ptr, self._c_ptr = m_max, y_ptr, c_ptr
        self._epoch = 0
        self._arrived = 0  # running sum of M * N over the fused calls so far
        self._world, self._rank = world, rank
        self._desc = GatherDesc()
        self._desc.world, self._desc.rank = world, rank
        self._desc.n_full, self._desc.col0 = self.n, self.start
        for r in range(world):
            self._desc.flag[r] = c_ptr[r]
        dist.barrier(group=self.group)

    def fused(self, x, alpha):
        """Y[M, N] on every rank with the gather fused into the GEMM.  The
        result is a view of one of two internal buffers used alternately.
        Every read of it must be stream-ordered before this rank's next
        fused() call (queued earlier on the same stream, or waited for):
        once this rank's next call has stored its rows, a faster peer's call
        after that may start storing into the buffer returned here."""
        import torch

        from . import gemm_allgather_ptr

        if getattr(self, "_desc", None) is None:
            # the peers' buffers are not mapped: the epilogue must not run
            raise RuntimeError("fused gather is not enabled (enable_fused_gather first)")
        m, k = int(x.shape[0]), int(x.shape[1])
        if m > self._m_max:
            raise ValueError(f"M={m} > m_max={self._m_max}")
        self._epoch += 1
        buf = self._epoch & 1
        plane = self._m_max * self.n * 2  # bytes of one [m_max, N] BF16 buffer
        for r in range(self._world):
            self._desc.y_full[r] = self._y_ptr[r] + buf * plane
        self._arrived += m * self.n
        self._desc.target = self._arrived
        stream = torch.cuda.current_stream(x.device).cuda_stream
        if isinstance(alpha, torch.Tensor):
            gemm_allgather_ptr(x.data_ptr(), self.w_local.data_ptr(), m, self.stop - self.start,
                               k, self._desc, alpha_ptr=alpha.data_ptr(), stream=stream)
        else:
            gemm_allgather_ptr(x.data_ptr(), self.w_local.data_ptr(), m, self.stop - self.start,
                               k, self._desc, alpha=float(alpha), stream=stream)
        return self._ybuf[buf, :m]

    def close_fused_gather(self):
        """Unmap the peers' buffers (collective: call on all ranks)."""
        import torch
        import torch.distributed as dist

        from . import ipc_close

        self._desc = None  # later fused() calls raise instead of storing to unmapped peers
        torch.cuda.synchronize()
        dist.barrier(group=self.group)
        for base in getattr(self, "_opened", []):
            ipc_close(base)
        self._opened = []

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
