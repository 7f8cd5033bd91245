"""Column-sharded (N-split) W4A16 / INT3 projections over torch.distributed.

The reference has no multi-GPU code; this is the one multi-GPU piece the
library adds.  Rank r of a G-rank group holds columns [r*N/G, (r+1)*N/G) of
every packed weight (word columns are sliced; the packed layout is unchanged)
and the matching scale / zero-point columns.  A forward pass runs the
single-GPU kernel on the local columns and gathers the G output slices with
one ``all_gather_into_tensor`` over NCCL (NVLink / NVSwitch on a B200 node).
Several projections that consume the same activation (q/k/v, gate/up) can
share one gather (``ShardedGroup``), which matters at M = 1 where the gather's
latency, not its bytes, dominates.

Collectives are issued in the same order on every rank; no rank skips one.
"""

import torch
import torch.distributed as dist

from . import ops


def shard_bounds(N, rank, world):
    """Column range of ``rank``; N must divide evenly (every Llama projection does)."""
    if N % world:
        raise ValueError(f"N={N} is not divisible by the world size {world}")
    n = N // world
    return rank * n, (rank + 1) * n


def shard_columns(t, rank, world):
    """Columns of a 2-D tensor (packed words, scales or zero points) owned by ``rank``."""
    if t is None:
        return None
    if t.dim() == 1:
        t = t.reshape(1, -1)
    lo, hi = shard_bounds(t.size(1), rank, world)
    return t[:, lo:hi].contiguous()


class ShardedLinear:
    """One column-sharded projection y = x @ dequant(W)."""

    def __init__(self, W_local, scales_local, zero_points_local=None, fmt="s4", group_size=100,
                 process_group=None):
        if fmt not in ("s4", "u4", "s3"):
            raise ValueError("fmt must be 's4', 'u4' or 's3'")
        self.W, self.S, self.Z = W_local, scales_local, zero_points_local
        self.fmt, self.group_size = fmt, group_size
        self.pg = process_group
        self.world = dist.get_world_size(process_group) if dist.is_initialized() else 1
        self.n_local = W_local.size(1)

    @classmethod
    def from_full(cls, W, scales, zero_points=None, fmt="s4", group_size=100, process_group=None):
        world = dist.get_world_size(process_group) if dist.is_initialized() else 1
        rank = dist.get_rank(process_group) if dist.is_initialized() else 0
        return cls(shard_columns(W, rank, world), shard_columns(scales, rank, world),
                   shard_columns(zero_points, rank, world), fmt, group_size, process_group)

    def local(self, x):
        """This rank's [M, N/G] slice of the output."""
        if self.fmt == "s4":
            return ops.fused_w4a16_gemm_s4(x, self.W, self.S, self.Z)
        if self.fmt == "u4":
            return ops.fused_w4a16_gemm_u4(x, self.W, self.S, self.Z)
        z = self.Z if self.Z is not None else torch.empty(0, dtype=torch.float16, device=x.device)
        return ops.fused_h17_gemv_s3(x, self.W, self.S, z, group_size=self.group_size)

    def __call__(self, x):
        return ShardedGroup([self], self.pg)(x)[0]


class ShardedGroup:
    """Projections that read the same activation; their local outputs are
    packed into one buffer and gathered with a single collective."""

    def __init__(self, linears, process_group=None):
        self.linears = list(linears)
        self.pg = process_group
        self.world = dist.get_world_size(process_group) if dist.is_initialized() else 1
        self._graph = None

    def capture_local(self, x):
        """Record this rank's local projections of activation ``x`` and their
        packing as one CUDA graph; a later call with the same ``x`` tensor (an
        activation buffer that stays in place) replays it instead of launching
        each kernel from Python.  The collective stays outside the graph."""
        s = torch.cuda.Stream(x.device)
        s.wait_stream(torch.cuda.current_stream(x.device))
        with torch.cuda.stream(s):
            for _ in range(2):
                self._local_packed(x)
        torch.cuda.current_stream(x.device).wait_stream(s)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            packed, widths = self._local_packed(x)
        self._graph, self._x, self._packed, self._widths = g, x, packed, widths

    def release_graph(self):
        self._graph = self._x = self._packed = None

    def _local_packed(self, x):
        locals_ = [lin.local(x) for lin in self.linears]
        widths = [t.size(1) for t in locals_]
        packed = torch.cat(locals_, dim=1) if len(locals_) > 1 else locals_[0]
        return packed, widths

    def __call__(self, x):
        if self._graph is not None and x is self._x:
            self._graph.replay()
            packed, widths = self._packed, self._widths
        else:
            if self.world == 1:
                return [lin.local(x) for lin in self.linears]
            packed, widths = self._local_packed(x)
        if self.world == 1:
            return [t.clone() for t in _split_columns(packed, widths)]
        M = packed.size(0)
        # gathered flat as [G * M, w] (rank-major), the form every backend
        # accepts for all_gather_into_tensor, then viewed as [G, M, w]
        gathered = torch.empty((self.world * M, packed.size(1)), dtype=packed.dtype, device=packed.device)
        dist.all_gather_into_tensor(gathered, packed.contiguous(), group=self.pg)
        return unpack_gathered(gathered.view(self.world, M, packed.size(1)), widths)


def _split_columns(packed, widths):
    outs, off = [], 0
    for w in widths:
        outs.append(packed[:, off:off + w])
        off += w
    return outs


def unpack_gathered(gathered, widths):
    """[G, M, sum(widths)] rank-major slices -> one [M, G*w] tensor per projection,
    columns in rank order (rank r's slice is columns [r*w, (r+1)*w))."""
    G, M, _ = gathered.shape
    outs, off = [], 0
    for w in widths:
        part = gathered[:, :, off:off + w]                    # [G, M, w]
        outs.append(part.permute(1, 0, 2).reshape(M, G * w))  # a copy only when M > 1 or several parts
        off += w
    return outs
