"""Column-sharded (N-split) W4A16 / INT3 projections over torch.distributed.

The reference has no multi-GPU code; this is the one multi-GPU piece the
library adds.  Rank r of a G-rank group holds columns [r*N/G, (r+1)*N/G) of
every packed weight (word columns are sliced; the packed layout is unchanged)
and the matching scale / zero-point columns.  A forward pass runs the
single-GPU kernel on the local columns and gathers the G output slices:
  * ``P2PGatherGroup``: the decode kernel stores its columns straight into
    every rank's receive buffer over NVLink, and a group's last launch ends
    once every rank's columns have arrived -- no collective call, so a whole
    step can be one CUDA graph;
  * ``ShardedGroup``: one ``all_gather_into_tensor`` (NCCL on GPUs) after the
    local kernels, for any shape and format.
Several projections that consume the same activation (q/k/v, gate/up) share
one gather, which matters at M = 1 where the gather's latency, not its bytes,
dominates.

Collectives are issued in the same order on every rank; no rank skips one.
"""

import ctypes

import torch
import torch.distributed as dist

from . import _lib, ops


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
        self._grouped = _grouped_args(self.linears)

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

    def _local_list(self, x):
        """This rank's outputs of every projection: one grouped call
        (ops.fused_w4a16_gemm_grouped) where the group allows it, else one
        call per projection (and for CPU tensors, which the ops reject as
        each projection's call does)."""
        if self._grouped is not None and x.is_cuda:
            return ops.fused_w4a16_gemm_grouped(x, *self._grouped)
        return [lin.local(x) for lin in self.linears]

    def _local_packed(self, x):
        locals_ = self._local_list(x)
        widths = [t.size(1) for t in locals_]
        packed = torch.cat(locals_, dim=1) if len(locals_) > 1 else locals_[0]
        return packed, widths

    def __call__(self, x):
        if self._graph is not None and x is self._x:
            self._graph.replay()
            packed, widths = self._packed, self._widths
        else:
            if self.world == 1:
                return self._local_list(x)
            packed, widths = self._local_packed(x)
        if self.world == 1:
            return [t.clone() for t in _split_columns(packed, widths)]
        M = packed.size(0)
        # gathered flat as [G * M, w] (rank-major), the form every backend
        # accepts for all_gather_into_tensor, then viewed as [G, M, w]
        gathered = torch.empty((self.world * M, packed.size(1)), dtype=packed.dtype, device=packed.device)
        dist.all_gather_into_tensor(gathered, packed.contiguous(), group=self.pg)
        return unpack_gathered(gathered.view(self.world, M, packed.size(1)), widths)


def _grouped_args(linears):
    """(W list, scales list, zero points list or None, signed) for one
    grouped call of these projections, or None when they do not form one:
    fewer than two, more than ops.GROUPED_MAX, not all s4 or all u4, or with
    different K, group sizes or presence of zero points."""
    if not 2 <= len(linears) <= ops.GROUPED_MAX:
        return None
    fmts = {lin.fmt for lin in linears}
    if fmts not in ({"s4"}, {"u4"}):
        return None
    def group_rows(t):
        return t.size(0) if t.dim() == 2 else 1
    if len({lin.W.size(0) for lin in linears}) != 1 or len({group_rows(lin.S) for lin in linears}) != 1:
        return None
    has_zp = [lin.Z is not None and lin.Z.numel() > 0 for lin in linears]
    if any(h != has_zp[0] for h in has_zp):
        return None
    Zs = [lin.Z for lin in linears] if has_zp[0] else None
    return [lin.W for lin in linears], [lin.S for lin in linears], Zs, fmts == {"s4"}


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


# ---------------------------------------------------------------- fused gather
def column_offsets(widths, world):
    """Start column of each projection in a group buffer: projection i holds
    world * widths[i] columns, rank r's slice at offset + r * widths[i]."""
    offs, off = [], 0
    for w in widths:
        offs.append(off)
        off += world * w
    return offs, off


class P2PGatherGroup:
    """Column-sharded projections that read the same activation, gathered by
    the decode kernel itself instead of a collective: each rank's GEMV stores
    its column pairs, tagged with the call's epoch, straight into every rank's
    receive buffer (peer memory over NVLink, mapped with CUDA IPC); the
    group's last launch polls this rank's receive buffer until the whole group
    has arrived and writes the local output (bounded waits; see
    t4b_fused_w4a16_gemv_allgather).  With no collective call in it, a step
    made of these groups can be captured as one CUDA graph.

    M and the projections' tensors are fixed (the buffers are allocated once,
    and the launches of a call are tabled at construction).  The outputs are
    views of this rank's output buffer, written only by this rank's own calls,
    and are overwritten by the group's next call.  Every rank must create its groups
    in the same order and call them in the same order.  Raises RuntimeError
    when the decode kernel does not take a shape (use ShardedGroup, the NCCL
    path, then).  With ``grouped`` (the default) a group of projections that
    one grouped launch takes (t4b_fused_w4a16_gemv_allgather_grouped: all s4
    or all u4, the same K and group size) is called as that one launch
    instead of one launch per projection."""

    def __init__(self, linears, M, process_group=None, grouped=True):
        self.linears = list(linears)
        self.pg = process_group
        self.world = dist.get_world_size(process_group)
        self.rank = dist.get_rank(process_group)
        if not 2 <= self.world <= 8:
            raise ValueError("the fused gather serves 2 to 8 ranks")
        if any(lin.fmt not in ("s4", "u4") for lin in self.linears):
            raise ValueError("the fused gather serves the W4A16 projections")
        self.M = M
        self.widths = [lin.n_local for lin in self.linears]
        if any(w % 2 for w in self.widths):
            raise ValueError("the fused gather moves column pairs: every shard width must be even")
        self.offsets, self.n_total = column_offsets(self.widths, self.world)
        self.device = self.linears[0].W.device
        lib = _lib.load()
        self._lib = lib
        with torch.cuda.device(self.device):
            for lin in self.linears:
                K = lin.W.size(0) * 8
                groups = lin.S.size(0) if lin.S.dim() == 2 else 1
                st = lib.t4b_fused_w4a16_gemv_allgather_supported(
                    M, lin.n_local, K, K // groups, int(lin.Z is not None and lin.Z.numel() > 0))
                if st:
                    raise RuntimeError(f"the fused gather does not take M={M}, K={K}, N={lin.n_local} "
                                       f"({lib.t4b_status_string(st).decode()}); use ShardedGroup")
        self._own, self._opened = [], []
        self.out = torch.empty((M, self.n_total), dtype=torch.float16, device=self.device)
        self.counter = torch.zeros(2, dtype=torch.int32, device=self.device)
        with torch.cuda.device(self.device):
            # receive buffer: two halves (epoch parity) of M x n_total/2 64-bit words
            recv_ptr = self._alloc(M * self.n_total * 8)
            everyone = [None] * self.world
            dist.all_gather_object(everyone, self._handle(recv_ptr), group=process_group)
            recv = [recv_ptr if g == self.rank else self._open(everyone[g]) for g in range(self.world)]
        self._grouped = None
        if grouped:
            args = _grouped_args(self.linears)
            if args is not None:
                lin0 = self.linears[0]
                K = lin0.W.size(0) * 8
                groups = lin0.S.size(0) if lin0.S.dim() == 2 else 1
                if ops.grouped_plan(self.widths, M, K, K // groups, args[2] is not None) is not None:
                    self._grouped = args
        self._gathers = []
        for i in range(len(self.linears)):
            g = _lib.T4BGather()
            for r in range(self.world):
                g.recv[r] = recv[r]
            g.out = self.out.data_ptr()
            g.counter = self.counter.data_ptr()
            g.world, g.rank, g.n_total = self.world, self.rank, self.n_total
            g.col_offset = self.offsets[i] + self.rank * self.widths[i]
            g.barrier = 1 if i == len(self.linears) - 1 else 0
            self._gathers.append(g)
        # every call returns the same views of the output buffer; the torch
        # binding, when built, issues a call's launches from this table
        self._views = [self.out[:, off:off + self.world * w] for off, w in zip(self.offsets, self.widths)]
        rows = []
        for lin, g in zip(self.linears, self._gathers):
            K = lin.W.size(0) * 8
            S = lin.S if lin.S.dim() == 2 else lin.S.reshape(1, -1)
            Z = lin.Z.data_ptr() if lin.Z is not None and lin.Z.numel() else 0
            rows.append([lin.W.data_ptr(), S.data_ptr(), Z, lin.n_local, K, K // S.size(0),
                         1 if lin.fmt == "s4" else 0, ctypes.addressof(g)])
        self._table = torch.tensor(rows, dtype=torch.int64)
        if self._grouped is not None:
            # one launch for the group: the last projection's descriptor
            # (barrier = 1) with every projection's column offset
            self._col_offsets = [g.col_offset for g in self._gathers]
            self._table = torch.tensor([r[:7] + [ctypes.addressof(self._gathers[-1]), off]
                                        for r, off in zip(rows, self._col_offsets)], dtype=torch.int64)
        self._bind = ops._binding()

    def _alloc(self, nbytes):
        p = ctypes.c_void_p()
        _lib.check(self._lib.t4b_ipc_alloc(nbytes, ctypes.byref(p)), "t4b_ipc_alloc")
        self._own.append(p.value)
        return p.value

    def _handle(self, ptr):
        buf = ctypes.create_string_buffer(64)
        _lib.check(self._lib.t4b_ipc_handle(ptr, buf), "t4b_ipc_handle")
        return buf.raw

    def _open(self, handle):
        buf = ctypes.create_string_buffer(handle, 64)
        p = ctypes.c_void_p()
        _lib.check(self._lib.t4b_ipc_open(buf, ctypes.byref(p)), "t4b_ipc_open")
        self._opened.append(p.value)
        return p.value

    def __call__(self, x):
        if self._bind is not None:
            if self._grouped is not None:
                self._bind.allgather_grouped(x, self._table, self.M)
            else:
                self._bind.allgather_group(x, self._table, self.M)
            return self._views
        if x.size(0) != self.M or x.dtype != torch.float16 or not x.is_contiguous():
            raise RuntimeError(f"the fused gather group takes contiguous fp16 activations of {self.M} rows")
        stream = torch._C._cuda_getCurrentRawStream(self.device.index)
        if self._grouped is not None:
            r = self._table.tolist()
            n = len(r)
            vp = ctypes.c_void_p * n
            st = self._lib.t4b_fused_w4a16_gemv_allgather_grouped(
                x.data_ptr(), n, vp(*[q[0] for q in r]), vp(*[q[1] for q in r]),
                vp(*[q[2] for q in r]) if r[0][2] else None, (ctypes.c_int * n)(*[q[3] for q in r]),
                (ctypes.c_int * n)(*[q[8] for q in r]), self.M, r[0][4], r[0][5], r[0][6],
                ctypes.byref(self._gathers[-1]), stream)
            if st:
                _lib.check(st, "t4b_fused_w4a16_gemv_allgather_grouped")
            return self._views
        fn = self._lib.t4b_fused_w4a16_gemv_allgather
        for lin, g in zip(self.linears, self._gathers):
            K = lin.W.size(0) * 8
            S = lin.S if lin.S.dim() == 2 else lin.S.reshape(1, -1)
            Z = lin.Z.data_ptr() if lin.Z is not None and lin.Z.numel() else None
            st = fn(x.data_ptr(), lin.W.data_ptr(), S.data_ptr(), Z, self.M, lin.n_local, K, K // S.size(0),
                    1 if lin.fmt == "s4" else 0, ctypes.byref(g), stream)
            if st:
                _lib.check(st, "t4b_fused_w4a16_gemv_allgather")
        return self._views

    def close(self):
        """Release the peers' mappings and this rank's buffers.  Call on every
        rank after a barrier, once no rank can still be writing."""
        for p in self._opened:
            self._lib.t4b_ipc_close(p)
        for p in self._own:
            self._lib.t4b_ipc_free(p)
        self._opened, self._own = [], []
