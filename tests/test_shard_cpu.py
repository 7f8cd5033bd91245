"""Host logic of the column-sharded wrapper (t4_cuda_b200/shard.py) on CPU.

The shard's device work is the single-GPU op on this rank's columns; here
that op is replaced by the oracle (each rank computes its slice on the CPU),
so what is tested is the wrapper itself: the column slicing of packed words,
scales and zero points, the packing of several projections into one gather,
the rank-major gather over a real process group (gloo, world size 2), and
the unpacking back to [M, N] per projection.
"""

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle
from t4_cuda_b200 import shard


def _oracle_local(self, x):
    """ShardedLinear.local restated on the CPU with the oracle (W4A16 only)."""
    A = x.numpy()
    W = self.W.numpy()
    S = self.S.numpy()
    Z = None if self.Z is None else self.Z.numpy()
    y = oracle.ref_w4_gemm(A, W, S, Z, signed=(self.fmt == "s4"))
    return torch.from_numpy(y.astype(np.float32))


def _full_case(seed, M, K, Ns, group=128):
    rng = np.random.default_rng(seed)
    A = rng.standard_normal((M, K)).astype(np.float16)
    projs = []
    for N in Ns:
        W = rng.integers(0, 2 ** 32, size=(K // 8, N), dtype=np.int64).astype(np.uint32).view(np.int32)
        S = (np.abs(rng.standard_normal((K // group, N))) * 0.02 + 1e-3).astype(np.float16)
        Z = rng.integers(0, 16, size=(K // group, N)).astype(np.float16)
        projs.append((W, S, Z))
    return A, projs


def test_shard_bounds_and_columns():
    assert shard.shard_bounds(1024, 0, 8) == (0, 128)
    assert shard.shard_bounds(1024, 7, 8) == (896, 1024)
    with pytest.raises(ValueError):
        shard.shard_bounds(1000, 0, 3)
    t = torch.arange(24, dtype=torch.int32).reshape(2, 12)
    parts = [shard.shard_columns(t, r, 3) for r in range(3)]
    assert all(p.is_contiguous() and p.shape == (2, 4) for p in parts)
    assert torch.equal(torch.cat(parts, dim=1), t)
    v = torch.arange(12, dtype=torch.float16)           # 1-D per-column scales become (1, N)
    assert shard.shard_columns(v, 1, 3).shape == (1, 4)
    assert shard.shard_columns(None, 0, 2) is None


def test_unpack_gathered_rank_major():
    G, M, widths = 4, 3, [2, 5]
    g = torch.zeros((G, M, sum(widths)))
    for r in range(G):
        for m in range(M):
            for c in range(sum(widths)):
                g[r, m, c] = 1000 * r + 10 * m + c
    a, b = shard.unpack_gathered(g, widths)
    assert a.shape == (M, G * 2) and b.shape == (M, G * 5)
    for r in range(G):
        assert torch.equal(a[:, 2 * r:2 * r + 2], g[r, :, 0:2])
        assert torch.equal(b[:, 5 * r:5 * r + 5], g[r, :, 2:7])


def test_single_process_group_is_local(monkeypatch):
    monkeypatch.setattr(shard.ShardedLinear, "local", _oracle_local)
    A, projs = _full_case(3, 2, 256, [64])
    W, S, Z = projs[0]
    lin = shard.ShardedLinear.from_full(torch.from_numpy(W), torch.from_numpy(S), torch.from_numpy(Z), "s4")
    y = lin(torch.from_numpy(A))
    ref = oracle.ref_w4_gemm(A, W, S, Z, signed=True)
    np.testing.assert_allclose(y.numpy(), ref, rtol=0, atol=0)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, out_dir):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        shard.ShardedLinear.local = _oracle_local
        A, projs = _full_case(11, 3, 512, [96, 32, 160])
        lins = [shard.ShardedLinear.from_full(torch.from_numpy(W), torch.from_numpy(S), torch.from_numpy(Z), "s4")
                for W, S, Z in projs]
        assert all(lin.n_local == W.shape[1] // world for lin, (W, _, _) in zip(lins, projs))
        outs = shard.ShardedGroup(lins)(torch.from_numpy(A))           # one gather for three projections
        single = lins[1](torch.from_numpy(A))                           # and one on its own
        np.savez(os.path.join(out_dir, f"rank{rank}.npz"), *[o.numpy() for o in outs], single=single.numpy())
    finally:
        dist.destroy_process_group()


def test_sharded_group_gloo_world2(tmp_path):
    world = 2
    mp.start_processes(_worker, args=(world, _free_port(), str(tmp_path)), nprocs=world, join=True,
                       start_method="spawn")
    A, projs = _full_case(11, 3, 512, [96, 32, 160])
    refs = [oracle.ref_w4_gemm(A, W, S, Z, signed=True) for W, S, Z in projs]
    for rank in range(world):
        d = np.load(os.path.join(tmp_path, f"rank{rank}.npz"))
        for i, ref in enumerate(refs):
            got = d[f"arr_{i}"]
            assert got.shape == ref.shape
            np.testing.assert_allclose(got, ref, rtol=0, atol=0)      # every rank holds the full output
        np.testing.assert_allclose(d["single"], refs[1], rtol=0, atol=0)


def test_grouped_args_rules():
    """Which projection groups ShardedGroup / P2PGatherGroup call as one
    grouped launch: 2..4 projections, all s4 or all u4, the same K and group
    size, zero points for all or none."""
    def lin(K, N, fmt="s4", groups=None, zp=False):
        G = groups or K // 128
        W = torch.zeros((K // 8, N), dtype=torch.int32)
        S = torch.ones((G, N), dtype=torch.float16)
        Z = torch.zeros((G, N), dtype=torch.float16) if zp else None
        return shard.ShardedLinear(W, S, Z, fmt)
    q, k, v = lin(512, 64), lin(512, 16), lin(512, 16)
    Ws, Ss, Zs, signed = shard._grouped_args([q, k, v])
    assert [w.size(1) for w in Ws] == [64, 16, 16] and Zs is None and signed is True
    assert shard._grouped_args([lin(512, 64, "u4"), lin(512, 32, "u4")])[3] is False
    z = shard._grouped_args([lin(512, 64, zp=True), lin(512, 32, zp=True)])[2]
    assert z is not None and len(z) == 2
    assert shard._grouped_args([q]) is None                                   # one projection
    assert shard._grouped_args([q] * 5) is None                               # more than 4
    assert shard._grouped_args([q, lin(512, 64, "u4")]) is None               # mixed formats
    assert shard._grouped_args([q, lin(1024, 64)]) is None                    # different K
    assert shard._grouped_args([q, lin(512, 64, groups=8)]) is None           # different group size
    assert shard._grouped_args([q, lin(512, 64, zp=True)]) is None            # zero points for some
    assert shard._grouped_args([lin(512, 64, "s3"), lin(512, 64, "s3")]) is None   # INT3 is not grouped
