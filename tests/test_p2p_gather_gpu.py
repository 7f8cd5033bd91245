"""The fused GEMV + all-gather on two and four GPUs (each case skipped with
fewer): the ranks (processes; NCCL only to exchange the receive buffers'
handles) each hold their share of the columns of the projections of two groups -- three projections at M = 1
and one at M = 3 -- and call them in the order G1, G2, G1, G2, G1 with fresh
activations each time -- G1 as one grouped launch (its three projections in
one decode launch) and as one launch per projection.  After every call each rank's outputs hold the whole
projection outputs, equal to the oracle within the GEMV gate, and the device
error word stays clear."""

import datetime
import os
import socket

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

K = 4096
G1 = (1, [1024, 256, 512])      # (M, full widths)
G2 = (3, [768])
CALLS = [0, 1, 0, 1, 0]


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _weights(seed, Ns, group=128):
    rng = np.random.default_rng(seed)
    out = []
    for N in Ns:
        W = rng.integers(0, 2 ** 32, size=(K // 8, N), dtype=np.int64).astype(np.uint32).view(np.int32)
        S = (np.abs(rng.standard_normal((K // group, N))) * 0.02 + 1e-3).astype(np.float16)
        out.append((W, S))
    return out


def _acts(call, M):
    return np.random.default_rng(100 + call).standard_normal((M, K)).astype(np.float16)


def _worker(rank, world, port, out_dir, grouped):
    import torch.distributed as dist
    from t4_cuda_b200 import ops, shard
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                            timeout=datetime.timedelta(seconds=60))
    try:
        groups = []
        for gi, (M, Ns) in enumerate((G1, G2)):
            lins = [shard.ShardedLinear.from_full(torch.from_numpy(W).to(dev), torch.from_numpy(S).to(dev),
                                                  None, "s4") for W, S in _weights(gi, Ns)]
            groups.append(shard.P2PGatherGroup(lins, M, grouped=grouped))
        # G1 (three s4 projections at M = 1) is one grouped launch when grouped
        assert (groups[0]._grouped is not None) == grouped
        res = {}
        for c, gi in enumerate(CALLS):
            x = torch.from_numpy(_acts(c, groups[gi].M)).to(dev)
            outs = groups[gi](x)
            for i, o in enumerate(outs):
                res[f"c{c}_p{i}"] = o.float().cpu().numpy()
        torch.cuda.synchronize()
        res["err"] = np.array(int(ops.device_error(dev)))
        np.savez(os.path.join(out_dir, f"rank{rank}.npz"), **res)
        dist.barrier()
        for g in groups:
            g.close()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("grouped", [True, False])
@pytest.mark.parametrize("world", [2, 4])
def test_fused_allgather_ranks(tmp_path, world, grouped):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    import oracle
    import torch.multiprocessing as mp
    mp.start_processes(_worker, args=(world, _free_port(), str(tmp_path), grouped), nprocs=world, join=True,
                       start_method="spawn")
    weights = [_weights(0, G1[1]), _weights(1, G2[1])]
    for rank in range(world):
        d = np.load(os.path.join(tmp_path, f"rank{rank}.npz"))
        assert int(d["err"]) == 0
        for c, gi in enumerate(CALLS):
            A = _acts(c, (G1, G2)[gi][0])
            for i, (W, S) in enumerate(weights[gi]):
                ref = oracle.ref_w4_gemm(A, W, S, None, signed=True)
                y = d[f"c{c}_p{i}"]
                assert y.shape == ref.shape
                assert np.abs(y - ref).max() <= 1e-2 * np.abs(ref).max(), (rank, c, i)
                assert np.abs(y - ref).mean() <= 1e-3 * np.abs(ref).mean(), (rank, c, i)
