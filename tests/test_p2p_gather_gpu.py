"""The fused GEMV + all-gather on two GPUs (skipped with fewer): two ranks
(processes, NCCL for the handle exchange only) each hold half the columns of
three projections that share an activation; after one call of the group every
rank's buffer holds the whole outputs, equal to the oracle within the GEMV
gate, and repeated calls keep working (epochs advance)."""

import datetime
import os
import socket

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _case(seed, K, Ns, group=128):
    rng = np.random.default_rng(seed)
    A = rng.standard_normal((1, K)).astype(np.float16)
    projs = []
    for N in Ns:
        W = rng.integers(0, 2 ** 32, size=(K // 8, N), dtype=np.int64).astype(np.uint32).view(np.int32)
        S = (np.abs(rng.standard_normal((K // group, N))) * 0.02 + 1e-3).astype(np.float16)
        projs.append((W, S))
    return A, projs


def _worker(rank, world, port, out_dir):
    import torch.distributed as dist
    from t4_cuda_b200 import shard
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                            timeout=datetime.timedelta(seconds=60))
    try:
        A, projs = _case(5, 4096, [1024, 256, 512])
        lins = [shard.ShardedLinear.from_full(torch.from_numpy(W).to(dev), torch.from_numpy(S).to(dev), None, "s4")
                for W, S in projs]
        grp = shard.P2PGatherGroup(lins, 1)
        x = torch.from_numpy(A).to(dev)
        for _ in range(3):
            outs = grp(x)
        torch.cuda.synchronize()
        from t4_cuda_b200 import ops
        err = ops.device_error(dev)
        np.savez(os.path.join(out_dir, f"rank{rank}.npz"), *[o.float().cpu().numpy() for o in outs], err=err)
        dist.barrier()
        grp.close()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_fused_allgather_two_ranks(tmp_path):
    import oracle
    import torch.multiprocessing as mp
    mp.start_processes(_worker, args=(2, _free_port(), str(tmp_path)), nprocs=2, join=True, start_method="spawn")
    A, projs = _case(5, 4096, [1024, 256, 512])
    for rank in range(2):
        d = np.load(os.path.join(tmp_path, f"rank{rank}.npz"))
        assert int(d["err"]) == 0
        for i, (W, S) in enumerate(projs):
            ref = oracle.ref_w4_gemm(A, W, S, None, signed=True)
            y = d[f"arr_{i}"]
            assert y.shape == ref.shape
            assert np.abs(y - ref).max() <= 1e-2 * np.abs(ref).max()
            assert np.abs(y - ref).mean() <= 1e-3 * np.abs(ref).mean()
