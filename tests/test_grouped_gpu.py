"""Grouped calls (ops.fused_w4a16_gemm_grouped / t4b_fused_w4a16_gemm_grouped):
projections that read the same activation -- a layer's q/k/v or gate/up --
in one call, checked against the oracle.

The reference has no grouped op: a layer's projections are separate
fused_w4a16_gemm_{s4,u4} calls (tests/test_fused_gemm_correctness.py:86-113
checks one projection per call), so every projection of a grouped call is
held to the same gate as a single call: max |y - y_ref| <= 1e-2 max |y_ref|
and mean |y - y_ref| <= 1e-3 mean |y_ref| against oracle.ref_w4_gemm.  For
M <= 16 the decode kernel runs the projections as one launch whose CTAs are
shared out by column tiles (each CTA works inside one projection); larger M
makes one call per projection inside the library.
"""

import numpy as np
import pytest
import torch

import oracle
import t4_kernels
from t4_cuda_b200 import ops, shard
from tests.test_configs_gpu import check
from tests.test_gemv_gpu import assert_gemm_close

pytestmark = pytest.mark.gpu

LLAMA8B_GROUPS = {"qkv": [4096, 1024, 1024], "gate_up": [14336, 14336]}
# the Llama-3-70B layer's groups (hidden 8192), whole (one GPU) and as an 8-way column shard sees them
LLAMA70B_GROUPS = {"qkv": [8192, 1024, 1024], "gate_up": [28672, 28672],
                   "qkv_shard8": [1024, 128, 128], "gate_up_shard8": [3584, 3584]}


def make_group(seed, M, K, Ns, dev, group=128, zp=False):
    """One activation and len(Ns) projections with the benchmark's
    distributions: A ~ N(0, 1) fp16, full-range random words, scales
    |N(0, 0.02)| + 1e-3, optional integer zero points."""
    rng = np.random.default_rng(seed)
    A = rng.standard_normal((M, K), dtype=np.float32).astype(np.float16)
    projs = []
    for N in Ns:
        W = rng.integers(0, 2 ** 32, size=(K // 8, N), dtype=np.uint32).view(np.int32)
        s = (np.abs(rng.standard_normal((K // group, N), dtype=np.float32) * 0.02) + 1e-3).astype(np.float16)
        z = rng.integers(0, 16, size=(K // group, N)).astype(np.float16) if zp else None
        projs.append((W, s, z))
    t = lambda x: None if x is None else torch.from_numpy(x).to(dev)     # noqa: E731
    dev_projs = [(t(W), t(s), t(z)) for W, s, z in projs]
    return rng, A, projs, t(A), dev_projs


def grouped(At, dev_projs, signed=True):
    Ws = [W for W, _, _ in dev_projs]
    Ss = [s for _, s, _ in dev_projs]
    Zs = [z for _, _, z in dev_projs] if dev_projs[0][2] is not None else None
    return ops.fused_w4a16_gemm_grouped(At, Ws, Ss, Zs, signed=signed)


@pytest.mark.parametrize("M", [1, 4, 8, 16])
@pytest.mark.parametrize("name", sorted(LLAMA8B_GROUPS))
def test_llama8b_groups(cuda_device, name, M):
    Ns = LLAMA8B_GROUPS[name]
    rng, A, projs, At, dev_projs = make_group(7000 + M + len(Ns), M, 4096, Ns, cuda_device)
    Cs = grouped(At, dev_projs)
    torch.cuda.synchronize(cuda_device)
    assert ops.device_error(cuda_device) == 0
    assert len(Cs) == len(Ns)
    for j, (C, (W, s, _)) in enumerate(zip(Cs, projs)):
        assert C.shape == (M, Ns[j])
        check(C, (A, W, s, None), rng, True, f"{name}[{j}] M={M} K=4096 N={Ns[j]}")


@pytest.mark.parametrize("M", [1, 16])
@pytest.mark.parametrize("name", sorted(LLAMA70B_GROUPS))
def test_llama70b_groups(cuda_device, name, M):
    Ns = LLAMA70B_GROUPS[name]
    rng, A, projs, At, dev_projs = make_group(8000 + M + sum(Ns) % 97, M, 8192, Ns, cuda_device)
    Cs = grouped(At, dev_projs)
    torch.cuda.synchronize(cuda_device)
    assert ops.device_error(cuda_device) == 0
    for j, (C, (W, s, _)) in enumerate(zip(Cs, projs)):
        check(C, (A, W, s, None), rng, True, f"70B {name}[{j}] M={M} K=8192 N={Ns[j]}")


@pytest.mark.parametrize("signed", [True, False])
@pytest.mark.parametrize("zp", [False, True])
@pytest.mark.parametrize("M", [1, 3, 9, 16])
@pytest.mark.parametrize("K,group,Ns", [
    (256, 64, [72, 200, 8]),            # ragged tails: tiles past the last column
    (512, 128, [16]),                   # one projection, one tile
    (512, 64, [8, 8, 8, 8]),            # T4B_GROUPED_MAX projections of one partial tile each
    (1024, 128, [2048, 520, 3000]),     # more tiles than SMs, shared out
    (384, 128, [4096, 4096]),           # group 128 = 16 word rows over a 48-row K
])
def test_small_shapes_against_oracle(cuda_device, K, group, Ns, M, zp, signed):
    rng, A, projs, At, dev_projs = make_group(K * 31 + M * 7 + len(Ns) + zp, M, K, Ns, cuda_device, group, zp)
    Cs = grouped(At, dev_projs, signed)
    Cs_py = ops._fused_grouped(At, [W for W, _, _ in dev_projs], [s for _, s, _ in dev_projs],
                               [z for _, _, z in dev_projs] if zp else None, signed)
    torch.cuda.synchronize(cuda_device)
    assert ops.device_error(cuda_device) == 0
    for j, (C, C_py, (W, s, z)) in enumerate(zip(Cs, Cs_py, projs)):
        ref = oracle.ref_w4_gemm(A, W, s, z, signed=signed)
        assert_gemm_close(C, ref, f"[{j}] M={M} K={K} N={Ns[j]} g{group} zp={zp} signed={signed}")
        assert torch.equal(C, C_py), "torch binding and ctypes path differ"


def test_one_projection_is_the_single_call(cuda_device):
    """A grouped call of one projection is the single op's launch, bit for bit."""
    for M, K, N in [(1, 4096, 4096), (4, 4096, 14336), (16, 14336, 4096), (2, 512, 72)]:
        _, _, _, At, dev_projs = make_group(M + K + N, M, K, [N], cuda_device)
        (C,) = grouped(At, dev_projs)
        W, s, _ = dev_projs[0]
        assert torch.equal(C, t4_kernels.fused_w4a16_gemm_s4(At, W, s, None)), (M, K, N)


def test_large_m_makes_single_calls(cuda_device):
    """Past M = 16 the library makes one call per projection: the same
    kernels as the single op, so the same bits."""
    for M in (17, 64, 256):
        rng, A, projs, At, dev_projs = make_group(900 + M, M, 1024, [1024, 256, 256], cuda_device)
        assert ops.grouped_plan([1024, 256, 256], M, 1024, 128) is None
        Cs = grouped(At, dev_projs)
        for C, (W, s, _), (Wh, sh, _) in zip(Cs, dev_projs, projs):
            assert torch.equal(C, t4_kernels.fused_w4a16_gemm_s4(At, W, s, None))
            check(C, (A, Wh, sh, None), rng, True, f"M={M} single calls")


def test_plan_shares_the_sms(cuda_device):
    sms = torch.cuda.get_device_properties(cuda_device).multi_processor_count
    for Ns in ([4096, 1024, 1024], [14336, 14336], [8192, 1024, 1024], [64, 64, 32]):
        ctas = ops.grouped_plan(Ns, 1, 4096, 128)
        assert ctas is not None and len(ctas) == len(Ns)
        tiles = [(n + 15) // 16 for n in Ns]
        assert all(1 <= c <= t for c, t in zip(ctas, tiles))
        if sum(tiles) <= sms:
            assert ctas == tiles                # one tile a CTA
        else:
            assert sum(ctas) == sms
            # no CTA could move to another projection and lower the largest share
            worst = max(-(-t // c) for t, c in zip(tiles, ctas))
            assert worst <= -(-sum(tiles) // sms) + 1, (Ns, ctas)
    assert ops.grouped_plan([14336, 14336], 1, 4096, 128) == [sms // 2, sms - sms // 2]


def test_chain_and_graph(cuda_device):
    """q of a grouped q/k/v call feeds the next grouped gate/up call as its
    activation (a read-after-write between launches, which the programmatic
    dependent launch must order), eager and replayed from a CUDA graph with
    new inputs."""
    M, K = 2, 4096
    rng, A, qkv, At, dev_qkv = make_group(4242, M, K, [4096, 1024, 1024], cuda_device)
    _, _, gu, _, dev_gu = make_group(4343, M, K, [14336, 14336], cuda_device)

    def layer(x):
        q, k, v = grouped(x, dev_qkv)
        g, u = grouped(q, dev_gu)
        return q, k, v, g, u

    def verify(x_host, outs, what):
        q = outs[0]
        check(q, (x_host, *qkv[0][:2], None), rng, True, f"{what} q")
        q_host = q.cpu().numpy()
        for j, C in enumerate(outs[3:]):
            W, s, _ = gu[j]
            check(C, (q_host, W, s, None), rng, True, f"{what} gate/up[{j}] on q")

    verify(A, layer(At), "eager")
    x = At.clone()
    s = torch.cuda.Stream(cuda_device)
    s.wait_stream(torch.cuda.current_stream(cuda_device))
    with torch.cuda.stream(s):
        layer(x)
    torch.cuda.current_stream(cuda_device).wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        outs = layer(x)
    for seed in (1, 2):
        A2 = np.random.default_rng(seed).standard_normal((M, K), dtype=np.float32).astype(np.float16)
        x.copy_(torch.from_numpy(A2).to(cuda_device))
        g.replay()
        torch.cuda.synchronize(cuda_device)
        verify(A2, outs, f"graph replay {seed}")
    del g
    assert ops.device_error(cuda_device) == 0


def test_sharded_group_on_one_gpu_uses_the_grouped_call(cuda_device):
    rng, A, projs, At, dev_projs = make_group(55, 1, 4096, [4096, 1024, 1024], cuda_device)
    lins = [shard.ShardedLinear(W, s, None, "s4") for W, s, _ in dev_projs]
    grp = shard.ShardedGroup(lins)
    assert grp._grouped is not None
    outs = grp(At)
    for C, C_direct in zip(outs, grouped(At, dev_projs)):
        assert torch.equal(C, C_direct)
    # a mixed group (s4 with u4) makes one call per projection
    mixed = shard.ShardedGroup([lins[0], shard.ShardedLinear(*dev_projs[1][:2], None, "u4")])
    assert mixed._grouped is None
    y0, y1 = mixed(At)
    assert torch.equal(y1, t4_kernels.fused_w4a16_gemm_u4(At, *dev_projs[1][:2], None))


def test_grouped_argument_errors(cuda_device):
    _, _, _, At, dev_projs = make_group(66, 1, 512, [64, 64], cuda_device)
    (W0, s0, _), (W1, _, _) = dev_projs
    s_g64 = torch.ones((512 // 64, 64), dtype=torch.float16, device=cuda_device)
    with pytest.raises(RuntimeError, match="same group size"):
        ops.fused_w4a16_gemm_grouped(At, [W0, W1], [s0, s_g64])
    z = torch.zeros_like(s0)
    with pytest.raises(RuntimeError, match="every projection of a grouped call or for none"):
        ops.fused_w4a16_gemm_grouped(At, [W0, W1], [s0, s0], [z, None])
    with pytest.raises(RuntimeError, match="W_packed must have K/8=64 rows"):
        ops.fused_w4a16_gemm_grouped(At, [W0, W1[:32]], [s0, s0])
