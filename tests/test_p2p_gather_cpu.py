"""Host side of the fused GEMV + all-gather (t4b_fused_w4a16_gemv_allgather,
t4_cuda_b200.shard.P2PGatherGroup) without a GPU: the ctypes mirror of the
T4BGather struct matches the C compiler's layout, the entry point rejects bad
descriptors before touching the GPU, and the group's column layout."""

import ctypes
import os
import shutil
import subprocess

import pytest

from t4_cuda_b200 import _lib, shard

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.fixture(scope="module")
def lib():
    return _lib.load()


@pytest.mark.skipif(shutil.which("gcc") is None, reason="needs gcc")
def test_gather_struct_layout_matches_c(tmp_path):
    src = tmp_path / "layout.c"
    src.write_text(
        "#include <stdio.h>\n#include <stddef.h>\n#include \"t4b200.h\"\n"
        "int main(void) { printf(\"%zu %zu %zu %zu %zu %zu %zu %zu %zu\\n\", sizeof(T4BGather),"
        " offsetof(T4BGather, recv), offsetof(T4BGather, out),"
        " offsetof(T4BGather, counter), offsetof(T4BGather, world), offsetof(T4BGather, rank),"
        " offsetof(T4BGather, n_total), offsetof(T4BGather, col_offset), offsetof(T4BGather, barrier));"
        " return 0; }\n")
    exe = tmp_path / "layout"
    subprocess.run(["gcc", "-I", os.path.join(ROOT, "include"), str(src), "-o", str(exe)], check=True)
    c = [int(v) for v in subprocess.run([str(exe)], capture_output=True, text=True, check=True).stdout.split()]
    G = _lib.T4BGather
    py = [ctypes.sizeof(G)] + [getattr(G, f).offset for f in
                               ("recv", "out", "counter", "world", "rank", "n_total",
                                "col_offset", "barrier")]
    assert py == c


def _gather(world=2, rank=0, n_total=256, col_offset=0, fill=True):
    g = _lib.T4BGather()
    g.world, g.rank, g.n_total, g.col_offset, g.barrier = world, rank, n_total, col_offset, 1
    if fill:
        for r in range(min(world, 8)):
            g.recv[r] = 0x10000 * (r + 1)
        g.out = 0x80000
        g.counter = 0x90000
    return g


def test_allgather_rejects_bad_descriptors(lib):
    p = ctypes.c_void_p(0x100000)
    call = lambda g, N=128: lib.t4b_fused_w4a16_gemv_allgather(p, p, p, None, 1, N, 4096, 128, 1,
                                                               ctypes.byref(g) if g is not None else None, None)
    assert call(None) == 2                                   # no descriptor
    assert call(_gather(world=1)) == 1                       # a gather needs 2..8 ranks
    assert call(_gather(world=9)) == 1
    assert call(_gather(rank=2)) == 1                        # rank outside the group
    assert call(_gather(col_offset=200)) == 1                # columns past the buffer's row
    assert call(_gather(col_offset=1)) == 1                  # column pairs: offsets even
    assert call(_gather(n_total=255)) == 1
    assert call(_gather(fill=False)) == 2                    # buffers missing
    assert lib.t4b_fused_w4a16_gemv_allgather(p, p, p, None, 1, 128, 100, 128, 1,
                                              ctypes.byref(_gather()), None) == 1   # K not a multiple of 8


def test_grouped_allgather_rejects_bad_descriptors(lib):
    p = ctypes.c_void_p(0x100000)
    vp2 = ctypes.c_void_p * 2
    ptrs = vp2(0x100000, 0x200000)
    i2 = ctypes.c_int * 2

    def call(g, N=(64, 64), offs=(0, 64), n=2, K=4096):
        return lib.t4b_fused_w4a16_gemv_allgather_grouped(p, n, ptrs, ptrs, None, i2(*N), i2(*offs), 1, K, 128, 1,
                                                          ctypes.byref(g) if g is not None else None, None)
    assert call(None) == 2                                   # no descriptor
    assert call(_gather(), n=0) == 1                         # no projection
    assert call(_gather(), n=5) == 1                         # more than T4B_GROUPED_MAX
    assert call(_gather(world=1)) == 1
    assert call(_gather(rank=3)) == 1
    assert call(_gather(), offs=(0, 200)) == 1               # second projection past the buffer's row
    assert call(_gather(), offs=(0, 63)) == 1                # column pairs: offsets even
    assert call(_gather(fill=False)) == 2                    # buffers missing
    assert call(_gather(), K=100) == 1                       # K not a multiple of 8


def test_group_column_layout():
    offs, total = shard.column_offsets([512, 128, 128], 8)
    assert offs == [0, 4096, 5120] and total == 6144
    # rank r's slice of projection i starts at offs[i] + r * width[i]
    w, world = [512, 128, 128], 8
    starts = sorted(o + r * wi for o, wi in zip(offs, w) for r in range(world))
    ends = sorted(o + (r + 1) * wi for o, wi in zip(offs, w) for r in range(world))
    assert starts[0] == 0 and ends[-1] == total
    assert all(a == b for a, b in zip(ends[:-1], starts[1:]))     # slices tile the row exactly


def test_support_query_rejects_bad_shapes(lib):
    q = lib.t4b_fused_w4a16_gemv_allgather_supported
    assert q(0, 256, 4096, 128, 0) == 1          # M < 1
    assert q(1, 256, 4100, 128, 0) == 1          # K not a multiple of the group
    assert q(1, 256, 4096, 12, 0) == 1           # group not a multiple of 8
    assert q(1, 255, 4096, 128, 0) == 4          # odd width: no whole column pairs
    assert q(17, 256, 4096, 128, 0) == 4         # M > 16: not a decode shape
