"""Build the CUDA C-ABI library ``libt4b200.so`` in-tree for sm_100a.

    python -m t4_cuda_b200.build          # or: from t4_cuda_b200.build import build; build()

Each ``csrc/*.cu`` is compiled to an object (in parallel, skipped when the
object is newer than its sources) and linked into one shared library next to
this file.  The CUDA runtime is linked statically, so the library needs only
the NVIDIA driver at run time and shares the primary context that PyTorch
(or any other runtime user) has made current.
"""

import concurrent.futures as cf
import glob
import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
INCLUDE = os.path.join(ROOT, "include")
BUILD = os.path.join(PKG, "_build")
LIB = os.path.join(PKG, "libt4b200.so")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
              "-Xptxas", "-v", "-I" + INCLUDE, "-I" + CSRC]


def nvcc():
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found (set NVCC or put the CUDA toolkit on PATH)")


def _headers():
    return glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(INCLUDE, "*.h"))


def _stale(target, deps):
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def _compile(src, verbose):
    obj = os.path.join(BUILD, os.path.basename(src)[:-3] + ".o")
    if not _stale(obj, [src] + _headers()):
        return obj, ""
    cmd = [nvcc()] + ARCH + NVCC_FLAGS + ["-c", src, "-o", obj]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed for {os.path.basename(src)}:\n{res.stdout}\n{res.stderr}")
    with open(obj + ".ptxas.txt", "w") as f:   # register / spill report from -Xptxas -v
        f.write(res.stderr)
    if verbose:
        print(f"[t4b200] compiled {os.path.basename(src)}", file=sys.stderr)
    return obj, res.stderr


def build(verbose=False, force=False):
    """Compile every kernel for sm_100a and link libt4b200.so; returns its path."""
    os.makedirs(BUILD, exist_ok=True)
    sources = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    if force:
        for o in glob.glob(os.path.join(BUILD, "*.o")):
            os.remove(o)
    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as ex:
        objs = [o for o, _ in ex.map(lambda s: _compile(s, verbose), sources)]
    if force or _stale(LIB, objs):
        tmp = LIB + ".tmp"
        cmd = [nvcc()] + ARCH + ["-shared", "-o", tmp] + objs + ["-lcudart_static", "-lrt", "-ldl", "-lpthread"]
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"link failed:\n{res.stdout}\n{res.stderr}")
        os.replace(tmp, LIB)
        if verbose:
            print(f"[t4b200] linked {LIB}", file=sys.stderr)
    return LIB


BIND_SRC = os.path.join(PKG, "bind", "torch_ops.cpp")


def binding_path():
    """In-tree path of the torch binding module (``_torch_ops``)."""
    import sysconfig
    return os.path.join(PKG, "_torch_ops" + sysconfig.get_config_var("EXT_SUFFIX"))


def build_binding(verbose=False, force=False):
    """Compile the torch binding of the fused ops (bind/torch_ops.cpp) with the
    host compiler against the installed torch; returns its path."""
    import sysconfig
    import torch
    from torch.utils import cpp_extension
    out = binding_path()
    if not force and not _stale(out, [BIND_SRC]):
        return out
    cxx = os.environ.get("CXX") or shutil.which("g++") or "c++"
    abi = int(bool(torch._C._GLIBCXX_USE_CXX11_ABI))
    inc = cpp_extension.include_paths() + [sysconfig.get_paths()["include"], os.path.join(_cuda_home(), "include")]
    libdirs = cpp_extension.library_paths()
    cmd = ([cxx, "-O2", "-std=c++17", "-shared", "-fPIC", "-fvisibility=hidden", f"-D_GLIBCXX_USE_CXX11_ABI={abi}",
            "-DTORCH_EXTENSION_NAME=_torch_ops", "-DTORCH_API_INCLUDE_EXTENSION_H"]
           + ["-I" + d for d in inc] + [BIND_SRC, "-o", out + ".tmp"]
           + ["-L" + d for d in libdirs] + ["-Wl,-rpath," + d for d in libdirs]
           + ["-lc10", "-lc10_cuda", "-ltorch", "-ltorch_cpu", "-ltorch_cuda", "-ltorch_python"])
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"torch binding build failed:\n{res.stdout}\n{res.stderr}")
    os.replace(out + ".tmp", out)
    if verbose:
        print(f"[t4b200] built {out}", file=sys.stderr)
    return out


def _cuda_home():
    nv = nvcc()
    return os.path.dirname(os.path.dirname(os.path.realpath(nv)))


if __name__ == "__main__":
    build(verbose=True, force="--force" in sys.argv)
    build_binding(verbose=True, force="--force" in sys.argv)
