"""Build the LSA B200 kernels into one in-tree shared library (``lsa_b200/liblsa_b200.so``).

Every ``csrc/*.cu`` is compiled for sm_100a only (``-gencode arch=compute_100a,code=sm_100a``)
and linked into a plain C-ABI library: the entry points are ``extern "C"`` with raw
pointers, sizes and a ``cudaStream_t`` (declared in ``include/lsa_b200.h``), so any host
language can bind them. No fast-math: selection arithmetic must match the checker bit for
bit. nvcc cross-compiles without a GPU, so this runs on CPU-only machines too.
"""

from __future__ import annotations

import concurrent.futures as cf
import os
import pathlib
import shutil
import subprocess
import sys

HERE = pathlib.Path(__file__).resolve().parent
CSRC = HERE / "csrc"
OUT_DIR = HERE / "lsa_b200"
LIB = OUT_DIR / "liblsa_b200.so"
OBJ_DIR = HERE / "_build"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
              "-diag-suppress", "177"]


def nvcc() -> str:
    path = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(path):
        raise RuntimeError("nvcc not found: the LSA kernels need the CUDA toolkit to build")
    return path


def _stale(obj: pathlib.Path, src: pathlib.Path) -> bool:
    if not obj.exists():
        return True
    deps = [src] + sorted(CSRC.glob("*.cuh"))
    return any(d.stat().st_mtime > obj.stat().st_mtime for d in deps)


def _compile(src: pathlib.Path) -> pathlib.Path:
    obj = OBJ_DIR / (src.stem + ".o")
    if _stale(obj, src):
        cmd = [nvcc(), *ARCH, *NVCC_FLAGS, "-c", str(src), "-o", str(obj)]
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"nvcc failed on {src.name}:\n{res.stderr[-4000:]}")
    return obj


TORCH_OPS_SRC = CSRC / "torch_ops.cpp"
TORCH_OPS_LIB = OUT_DIR / "_lsa_torch_ops.so"


def build_torch_ops(force: bool = False) -> pathlib.Path:
    """The torch.library operators (csrc/torch_ops.cpp): a C++ shared library over the C ABI,
    compiled against this torch's headers and ABI and linked to liblsa_b200.so beside it."""
    import torch
    from torch.utils import cpp_extension as ce

    header = HERE.parent / "include" / "lsa_b200.h"
    deps = [TORCH_OPS_SRC, header, LIB]
    if not force and TORCH_OPS_LIB.exists() and all(d.stat().st_mtime <= TORCH_OPS_LIB.stat().st_mtime for d in deps):
        return TORCH_OPS_LIB
    cxx = shutil.which("g++") or "g++"
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    torch_lib = pathlib.Path(torch.__file__).resolve().parent / "lib"
    cuda_home = pathlib.Path(ce.CUDA_HOME or "/usr/local/cuda")
    incs = [p for p in (ce.include_paths() + [str(cuda_home / "include")])]
    cmd = [cxx, "-O2", "-std=c++17", "-shared", "-fPIC", f"-D_GLIBCXX_USE_CXX11_ABI={abi}",
           *[f"-I{i}" for i in incs], str(TORCH_OPS_SRC), "-o", str(TORCH_OPS_LIB) + ".tmp",
           f"-L{torch_lib}", "-lc10", "-lc10_cuda", "-ltorch", "-ltorch_cpu", "-ltorch_cuda",
           f"-L{OUT_DIR}", "-llsa_b200", f"-L{cuda_home / 'lib64'}", "-lcudart", "-Wl,-rpath,$ORIGIN"]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"torch ops build failed:\n{res.stderr[-4000:]}")
    os.replace(str(TORCH_OPS_LIB) + ".tmp", TORCH_OPS_LIB)
    return TORCH_OPS_LIB


def build(force: bool = False, verbose: bool = False) -> pathlib.Path:
    """Compile every kernel source (in parallel) and link ``liblsa_b200.so`` in place."""
    OBJ_DIR.mkdir(exist_ok=True)
    sources = sorted(CSRC.glob("*.cu"))
    if force:
        for o in OBJ_DIR.glob("*.o"):
            o.unlink()
    with cf.ThreadPoolExecutor(max_workers=min(8, len(sources))) as pool:
        objs = list(pool.map(_compile, sources))
    if force or not LIB.exists() or any(o.stat().st_mtime > LIB.stat().st_mtime for o in objs):
        tmp = LIB.with_suffix(".so.tmp")
        cmd = [nvcc(), *ARCH, "-shared", "-Xcompiler", "-fPIC", *map(str, objs), "-o", str(tmp), "-lcudart"]
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"link failed:\n{res.stderr[-4000:]}")
        os.replace(tmp, LIB)
    build_torch_ops(force)
    if verbose:
        print(f"built {LIB} and {TORCH_OPS_LIB.name}")
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose=True)
