"""Ahead-of-time build of the two native libraries, in-tree.

* ``libnib_b200.so``  - the CUDA kernels and their C ABI (``include/nib_b200.h``),
  compiled by nvcc for sm_100a only (``-gencode arch=compute_100a,code=sm_100a``),
  no fast-math (the kernels rely on IEEE division, sqrt and libm-accurate
  sincos/exp where the reference's numerics need them). CUDA runtime linked
  statically, so the library stands alone behind its C ABI.
* ``_nib_torch.so``   - the PyTorch binding (``csrc/torch_shim.cpp``), compiled by
  g++ against the installed torch headers, linked to ``libnib_b200.so`` through
  an ``$ORIGIN`` rpath.

Both land next to this file so they travel with the source tree. A stamp file
records a hash of every source, header and flag; an unchanged tree is not
rebuilt.
"""

from __future__ import annotations

import hashlib
import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PKG = Path(__file__).resolve().parent
REPO = PKG.parent
CSRC = PKG / "csrc"
INCLUDE = REPO / "include"
BUILD_DIR = REPO / "_build"
LIB = PKG / "libnib_b200.so"
SHIM = PKG / "_nib_torch.so"
STAMP = PKG / ".build_stamp"

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-Xcompiler",
              "-fvisibility=hidden", "-Xptxas", "-warn-spills"]
CXX_FLAGS = ["-O2", "-std=c++17", "-fPIC", "-shared", "-fvisibility=hidden"]


def cuda_home() -> Path:
    env = os.environ.get("CUDA_HOME") or os.environ.get("CUDA_PATH")
    if env:
        return Path(env)
    nvcc = shutil.which("nvcc")
    if nvcc:
        return Path(nvcc).resolve().parent.parent
    return Path("/usr/local/cuda")


def _torch_flags():
    import torch
    from torch.utils import cpp_extension

    inc = [f"-I{p}" for p in cpp_extension.include_paths()]
    libdir = cpp_extension.library_paths()[0]
    abi = int(torch.compiled_with_cxx11_abi())
    return inc, libdir, [f"-D_GLIBCXX_USE_CXX11_ABI={abi}"]


def _digest() -> str:
    h = hashlib.sha256()
    files = sorted(CSRC.glob("*.cu")) + sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.cpp"))
    files += [INCLUDE / "nib_b200.h", Path(__file__)]
    for f in files:
        h.update(f.name.encode())
        h.update(f.read_bytes())
    h.update(" ".join(ARCH_FLAGS + NVCC_FLAGS + CXX_FLAGS).encode())
    try:
        import torch
        h.update(torch.__version__.encode())
    except ImportError:
        pass
    return h.hexdigest()


def _run(cmd, verbose):
    if verbose:
        print(" ".join(str(c) for c in cmd), flush=True)
    r = subprocess.run([str(c) for c in cmd], capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"build step failed ({r.returncode}): {' '.join(map(str, cmd))}\n"
                           f"{r.stdout}\n{r.stderr}")
    if verbose and (r.stdout or r.stderr):
        print(r.stdout, r.stderr, flush=True)
    return r


def up_to_date() -> bool:
    return LIB.exists() and SHIM.exists() and STAMP.exists() and STAMP.read_text().strip() == _digest()


def build(verbose: bool = False, force: bool = False) -> None:
    """Compile both libraries unless the stamp says they are current."""
    if not force and up_to_date():
        return
    nvcc = cuda_home() / "bin" / "nvcc"
    BUILD_DIR.mkdir(exist_ok=True)
    sources = sorted(CSRC.glob("*.cu"))
    objs = [BUILD_DIR / (s.stem + ".o") for s in sources]

    def compile_one(pair):
        src, obj = pair
        _run([nvcc, *ARCH_FLAGS, *NVCC_FLAGS, f"-I{INCLUDE}", "-c", src, "-o", obj], verbose)

    with ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 4)) as ex:
        list(ex.map(compile_one, zip(sources, objs)))
    tmp_lib = LIB.with_suffix(".so.tmp")
    _run([nvcc, *ARCH_FLAGS, "-shared", "-Xcompiler", "-fPIC", *objs, "-o", tmp_lib], verbose)
    os.replace(tmp_lib, LIB)

    inc, libdir, defs = _torch_flags()
    cuda = cuda_home()
    tmp_shim = SHIM.with_suffix(".so.tmp")
    _run(["g++", *CXX_FLAGS, *defs, f"-I{INCLUDE}", *inc, f"-I{cuda / 'include'}",
          CSRC / "torch_shim.cpp", "-o", tmp_shim,
          f"-L{PKG}", "-lnib_b200", f"-L{libdir}", "-lc10", "-lc10_cuda", "-ltorch_cpu",
          "-ltorch_cuda", "-ltorch", f"-L{cuda / 'lib64'}", "-lcudart", "-Wl,-rpath,$ORIGIN"],
         verbose)
    os.replace(tmp_shim, SHIM)
    STAMP.write_text(_digest() + "\n")


if __name__ == "__main__":
    build(verbose="-v" in sys.argv, force="-f" in sys.argv)
    print(f"built {LIB.name} and {SHIM.name}")
