"""Compile the reference's own paged-KV CUDA extension, for comparison only.

TEST INFRASTRUCTURE ONLY. The reference ships one GPU kernel pair on this path:
the ``nanovllm_paged_kv`` store / gather extension (``csrc/paged_kv/
{paged_kv.cpp, paged_kv_cuda.cu, paged_kv_runtime.h}`` of the NanoInfer
checkout, JIT-built there by ``nanovllm/layers/paged_kv/loader.py``). This
recipe compiles those three files where they lie, with nvcc for sm_100a and
g++ against the installed torch (the same headers and libraries this repo's own
binding uses), into ``oracle/_ref/nanovllm_paged_kv_ref.so``. It does not run
the reference's build system. Nothing is copied; the output directory is
git-ignored and travels to the GPU box with the tree.

``tests/test_gpu_reference_paged_kv.py`` loads the library in a child process
(it registers the same ``nanovllm_paged_kv`` namespace as this repo's binding,
so the two cannot share a process) and checks this repo's store and gather bit
for bit against it, on the same inputs, timing both.

Usage: ``NANOINFER_REF=<checkout> python oracle/build_ref_ext.py`` (a no-op
when the checkout or its sources are absent, or the library is up to date).
"""

from __future__ import annotations

import hashlib
import os
import subprocess
import sys
import sysconfig
from pathlib import Path

HERE = Path(__file__).resolve().parent
OUT_DIR = HERE / "_ref"
LIB = OUT_DIR / "nanovllm_paged_kv_ref.so"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def sources(ref: Path) -> list[Path]:
    d = ref / "csrc" / "paged_kv"
    return [d / "paged_kv.cpp", d / "paged_kv_cuda.cu", d / "paged_kv_runtime.h"]


def _digest(files: list[Path]) -> str:
    h = hashlib.sha256()
    for f in files:
        h.update(f.name.encode())
        h.update(f.read_bytes())
    import torch
    h.update(torch.__version__.encode())
    h.update(" ".join(ARCH).encode())
    return h.hexdigest()


def build(ref: Path | None = None, verbose: bool = False) -> Path | None:
    """Build the library if the checkout is present; returns its path or None."""
    if ref is None:
        env = os.environ.get("NANOINFER_REF")
        ref = Path(env) if env else None
    if ref is None or not all(f.is_file() for f in sources(ref)):
        return LIB if LIB.exists() else None
    import torch
    from torch.utils import cpp_extension

    files = sources(ref)
    stamp = OUT_DIR / ".stamp"
    digest = _digest(files)
    if LIB.exists() and stamp.exists() and stamp.read_text().strip() == digest:
        return LIB
    OUT_DIR.mkdir(exist_ok=True)
    inc = [f"-I{p}" for p in cpp_extension.include_paths()] + [f"-I{sysconfig.get_paths()['include']}",
                                                               f"-I{files[0].parent}"]
    abi = f"-D_GLIBCXX_USE_CXX11_ABI={int(torch.compiled_with_cxx11_abi())}"
    defs = [abi, "-DTORCH_EXTENSION_NAME=nanovllm_paged_kv_ref", "-DTORCH_API_INCLUDE_EXTENSION_H"]
    cuda_home = Path(cpp_extension.CUDA_HOME or "/usr/local/cuda")
    nvcc = cuda_home / "bin" / "nvcc"
    cu_obj, cpp_obj = OUT_DIR / "paged_kv_cuda.o", OUT_DIR / "paged_kv.o"
    cmds = [
        [str(nvcc), *ARCH, "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", *defs, *inc, "-c",
         str(files[1]), "-o", str(cu_obj)],
        ["g++", "-O3", "-std=c++17", "-fPIC", *defs, *inc, f"-I{cuda_home / 'include'}", "-c", str(files[0]),
         "-o", str(cpp_obj)],
        ["g++", "-shared", str(cpp_obj), str(cu_obj), "-o", str(LIB), f"-L{cpp_extension.library_paths()[0]}",
         "-lc10", "-lc10_cuda", "-ltorch_cpu", "-ltorch_cuda", "-ltorch", f"-L{cuda_home / 'lib64'}", "-lcudart"],
    ]
    for cmd in cmds:
        if verbose:
            print(" ".join(cmd), flush=True)
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"building the reference extension failed:\n{' '.join(cmd)}\n{r.stderr[-3000:]}")
    cu_obj.unlink()
    cpp_obj.unlink()
    stamp.write_text(digest + "\n")
    return LIB


if __name__ == "__main__":
    out = build(verbose="-v" in sys.argv)
    print(out if out else "reference checkout not found (set NANOINFER_REF)")
