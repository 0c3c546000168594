"""In-tree build of the native libraries (sm_100a).

Produces, next to this file:

* ``lib/libtmjv.so`` -- the CUDA kernels behind the plain C ABI of
  ``include/torchmatch_b200.h`` (no torch dependency).
* ``lib/libtmjv_torch.so`` -- the ``TORCH_LIBRARY_IMPL(assignment, CUDA)``
  registration of ``jonker_dense_batch`` that calls into ``libtmjv.so``.

Run ``python torchmatch_b200/_build.py`` (``__graft_entry__.build()`` does); it is
run by path because importing the package requires the built libraries.
nvcc cross-compiles for sm_100a without a GPU present.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
import sysconfig
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
INCLUDE = ROOT / "include"
LIBDIR = PKG / "lib"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", *ARCH]


def _cuda_home() -> Path:
    env = os.environ.get("CUDA_HOME") or os.environ.get("CUDA_PATH")
    if env:
        return Path(env)
    nvcc = shutil.which("nvcc")
    if nvcc:
        return Path(nvcc).resolve().parent.parent
    return Path("/usr/local/cuda")


def _run(cmd: list[str]) -> None:
    print("+", " ".join(cmd), flush=True)
    subprocess.run(cmd, check=True)


def _stale(target: Path, deps: list[Path]) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def build_core(force: bool = False) -> Path:
    """nvcc -> lib/libtmjv.so (kernels + C ABI)."""
    LIBDIR.mkdir(exist_ok=True)
    out = LIBDIR / "libtmjv.so"
    deps = [CSRC / "jv_kernels.cu", INCLUDE / "torchmatch_b200.h"]
    if force or _stale(out, deps):
        nvcc = str(_cuda_home() / "bin" / "nvcc")
        _run(
            [nvcc, *NVCC_FLAGS, "-shared", f"-I{INCLUDE}", str(CSRC / "jv_kernels.cu"),
             "-o", str(out)]
        )
    return out


def build_torch_shim(force: bool = False) -> Path:
    """g++ -> lib/libtmjv_torch.so (TORCH_LIBRARY_IMPL over the C ABI)."""
    import torch
    from torch.utils import cpp_extension

    core = build_core(force)
    out = LIBDIR / "libtmjv_torch.so"
    deps = [CSRC / "jv_op.cpp", INCLUDE / "torchmatch_b200.h", core]
    if not (force or _stale(out, deps)):
        return out
    cuda = _cuda_home()
    incs = [*cpp_extension.include_paths(device_type="cuda"), str(cuda / "include"), str(INCLUDE)]
    libdirs = [*cpp_extension.library_paths(device_type="cuda"), str(LIBDIR)]
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    cmd = [
        "g++", "-O2", "-std=c++17", "-fPIC", "-shared",
        f"-D_GLIBCXX_USE_CXX11_ABI={abi}",
        *[f"-I{p}" for p in incs],
        str(CSRC / "jv_op.cpp"),
        *[f"-L{p}" for p in libdirs],
        "-ltmjv", "-lc10", "-lc10_cuda", "-ltorch_cpu", "-ltorch_cuda", "-ltorch",
        f"-L{cuda / 'lib64'}", "-lcudart",
        "-Wl,-rpath,$ORIGIN",
        "-o", str(out),
    ]
    _run(cmd)
    return out


def build(force: bool = False) -> None:
    build_torch_shim(force)


if __name__ == "__main__":
    build(force="--force" in sys.argv)
