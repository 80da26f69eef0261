"""Ahead-of-time build of the sm_100a kernel library.

Every ``csrc/*.cu`` file is compiled with nvcc for ``sm_100a`` only and linked into
``fastafd_b200/_C/libfastafd_kernels.so`` (in-tree, so the binary travels with the
source tree to the GPU machine). The library exposes a plain C ABI that
``fastafd_b200.ops`` calls through ctypes; there is no runtime JIT.

The reference compiles its kernels at run time (tvm-ffi ``load_jit``,
python/minisgl/kernel/utils.py:48-124, and the DeepGEMM JIT,
python/minisgl/kernel/csrc/deepgemm/csrc/jit/compiler.hpp); a fixed set of
instantiations built once is the simpler fit for a single target architecture.
"""
from __future__ import annotations

import hashlib
import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
CSRC = PKG_DIR / "csrc"
OUT_DIR = PKG_DIR / "_C"
LIB_NAME = "libfastafd_kernels.so"

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-lineinfo", "-O3", "-std=c++17",
    "-Xcompiler", "-fPIC",
    "--expt-relaxed-constexpr",
]


def nvcc_path() -> str:
    cand = os.environ.get("NVCC") or shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(cand).exists():
        raise RuntimeError("nvcc not found; set NVCC")
    return cand


def _digest(paths) -> str:
    h = hashlib.sha256()
    for p in sorted(paths):
        h.update(p.name.encode())
        h.update(p.read_bytes())
    h.update(" ".join(NVCC_FLAGS).encode())
    return h.hexdigest()


def lib_path() -> Path:
    return OUT_DIR / LIB_NAME


def build_extension(force: bool = False, verbose: bool = False) -> Path:
    """Compile and link the kernel library; returns its path. Up-to-date builds are skipped."""
    sources = sorted(CSRC.glob("*.cu"))
    headers = sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.h"))
    OUT_DIR.mkdir(exist_ok=True)
    stamp = OUT_DIR / "build.stamp"
    digest = _digest(sources + headers)
    if not force and lib_path().exists() and stamp.exists() and stamp.read_text() == digest:
        return lib_path()
    nvcc = nvcc_path()

    def compile_one(src: Path) -> Path:
        obj = OUT_DIR / (src.stem + ".o")
        cmd = [nvcc, *NVCC_FLAGS, "-I", str(CSRC), "-c", str(src), "-o", str(obj)]
        if verbose:
            cmd.insert(1, "-Xptxas=-v")
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed for {src.name}:\n{r.stdout}\n{r.stderr}")
        if verbose:
            sys.stderr.write(r.stderr)
        return obj

    with ThreadPoolExecutor(max_workers=min(8, len(sources))) as ex:
        objs = list(ex.map(compile_one, sources))
    # The CUDA runtime is linked dynamically: the process already holds torch's libcudart.so.12,
    # so kernels, streams and allocations share one runtime instance with PyTorch.
    link = [nvcc, "-shared", "--cudart", "shared", "-o", str(lib_path()), *map(str, objs), "-gencode",
            "arch=compute_100a,code=sm_100a"]
    r = subprocess.run(link, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    stamp.write_text(digest)
    return lib_path()


NCCL_LIB_NAME = "libfastafd_nccl.so"


def nccl_lib_path() -> Path:
    return OUT_DIR / NCCL_LIB_NAME


def _nccl_dirs():
    import importlib.util

    spec = importlib.util.find_spec("nvidia.nccl")
    if spec is None or not spec.submodule_search_locations:
        return None
    base = Path(list(spec.submodule_search_locations)[0])
    return base / "include", base / "lib"


def build_nccl_wrapper(force: bool = False) -> Path:
    """Compile csrc/nccl/nccl_comm.cpp against the NCCL that ships with PyTorch. The library
    is resolved at run time from the already loaded libnccl.so.2 of the torch process."""
    src = CSRC / "nccl" / "nccl_comm.cpp"
    out = nccl_lib_path()
    OUT_DIR.mkdir(exist_ok=True)
    if not force and out.exists() and out.stat().st_mtime >= src.stat().st_mtime:
        return out
    dirs = _nccl_dirs()
    if dirs is None:
        raise RuntimeError("the nvidia.nccl package (NCCL headers and library) is not installed")
    inc, lib = dirs
    cmd = [nvcc_path(), "-O2", "-std=c++17", "-shared", "-Xcompiler", "-fPIC", "--cudart", "shared", "-I", str(inc),
           str(src), "-o", str(out), "-L", str(lib), "-l:libnccl.so.2", "-Xlinker", f"-rpath={lib}"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nccl wrapper build failed:\n{r.stdout}\n{r.stderr}")
    return out


HOST_LIB_NAME = "libfastafd_host.so"


def host_lib_path() -> Path:
    return OUT_DIR / HOST_LIB_NAME


def build_host_lib(force: bool = False) -> Path:
    """Compile csrc/host/host_runtime.cpp (control-plane helpers; no CUDA) with the host compiler."""
    src = CSRC / "host" / "host_runtime.cpp"
    out = host_lib_path()
    OUT_DIR.mkdir(exist_ok=True)
    if not force and out.exists() and out.stat().st_mtime >= src.stat().st_mtime:
        return out
    cxx = os.environ.get("CXX", "g++")
    r = subprocess.run([cxx, "-O2", "-std=c++17", "-shared", "-fPIC", str(src), "-o", str(out)],
                       capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"host library build failed:\n{r.stdout}\n{r.stderr}")
    return out


if __name__ == "__main__":
    build_host_lib(force="--force" in sys.argv)
    build_nccl_wrapper(force="--force" in sys.argv)
    print(build_extension(force="--force" in sys.argv, verbose="-v" in sys.argv))
