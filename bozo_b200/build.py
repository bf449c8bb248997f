"""Build ``bozo_b200/_lib/libbozo_tension.so`` from ``bozo_b200/csrc/*.cu``.

Plain nvcc for sm_100a (``-gencode arch=compute_100a,code=sm_100a``), one
object per source compiled in parallel, linked into one shared library with
the CUDA runtime linked statically, so the library loads without a GPU
driver (symbol checks on CPU hosts) and carries no framework dependency.

    python -m bozo_b200.build            # incremental
    python -m bozo_b200.build --force    # rebuild everything
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
INCLUDE = os.path.join(ROOT, "include")
OUT_DIR = os.path.join(PKG, "_lib")
BUILD_DIR = os.path.join(ROOT, "_build")
LIB_NAME = "libbozo_tension.so"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC",
              "--expt-relaxed-constexpr", "-Xptxas", "-v"]


def nvcc() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(cand):
        raise RuntimeError("nvcc not found; the CUDA toolkit is required to build")
    return cand


def sources():
    return sorted(os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith(".cu"))


def headers():
    hs = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cuh", ".h"))]
    hs += [os.path.join(INCLUDE, f) for f in os.listdir(INCLUDE) if f.endswith(".h")]
    return hs


def _newer(src_list, target) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(s) > t for s in src_list)


def _compile(src: str, force: bool, verbose: bool) -> tuple[str, str]:
    obj = os.path.join(BUILD_DIR, os.path.basename(src) + ".o")
    if not force and not _newer([src] + headers(), obj):
        return obj, ""
    cmd = [nvcc(), *ARCH, *NVCC_FLAGS, "-I", INCLUDE, "-I", CSRC, "-c", src, "-o", obj]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src}:\n{r.stdout}\n{r.stderr}")
    return obj, (r.stdout + r.stderr) if verbose else ""


def build(force: bool = False, verbose: bool = False) -> str:
    os.makedirs(OUT_DIR, exist_ok=True)
    os.makedirs(BUILD_DIR, exist_ok=True)
    srcs = sources()
    with cf.ThreadPoolExecutor(max_workers=min(8, len(srcs))) as ex:
        results = list(ex.map(lambda s: _compile(s, force, verbose), srcs))
    objs = [o for o, _ in results]
    for _, log in results:
        if log:
            sys.stderr.write(log)
    lib = os.path.join(OUT_DIR, LIB_NAME)
    if force or _newer(objs, lib):
        cmd = [nvcc(), *ARCH, "-shared", "-cudart", "static", "-o", lib, *objs,
               "-lrt", "-ldl", "-lpthread"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    return lib


EXT_SRC = os.path.join(CSRC, "host", "torch_ext.cpp")
EXT_NAME = "_torch_ext"


def ext_path() -> str:
    import sysconfig
    return os.path.join(OUT_DIR, EXT_NAME + sysconfig.get_config_var("EXT_SUFFIX"))


def build_ext(force: bool = False) -> str:
    """Compile the PyTorch C++ extension (csrc/host/torch_ext.cpp) against the
    installed torch and link it to the C-ABI library beside it ($ORIGIN)."""
    import sysconfig
    import torch
    from torch.utils import cpp_extension as ce
    lib = os.path.join(OUT_DIR, LIB_NAME)
    out = ext_path()
    if not force and not _newer([EXT_SRC, lib] + headers(), out):
        return out
    torch_lib = ce.library_paths()[0]
    cuda_inc = os.path.join(os.path.dirname(os.path.dirname(nvcc())), "include")
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    cmd = ["g++", "-O2", "-std=c++17", "-shared", "-fPIC", "-w",
           f"-D_GLIBCXX_USE_CXX11_ABI={abi}", f"-DTORCH_EXTENSION_NAME={EXT_NAME}",
           "-DTORCH_API_INCLUDE_EXTENSION_H",
           *[f"-I{p}" for p in ce.include_paths()], f"-I{sysconfig.get_paths()['include']}",
           f"-I{cuda_inc}", f"-I{INCLUDE}", EXT_SRC, "-o", out,
           f"-L{torch_lib}", "-lc10", "-ltorch", "-ltorch_cpu", "-ltorch_python", "-lc10_cuda",
           "-ltorch_cuda", f"-L{OUT_DIR}", "-lbozo_tension",
           "-Wl,-rpath,$ORIGIN", f"-Wl,-rpath,{torch_lib}"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"torch extension build failed:\n{r.stdout}\n{r.stderr}")
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true", help="print ptxas resource usage")
    a = ap.parse_args()
    print(build(force=a.force, verbose=a.verbose))
    print(build_ext(force=a.force))


if __name__ == "__main__":
    main()
