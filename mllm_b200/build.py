"""Build the sm_100a attention library in-tree: mllm_b200/lib/libmllm_attn.so.

    python -m mllm_b200.build [--force] [--verbose]

Every .cu file under mllm_b200/csrc is compiled with nvcc for sm_100a (whole-program device
code per file: no relocatable device code, which would make ptxas ignore setmaxnreg) and
linked into one shared library with the CUDA runtime linked statically and NCCL linked
dynamically (the libnccl.so.2 that PyTorch loads, found through an rpath).  The library exports only the
extern "C" entry points declared in include/mllm_attn.h.
"""
from __future__ import annotations

import argparse
import glob
import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
LIB_DIR = os.path.join(PKG, "lib")
OBJ_DIR = os.path.join(PKG, "_build")
LIB_NAME = "libmllm_attn.so"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-Xcompiler",
              "-fvisibility=hidden", "--expt-relaxed-constexpr", "-Xptxas", "-warn-spills"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def nccl_lib_dir() -> str:
    """Directory of the libnccl.so.2 that PyTorch itself loads (the library links the same one, so a
    process that holds both has one NCCL); the system copy otherwise."""
    import importlib.util
    spec = importlib.util.find_spec("nvidia")
    for base in (list(spec.submodule_search_locations) if spec and spec.submodule_search_locations else []):
        d = os.path.join(base, "nccl", "lib")
        if os.path.exists(os.path.join(d, "libnccl.so.2")):
            return d
    for d in ("/usr/lib/x86_64-linux-gnu", "/usr/local/cuda/lib64"):
        if os.path.exists(os.path.join(d, "libnccl.so.2")):
            return d
    raise RuntimeError("libnccl.so.2 not found")


def lib_path() -> str:
    return os.path.join(LIB_DIR, LIB_NAME)


def _sources():
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")))


def _deps():
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")) + glob.glob(os.path.join(CSRC, "*.cuh")) +
                  glob.glob(os.path.join(CSRC, "*.h")) + [os.path.join(ROOT, "include", "mllm_attn.h")])


def up_to_date() -> bool:
    out = lib_path()
    if not os.path.exists(out):
        return False
    t = os.path.getmtime(out)
    return all(os.path.getmtime(d) <= t for d in _deps())


def build(force: bool = False, verbose: bool = False, ptxas_verbose: bool = False) -> str:
    out = lib_path()
    if not force and up_to_date():
        return out
    os.makedirs(LIB_DIR, exist_ok=True)
    os.makedirs(OBJ_DIR, exist_ok=True)
    cc = nvcc()
    def compile_one(src):
        obj = os.path.join(OBJ_DIR, os.path.basename(src).replace(".cu", ".o"))
        cmd = [cc, *ARCH, *NVCC_FLAGS, "-I", os.path.join(ROOT, "include"), "-c", src, "-o", obj]
        if ptxas_verbose:
            cmd += ["-Xptxas", "-v"]
        if verbose:
            print(" ".join(cmd), file=sys.stderr)
        subprocess.run(cmd, check=True)
        return obj

    # one nvcc per translation unit, in parallel (each is independent whole-program device code)
    import concurrent.futures as cf
    with cf.ThreadPoolExecutor(max_workers=max(1, min(len(_sources()), os.cpu_count() or 1))) as ex:
        objs = list(ex.map(compile_one, _sources()))
    tmp = out + ".tmp"
    nccl_dir = nccl_lib_dir()
    cmd = [cc, *ARCH, "-shared", "-cudart", "static", *objs, "-o", tmp,
           "-Xcompiler", "-fPIC", "-Xlinker", "--exclude-libs,ALL",
           f"-L{nccl_dir}", "-Xlinker", f"-rpath,{nccl_dir}", "-l:libnccl.so.2"]
    if verbose:
        print(" ".join(cmd), file=sys.stderr)
    subprocess.run(cmd, check=True)
    os.replace(tmp, out)
    return out


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--ptxas-verbose", action="store_true")
    a = ap.parse_args()
    print(build(a.force, a.verbose, a.ptxas_verbose))


if __name__ == "__main__":
    main()
