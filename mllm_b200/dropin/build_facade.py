"""Compile recipes for the C++ drop-in headers (mllm_b200/dropin/core/runtime/*.h).

1. `check_runners()` compiles the reference's UNCHANGED model runners (QwenRunner.cpp,
   LlamaRunner.cpp) with this directory ahead of the reference's own include path, proving
   that the drop-in headers keep every symbol and signature the runners use.  It needs the
   reference tree (build container only) and writes objects under mllm_b200/_build/.
2. `build_runner_module(flavor)` links the same unchanged runners into a Python module, built
   once on the reference's own runtime headers and once on the drop-in headers, which the GPU
   tests and the generate benchmark load side by side.

The reference tree is found at $MLLM_REFERENCE_DIR, else in a directory named `reference` beside
this repository's checkout; where neither exists the recipes are skipped.

The reference tree spells the runner interface header `ImodelRunner.h` but includes it as
`IModelRunner.h` (works only on case-insensitive file systems), so a one-file shim directory
with that name is generated under mllm_b200/_build/shim.
"""
from __future__ import annotations

import os
import subprocess
import sys
import sysconfig

HERE = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.dirname(HERE)
ROOT = os.path.dirname(PKG)
BUILD = os.path.join(PKG, "_build")


def reference_dir() -> str:
    """The reference tree: $MLLM_REFERENCE_DIR, else `reference` beside the repository."""
    return os.environ.get("MLLM_REFERENCE_DIR") or os.path.join(os.path.dirname(ROOT), "reference")


REFERENCE = reference_dir()


def _torch_flags():
    import torch
    from torch.utils import cpp_extension as ce
    inc = [f"-I{p}" for p in ce.include_paths()] + ["-I/usr/local/cuda/include"]
    libs = []
    for p in ce.library_paths():
        libs += [f"-L{p}", f"-Wl,-rpath,{p}"]
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    return inc, libs, [f"-D_GLIBCXX_USE_CXX11_ABI={abi}"]


def _shim(reference: str) -> str:
    d = os.path.join(BUILD, "shim", "models", "base")
    os.makedirs(d, exist_ok=True)
    link = os.path.join(d, "IModelRunner.h")
    target = os.path.join(reference, "src", "models", "base", "ImodelRunner.h")
    if not os.path.exists(link):
        with open(link, "w") as f:
            f.write(f'#include "{target}"\n')
    return os.path.join(BUILD, "shim")


def include_flags(reference: str = REFERENCE) -> list[str]:
    """Drop-in headers first, then the C ABI, then the reference tree."""
    return [f"-I{HERE}", f"-I{os.path.join(ROOT, 'include')}", f"-I{_shim(reference)}",
            f"-I{os.path.join(reference, 'src')}", f"-I{os.path.join(reference, 'external')}"]


def check_runners(reference: str = REFERENCE, verbose: bool = False) -> list[str]:
    if not os.path.isdir(os.path.join(reference, "src", "models")):
        raise FileNotFoundError("reference tree not present")
    inc, _, defs = _torch_flags()
    os.makedirs(BUILD, exist_ok=True)
    outs = []
    for src in ("models/qwen/QwenRunner.cpp", "models/llama/LlamaRunner.cpp"):
        obj = os.path.join(BUILD, os.path.basename(src).replace(".cpp", ".o"))
        cmd = ["g++", "-std=c++17", "-O1", "-fPIC", "-w", "-c", *defs, *include_flags(reference), *inc,
               os.path.join(reference, "src", src), "-o", obj]
        if verbose:
            print(" ".join(cmd), file=sys.stderr)
        subprocess.run(cmd, check=True)
        outs.append(obj)
    return outs


RUNNER_SOURCES = ["models/qwen/QwenRunner.cpp", "models/llama/LlamaRunner.cpp", "core/runtime/Sampler.cpp",
                  "tokenizer/BpeTokenizer.cpp", "tokenizer/LlamaTokenizer.cpp", "tokenizer/QwenTokenizer.cpp",
                  "tokenizer/TokenizerJsonLoader.cpp"]


def runner_module_path(flavor: str) -> str:
    ext = sysconfig.get_config_var("EXT_SUFFIX")
    if flavor == "reference":
        return os.path.join(ROOT, "oracle", "_ref", "mllm_ref_runner" + ext)
    return os.path.join(ROOT, "tests", "facade", "mllm_dropin_runner" + ext)


def build_runner_module(flavor: str, reference: str = REFERENCE, verbose: bool = False, force: bool = False) -> str:
    """Compile tests/facade/runner_binding.cpp with the reference's unchanged runners, either
    against the reference's own runtime headers ("reference") or with the drop-in headers
    first ("dropin").  Returns the module path."""
    import concurrent.futures as cf
    assert flavor in ("reference", "dropin")
    if not os.path.isdir(os.path.join(reference, "src", "models")):
        raise FileNotFoundError("reference tree not present")
    out = runner_module_path(flavor)
    binding = os.path.join(ROOT, "tests", "facade", "runner_binding.cpp")
    deps = [binding] + ([os.path.join(HERE, "core", "runtime", f) for f in os.listdir(os.path.join(HERE, "core", "runtime"))]
                        if flavor == "dropin" else [])
    if not force and os.path.exists(out) and all(os.path.getmtime(d) <= os.path.getmtime(out) for d in deps):
        return out
    inc, libs, defs = _torch_flags()
    if flavor == "dropin":
        from mllm_b200 import build as libbuild
        lib = libbuild.build()
        incs = include_flags(reference)
        extra = [f"-L{os.path.dirname(lib)}", "-Wl,-rpath,$ORIGIN/../../mllm_b200/lib", "-lmllm_attn"]
        defs = defs + ["-DMLLM_DROPIN"]
    else:
        incs = [f"-I{_shim(reference)}", f"-I{os.path.join(reference, 'src')}",
                f"-I{os.path.join(reference, 'external')}"]
        extra = []
    obj_dir = os.path.join(BUILD, "runner_" + flavor)
    os.makedirs(obj_dir, exist_ok=True)
    os.makedirs(os.path.dirname(out), exist_ok=True)
    # the drop-in Sampler.h is header-only: the reference's Sampler.cpp is not linked with it
    sources = [x for x in RUNNER_SOURCES if not (flavor == "dropin" and x == "core/runtime/Sampler.cpp")]
    srcs = [binding] + [os.path.join(reference, "src", x) for x in sources]
    cflags = ["g++", "-std=c++17", "-O2", "-fPIC", "-w", *defs, "-DTORCH_EXTENSION_NAME=" + os.path.basename(out).split(".")[0],
              f"-I{sysconfig.get_paths()['include']}", *incs, *inc]

    def compile_one(src):
        obj = os.path.join(obj_dir, os.path.basename(src).replace(".cpp", ".o"))
        cmd = cflags + ["-c", src, "-o", obj]
        if verbose:
            print(" ".join(cmd), file=sys.stderr)
        subprocess.run(cmd, check=True)
        return obj

    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as ex:
        objs = list(ex.map(compile_one, srcs))
    cmd = ["g++", "-shared", "-fPIC", *objs, "-o", out, *libs, *extra,
           "-ltorch", "-ltorch_cpu", "-ltorch_cuda", "-lc10", "-lc10_cuda", "-ltorch_python"]
    if verbose:
        print(" ".join(cmd), file=sys.stderr)
    subprocess.run(cmd, check=True)
    return out


if __name__ == "__main__":
    print(check_runners(verbose=True))
    for fl in ("reference", "dropin"):
        print(build_runner_module(fl, verbose=True))
