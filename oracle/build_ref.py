"""Build recipe for oracle/_ref: the mLLM reference runtime compiled from its own sources.

Test infrastructure only (the checker and the CPU baseline), never product code.

The reference (pym2282/mLLM) is header-only C++17 on LibTorch for the attention path
(src/core/runtime/{Attention,RoPE,KVCache,RMSNorm,Linear,MLP,TransformerBlock}.h).
Its own CMakeLists.txt is Windows-only, so this recipe compiles oracle/ref_binding.cpp,
which #includes those headers straight from the reference tree, with g++ against the
installed LibTorch.  The output goes to oracle/_ref/ (git-ignored; it is copied with the rest
of the working tree to machines that do not have the reference tree).

Usage:  python oracle/build_ref.py [--reference /path/to/mLLM] [--force]

The reference tree defaults to $MLLM_REFERENCE_DIR, else a directory named `reference` beside
this repository's checkout.
"""
from __future__ import annotations

import argparse
import os
import subprocess
import sys
import sysconfig

HERE = os.path.dirname(os.path.abspath(__file__))
OUT_DIR = os.path.join(HERE, "_ref")
MODULE = "mllm_ref"
DEFAULT_REFERENCE = (os.environ.get("MLLM_REFERENCE_DIR")
                     or os.path.join(os.path.dirname(os.path.dirname(HERE)), "reference"))


def output_path() -> str:
    return os.path.join(OUT_DIR, MODULE + sysconfig.get_config_var("EXT_SUFFIX"))


def build(reference: str = DEFAULT_REFERENCE, force: bool = False, verbose: bool = True) -> str | None:
    """Compile the reference binding.  Returns the .so path, or None if the tree is absent."""
    src_root = os.path.join(reference, "src")
    if not os.path.isdir(os.path.join(src_root, "core", "runtime")):
        if verbose:
            print(f"[oracle/_ref] reference tree not found at {reference}; skipping", file=sys.stderr)
        return None
    out = output_path()
    binding = os.path.join(HERE, "ref_binding.cpp")
    if (not force and os.path.exists(out)
            and os.path.getmtime(out) >= os.path.getmtime(binding)):
        return out
    os.makedirs(OUT_DIR, exist_ok=True)
    import torch
    from torch.utils import cpp_extension as ce

    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    cmd = ["g++", "-O2", "-std=c++17", "-shared", "-fPIC", "-w",
           f"-D_GLIBCXX_USE_CXX11_ABI={abi}", f"-DTORCH_EXTENSION_NAME={MODULE}",
           f"-I{sysconfig.get_paths()['include']}", f"-I{src_root}",
           f"-I{os.path.join(src_root, 'core', 'runtime')}"]
    for p in ce.include_paths():
        cmd.append(f"-I{p}")
    # the runtime is header-only except the sampler, whose source is compiled alongside
    cmd += [binding, os.path.join(src_root, "core", "runtime", "Sampler.cpp"), "-o", out]
    for p in ce.library_paths():
        cmd += [f"-L{p}", f"-Wl,-rpath,{p}"]
    cmd += ["-ltorch", "-ltorch_cpu", "-lc10", "-ltorch_python"]
    if verbose:
        print("[oracle/_ref]", " ".join(cmd), file=sys.stderr)
    subprocess.run(cmd, check=True)
    return out


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=DEFAULT_REFERENCE)
    ap.add_argument("--force", action="store_true")
    a = ap.parse_args()
    print(build(a.reference, a.force))


if __name__ == "__main__":
    main()
