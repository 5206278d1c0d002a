"""Build libtsfa.so (sm_100a) next to the Python modules.

    python eagle3-tree-sparse-flashattn_b200/csrc/build.py [--debug] [--verbose-ptxas]

--debug builds libtsfa_debug.so: the same library with device-side bounds
checks on every metadata index the forward reads (-DTSFA_DEBUG).

nvcc cross-compiles for sm_100a without a GPU.  The library links only the
CUDA runtime (statically) and resolves driver entry points (TMA descriptor
encoding) at run time through cudaGetDriverEntryPoint.
"""

from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.dirname(HERE)
REPO = os.path.dirname(PKG)
SOURCES = ["tsfa_api.cu", "tsfa_meta.cu", "tsfa_fwd_tc.cu"]
OUT = os.path.join(PKG, "libtsfa.so")
OUT_DEBUG = os.path.join(PKG, "libtsfa_debug.so")
OUT_TORCH = os.path.join(PKG, "libtsfa_torch.so")


def nvcc_path() -> str:
    for cand in (shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def build(debug: bool = False, verbose_ptxas: bool = False, out: str | None = None) -> str:
    """Compile the sources (in parallel) and link the library.  The debug
    build (-DTSFA_DEBUG: device-side bounds checks on every metadata read)
    goes to libtsfa_debug.so unless `out` says otherwise."""
    out = out or (OUT_DEBUG if debug else OUT)
    build_dir = os.path.join(PKG, "_build_debug" if debug else "_build")
    os.makedirs(build_dir, exist_ok=True)
    flags = [
        "-gencode", "arch=compute_100a,code=sm_100a",
        "-std=c++17", "-O3", "-lineinfo",
        "-Xcompiler", "-fPIC,-fvisibility=hidden",
        "--expt-relaxed-constexpr",
        f"-I{os.path.join(REPO, 'include')}",
        f"-I{HERE}",
    ]
    if debug:
        flags += ["-DTSFA_DEBUG=1"]
    if verbose_ptxas:
        flags += ["-Xptxas", "-v"]
    objs = []
    nvcc = nvcc_path()
    procs = []
    for src in SOURCES:
        obj = os.path.join(build_dir, src.replace(".cu", ".o"))
        cmd = [nvcc, *flags, "-c", os.path.join(HERE, src), "-o", obj]
        procs.append((cmd, subprocess.Popen(cmd)))
        objs.append(obj)
    for cmd, proc in procs:
        if proc.wait() != 0:
            raise subprocess.CalledProcessError(proc.returncode, cmd)
    tmp = out + ".tmp"
    subprocess.run([nvcc, "-shared", "-gencode", "arch=compute_100a,code=sm_100a", *objs, "-o", tmp,
                    "-cudart", "static"], check=True)
    os.replace(tmp, out)
    return out


def build_torch_op(out: str = OUT_TORCH) -> str:
    """The PyTorch operator binding (torch.ops.tsfa.*, tsfa_torch_op.cpp): a
    host-only C++ library over libtsfa.so's C ABI, linked against the
    installed torch (no nvcc needed: it launches nothing itself)."""
    import torch
    from torch.utils import cpp_extension

    cuda_home = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    incs = [os.path.join(REPO, "include"), *cpp_extension.include_paths(), os.path.join(cuda_home, "include")]
    tlib = cpp_extension.library_paths()[0]
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    tmp = out + ".tmp"
    cmd = ["g++", "-std=c++17", "-O2", "-fPIC", "-shared", f"-D_GLIBCXX_USE_CXX11_ABI={abi}",
           *[f"-I{i}" for i in incs], os.path.join(HERE, "tsfa_torch_op.cpp"), "-o", tmp,
           f"-L{PKG}", "-ltsfa", f"-L{tlib}", "-lc10", "-lc10_cuda", "-ltorch_cpu", "-ltorch",
           "-Wl,-rpath,$ORIGIN", f"-Wl,-rpath,{tlib}"]
    subprocess.run(cmd, check=True)
    os.replace(tmp, out)
    return out


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--debug", action="store_true")
    ap.add_argument("--verbose-ptxas", action="store_true")
    ap.add_argument("--torch-op", action="store_true", help="build only the torch operator binding")
    args = ap.parse_args(argv)
    if args.torch_op:
        print(build_torch_op())
        return
    print(build(args.debug, args.verbose_ptxas))
    if not args.debug:
        print(build_torch_op())


if __name__ == "__main__":
    sys.exit(main())
