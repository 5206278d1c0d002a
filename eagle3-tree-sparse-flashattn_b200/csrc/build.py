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


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--debug", action="store_true")
    ap.add_argument("--verbose-ptxas", action="store_true")
    args = ap.parse_args(argv)
    print(build(args.debug, args.verbose_ptxas))


if __name__ == "__main__":
    sys.exit(main())
