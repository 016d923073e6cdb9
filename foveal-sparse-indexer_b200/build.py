"""Build libfovealpatt.so (the C-ABI CUDA library) in-tree for sm_100a.

    python foveal-sparse-indexer_b200/build.py [--force] [--verbose]

Compiles every ``csrc/*.cu`` with ``nvcc -gencode arch=compute_100a,code=sm_100a`` into one shared
library next to this file.  nvcc cross-compiles without a GPU.  The build is skipped when the library
is newer than every source and header.
"""

from __future__ import annotations

import argparse
import glob
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
INCLUDE = os.path.join(REPO, "include")
LIB_NAME = "libfovealpatt.so"
LIB_PATH = os.path.join(HERE, LIB_NAME)

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-std=c++17", "-lineinfo", "--expt-relaxed-constexpr", "-Xcompiler", "-fPIC",
              "-Xcompiler", "-fvisibility=hidden", "-DNDEBUG"]


def nvcc_path() -> str:
    cand = os.environ.get("NVCC") or shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(cand):
        raise RuntimeError("nvcc not found: set NVCC or put the CUDA toolkit on PATH")
    return cand


def sources():
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")))


def _inputs():
    return sources() + glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(INCLUDE, "*.h")) + [__file__]


def up_to_date() -> bool:
    if not os.path.exists(LIB_PATH):
        return False
    t = os.path.getmtime(LIB_PATH)
    return all(os.path.getmtime(p) <= t for p in _inputs())


def build(force: bool = False, verbose: bool = False, extra_flags=None) -> str:
    if not force and up_to_date():
        return LIB_PATH
    nvcc = nvcc_path()
    objdir = os.path.join(HERE, "_build")
    os.makedirs(objdir, exist_ok=True)
    objs = []
    flags = ARCH_FLAGS + NVCC_FLAGS + ["-I", INCLUDE, "-I", CSRC] + list(extra_flags or [])
    procs = []
    for src in sources():
        obj = os.path.join(objdir, os.path.basename(src) + ".o")
        cmd = [nvcc, *flags, "-c", src, "-o", obj]
        if verbose:
            print(" ".join(cmd), flush=True)
        procs.append((src, subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT)))
        objs.append(obj)
    failed = []
    for src, p in procs:
        out, _ = p.communicate()
        text = out.decode(errors="replace")
        if p.returncode != 0:
            failed.append((src, text))
        elif verbose and text.strip():
            print(text)
    if failed:
        msg = "\n".join(f"--- {s}\n{t}" for s, t in failed)
        raise RuntimeError(f"nvcc failed:\n{msg}")
    tmp = LIB_PATH + ".tmp"
    cmd = [nvcc, *ARCH_FLAGS, "-shared", "-o", tmp, *objs, "-lcudart"]
    if verbose:
        print(" ".join(cmd), flush=True)
    subprocess.run(cmd, check=True)
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--ptxas-v", action="store_true", help="print register/shared-memory usage")
    a = ap.parse_args(argv)
    extra = ["-Xptxas", "-v"] if a.ptxas_v else []
    print(build(force=a.force or a.ptxas_v, verbose=a.verbose or a.ptxas_v, extra_flags=extra))


if __name__ == "__main__":
    sys.exit(main())
