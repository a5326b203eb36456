"""Build ``dsv4_plugin/libdsv4moe.so`` (the C-ABI CUDA library) in-tree.

    python deepseek-v4-flash-offload_b200/build_ext.py [-v] [--force]

Compiles every ``csrc/*.cu`` / ``csrc/*.cpp`` with nvcc for sm_100a
(``-gencode arch=compute_100a,code=sm_100a -lineinfo -O3``) into objects
under ``_build/`` (git-ignored), in parallel, and links one shared library
with the CUDA runtime linked statically (the library carries no torch
dependency; callers pass raw pointers and streams).  Rebuilds only what
changed unless ``--force``.
"""

from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
INCLUDE = os.path.join(os.path.dirname(HERE), "include")
BUILD = os.path.join(os.path.dirname(HERE), "_build")
OUT = os.path.join(HERE, "dsv4_plugin", "libdsv4moe.so")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-std=c++17", "-O3", "-lineinfo", "-Xcompiler", "-fPIC,-O3", "--expt-relaxed-constexpr",
              "-DNDEBUG", "-I" + INCLUDE]


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def _sources():
    return sorted(os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cu", ".cpp")))


def _deps_mtime():
    files = [os.path.join(CSRC, f) for f in os.listdir(CSRC)] + [os.path.join(INCLUDE, f) for f in os.listdir(INCLUDE)]
    return max(os.path.getmtime(f) for f in files)


def _compile(nvcc, src, obj, verbose, extra):
    cmd = [nvcc, *ARCH, *NVCC_FLAGS, *extra, "-c", src, "-o", obj]
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {os.path.basename(src)}:\n{r.stdout}\n{r.stderr}")
    return r.stderr


def build(verbose: bool = False, force: bool = False, ptxas_info: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    nvcc = _nvcc()
    srcs = _sources()
    newest = _deps_mtime()
    if (not force and os.path.exists(OUT) and os.path.getmtime(OUT) >= newest
            and os.path.getmtime(OUT) >= os.path.getmtime(__file__)):
        return OUT
    extra = ["-Xptxas", "-v"] if ptxas_info else []
    objs = [os.path.join(BUILD, os.path.basename(s) + ".o") for s in srcs]
    with cf.ThreadPoolExecutor(max_workers=min(8, len(srcs))) as ex:
        futs = {ex.submit(_compile, nvcc, s, o, verbose, extra): s for s, o in zip(srcs, objs)}
        for f in cf.as_completed(futs):
            msg = f.result()
            if ptxas_info and msg:
                print(f"== {os.path.basename(futs[f])}\n{msg}", flush=True)
    tmp = OUT + ".tmp"
    cmd = [nvcc, *ARCH, "-shared", "-cudart", "static", "-o", tmp, *objs, "-lpthread", "-ldl", "-lrt"]
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    os.replace(tmp, OUT)
    return OUT


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("-v", "--verbose", action="store_true")
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--ptxas-info", action="store_true", help="print -Xptxas -v register/smem usage")
    a = ap.parse_args(argv)
    print(build(a.verbose, a.force or a.ptxas_info, a.ptxas_info))


if __name__ == "__main__":
    sys.exit(main())
