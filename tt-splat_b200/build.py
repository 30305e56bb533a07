"""Build ``libttsplat_b200.so`` (sm_100a) in-tree with nvcc.

Each ``csrc/*.cu`` compiles to an object with relocatable device code (the device status word
is shared across translation units), then nvcc links them into one shared library next to this
file.  Objects are rebuilt only when a source or header is newer.  Usage:

    python tt-splat_b200/build.py            # or __graft_entry__.build()
"""
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "libttsplat_b200.so")
INCLUDE = os.path.join(os.path.dirname(HERE), "include")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-rdc=true", "-Xcompiler", "-fPIC", "-Xcompiler", "-O3",
         "--expt-relaxed-constexpr", "-I", INCLUDE]


def nvcc():
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found: the CUDA library cannot be built")


def _sources():
    return sorted(f for f in os.listdir(CSRC) if f.endswith(".cu"))


def _headers_mtime():
    paths = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cuh", ".h"))]
    paths += [os.path.join(INCLUDE, f) for f in os.listdir(INCLUDE)]
    return max((os.path.getmtime(p) for p in paths), default=0.0)


def build_library(verbose=True, extra_flags=()):
    os.makedirs(BUILD, exist_ok=True)
    cc = nvcc()
    hdr = _headers_mtime()
    jobs = []
    objs = []
    for src in _sources():
        s = os.path.join(CSRC, src)
        o = os.path.join(BUILD, src[:-3] + ".o")
        objs.append(o)
        if not os.path.exists(o) or os.path.getmtime(o) < max(os.path.getmtime(s), hdr):
            jobs.append([cc, *ARCH, *FLAGS, *extra_flags, "-c", s, "-o", o])
    with cf.ThreadPoolExecutor(max_workers=max(1, os.cpu_count() or 1)) as ex:
        for cmd, res in zip(jobs, ex.map(lambda c: subprocess.run(c, capture_output=True, text=True), jobs)):
            if verbose:
                print(" ".join(os.path.basename(x) if x.endswith((".cu", ".o")) else x for x in cmd[-3:]), flush=True)
            if res.returncode != 0:
                sys.stderr.write(res.stdout + res.stderr)
                raise RuntimeError(f"nvcc failed on {cmd[-3]}")
            if res.stderr.strip() and verbose:
                sys.stderr.write(res.stderr)
    if jobs or not os.path.exists(LIB) or os.path.getmtime(LIB) < max(os.path.getmtime(o) for o in objs):
        cmd = [cc, *ARCH, "-shared", "-o", LIB, *objs]
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            sys.stderr.write(res.stdout + res.stderr)
            raise RuntimeError("nvcc link failed")
    return LIB


if __name__ == "__main__":
    print(build_library())
