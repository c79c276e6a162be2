"""Build recipe for libfeml_b200.so (sm_100a only).

Compiles every .cu / .cpp under feml_b200/csrc with nvcc for
`-gencode arch=compute_100a,code=sm_100a` and links one shared library
in-tree at feml_b200/libfeml_b200.so (static CUDA runtime). Objects go to
feml_b200/_build/. Incremental: a source is recompiled when it or any header
is newer than its object.
"""
import concurrent.futures as cf
import glob
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "libfeml_b200.so")
REPO = os.path.dirname(HERE)
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC,-fvisibility=hidden",
         "-I" + os.path.join(REPO, "include"), "--expt-relaxed-constexpr",
         "-Xcudafe", "--diag_suppress=177"]


def _sources():
    return sorted(glob.glob(os.path.join(CSRC, "**", "*.cu"), recursive=True)
                  + glob.glob(os.path.join(CSRC, "**", "*.cpp"), recursive=True))


def _headers():
    return (glob.glob(os.path.join(CSRC, "**", "*.h"), recursive=True)
            + glob.glob(os.path.join(CSRC, "**", "*.cuh"), recursive=True)
            + glob.glob(os.path.join(REPO, "include", "*.h")))


def _obj(src):
    rel = os.path.relpath(src, CSRC).replace(os.sep, "_")
    return os.path.join(BUILD, rel + ".o")


def _compile(src, extra):
    obj = _obj(src)
    cmd = [NVCC, *ARCH, *FLAGS, *extra, "-c", src, "-o", obj]
    if src.endswith(".cpp"):
        cmd = [NVCC, *FLAGS, *extra, "-x", "c++", "-c", src, "-o", obj]
    r = subprocess.run(cmd, capture_output=True, text=True)
    return src, r.returncode, r.stdout + r.stderr


def build(force=False, verbose=False, extra=()):
    os.makedirs(BUILD, exist_ok=True)
    srcs = _sources()
    newest_hdr = max((os.path.getmtime(h) for h in _headers()), default=0)
    todo = []
    for s in srcs:
        o = _obj(s)
        if force or not os.path.exists(o) or os.path.getmtime(o) < max(os.path.getmtime(s), newest_hdr):
            todo.append(s)
    with cf.ThreadPoolExecutor(max_workers=os.cpu_count() or 4) as ex:
        for src, rc, out in ex.map(lambda s: _compile(s, list(extra)), todo):
            if verbose or rc:
                sys.stderr.write(f"== {os.path.relpath(src, REPO)}\n{out}")
            if rc:
                raise RuntimeError(f"nvcc failed on {src}")
    objs = [_obj(s) for s in srcs]
    if force or todo or not os.path.exists(LIB):
        tmp = LIB + f".tmp{os.getpid()}"
        subprocess.check_call([NVCC, *ARCH, "-shared", "-o", tmp, *objs, "-lpthread"])
        os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    extra = []
    if "--ptxas-v" in sys.argv:
        extra = ["-Xptxas", "-v"]
    print(build(force="--force" in sys.argv or bool(extra), verbose="-v" in sys.argv or bool(extra), extra=extra))
