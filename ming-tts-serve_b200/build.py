"""Builds libming_cuda.so (the sm_100a kernels + the C ABI of include/ming_cuda.h)
in-tree with nvcc. Objects go to build/ next to this file; the library lands
next to this file so it travels with the source tree.

    python ming-tts-serve_b200/build.py [-j N] [--force]
"""
import argparse
import os
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
OBJ = os.path.join(HERE, "build")
LIB = os.path.join(HERE, "libming_cuda.so")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-Xcompiler", "-O3",
         "--expt-relaxed-constexpr", "-Xptxas", "-O3"]


def _nvcc():
    for c in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", "nvcc"):
        if c and (os.path.isabs(c) and os.path.exists(c) or not os.path.isabs(c)):
            return c
    return "nvcc"


def _sources():
    return sorted(f for f in os.listdir(CSRC) if f.endswith((".cu", ".cpp")))


def _headers_mtime():
    paths = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cuh", ".h"))]
    paths.append(os.path.join(HERE, "..", "include", "ming_cuda.h"))
    return max(os.path.getmtime(p) for p in paths if os.path.exists(p))


def build(jobs=None, force=False, verbose=False):
    os.makedirs(OBJ, exist_ok=True)
    nvcc = _nvcc()
    hdr = _headers_mtime()
    todo = []
    objs = []
    for src in _sources():
        s = os.path.join(CSRC, src)
        o = os.path.join(OBJ, src + ".o")
        objs.append(o)
        if force or not os.path.exists(o) or os.path.getmtime(o) < max(os.path.getmtime(s), hdr):
            todo.append((s, o))

    def compile_one(so):
        s, o = so
        cmd = [nvcc] + ARCH + FLAGS + ["-c", s, "-o", o]
        if s.endswith(".cpp"):
            cmd = [nvcc] + ["-std=c++17", "-O3", "-Xcompiler", "-fPIC", "-x", "c++", "-c", s, "-o", o]
        r = subprocess.run(cmd, capture_output=True, text=True)
        return s, r.returncode, r.stdout + r.stderr

    jobs = jobs or min(8, os.cpu_count() or 4)
    with ThreadPoolExecutor(jobs) as ex:
        for s, rc, out in ex.map(compile_one, todo):
            if verbose or rc:
                sys.stderr.write(out)
            if rc:
                raise RuntimeError(f"nvcc failed on {s}")
    if todo or not os.path.exists(LIB):
        cmd = [nvcc] + ARCH + ["-shared", "-o", LIB] + objs + ["-lcudart"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode:
            sys.stderr.write(r.stdout + r.stderr)
            raise RuntimeError("link failed")
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("-j", type=int, default=None)
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-v", action="store_true")
    a = ap.parse_args()
    print(build(a.j, a.force, a.v))
