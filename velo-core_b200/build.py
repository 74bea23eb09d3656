"""Build libvelo_cuda.so in-tree with nvcc for sm_100a.

Usage: python velo-core_b200/build.py [--force] [--verbose]

Every .cu / .cpp under csrc/ is compiled with
  -gencode arch=compute_100a,code=sm_100a -lineinfo -O3
and linked (CUDA runtime linked statically) into velo-core_b200/libvelo_cuda.so.
Objects go to velo-core_b200/_build/ and are rebuilt when any source or header
is newer than the library.
"""
import argparse
import concurrent.futures as cf
import glob
import os
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
BUILD = os.path.join(PKG, "_build")
LIB = os.path.join(PKG, "libvelo_cuda.so")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + [
    "-lineinfo", "-O3", "-std=c++17", "--expt-relaxed-constexpr",
    "-Xcompiler", "-fPIC,-O2,-Wall,-fvisibility=hidden",
    "-I" + os.path.join(ROOT, "include"), "-I" + CSRC,
]


def nvcc():
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", "nvcc"):
        if cand and (os.path.isabs(cand) and os.path.exists(cand) or not os.path.isabs(cand)):
            return cand
    return "nvcc"


def sources():
    out = []
    for ext in ("cu", "cpp"):
        out += glob.glob(os.path.join(CSRC, "**", "*." + ext), recursive=True)
    return sorted(out)


def headers():
    hs = glob.glob(os.path.join(CSRC, "**", "*.h"), recursive=True)
    hs += glob.glob(os.path.join(CSRC, "**", "*.cuh"), recursive=True)
    hs += glob.glob(os.path.join(ROOT, "include", "*.h"))
    return hs


def _obj(src):
    rel = os.path.relpath(src, CSRC).replace(os.sep, "_")
    return os.path.join(BUILD, rel + ".o")


def _compile(src, verbose):
    obj = _obj(src)
    cmd = [nvcc()] + NVCC_FLAGS + ["-c", src, "-o", obj]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    r = subprocess.run(cmd, capture_output=True, text=True)
    return src, r.returncode, r.stdout + r.stderr


def build(force=False, verbose=False):
    os.makedirs(BUILD, exist_ok=True)
    srcs = sources()
    hdr_mtime = max([os.path.getmtime(h) for h in headers()] + [os.path.getmtime(__file__)])
    todo = []
    for s in srcs:
        o = _obj(s)
        if force or not os.path.exists(o) or os.path.getmtime(o) < max(os.path.getmtime(s), hdr_mtime):
            todo.append(s)
    if todo:
        with cf.ThreadPoolExecutor(max_workers=min(8, len(todo))) as ex:
            for src, rc, log in ex.map(lambda s: _compile(s, verbose), todo):
                if rc != 0 or verbose:
                    sys.stderr.write(f"--- {os.path.relpath(src, ROOT)}\n{log}")
                if rc != 0:
                    raise RuntimeError(f"nvcc failed on {src}")
    objs = [_obj(s) for s in srcs]
    if todo or not os.path.exists(LIB):
        # linked beside the library and renamed over it, so that a process loading it
        # meanwhile sees the old or the new file, never a partial one
        tmp = LIB + ".partial"
        cmd = [nvcc()] + ARCH + ["-shared", "-o", tmp] + objs + ["-ldl", "-lpthread"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            sys.stderr.write(r.stdout + r.stderr)
            raise RuntimeError("link of libvelo_cuda.so failed")
        os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    a = ap.parse_args()
    print(build(a.force, a.verbose))
