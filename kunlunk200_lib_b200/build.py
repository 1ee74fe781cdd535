"""In-tree build of libkunlunk200.so.0 for sm_100a.

    python -m kunlunk200_lib_b200.build [--force] [--verbose]

Compiles every CUDA and C++ source under ``csrc/`` with nvcc
(``-gencode arch=compute_100a,code=sm_100a -lineinfo``), links them into
``lib/libkunlunk200.so.0.7.12`` with SONAME ``libkunlunk200.so.0`` (the
reference's packaging contract, CMakeLists.txt:47-57) and creates the
``libkunlunk200.so.0`` / ``libkunlunk200.so`` links.  Objects go to
``_build/`` (ignored by git).  nvcc cross-compiles, so no GPU is needed.
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
BUILD = os.path.join(ROOT, "_build")
LIBDIR = os.path.join(PKG, "lib")
VERSION = "0.7.12"
SONAME = "libkunlunk200.so.0"
REALNAME = f"libkunlunk200.so.{VERSION}"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC",
          f"-I{os.path.join(ROOT, 'include')}", f"-I{CSRC}"]


def nvcc() -> str:
    for cand in (shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def _sources():
    out = []
    for name in sorted(os.listdir(CSRC)):
        if name.endswith((".cu", ".cpp")):
            out.append(os.path.join(CSRC, name))
    return out


def _headers_mtime() -> float:
    paths = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".h", ".cuh"))]
    inc = os.path.join(ROOT, "include")
    for dirpath, _, files in os.walk(inc):
        paths += [os.path.join(dirpath, f) for f in files]
    return max((os.path.getmtime(p) for p in paths), default=0.0)


def _compile(src: str, force: bool, verbose: bool) -> str:
    obj = os.path.join(BUILD, os.path.basename(src) + ".o")
    if not force and os.path.exists(obj):
        if os.path.getmtime(obj) >= max(os.path.getmtime(src), _headers_mtime()):
            return obj
    cmd = [nvcc(), *ARCH, *COMMON, "-c", src, "-o", obj]
    if src.endswith(".cu"):
        cmd += ["-Xptxas", "-v"] if verbose else []
        cmd += ["--expt-relaxed-constexpr"]
    res = subprocess.run(cmd, capture_output=True, text=True)
    log = os.path.join(BUILD, os.path.basename(src) + ".log")
    with open(log, "w") as f:
        f.write(" ".join(cmd) + "\n" + res.stdout + res.stderr)
    if res.returncode != 0:
        sys.stderr.write(res.stdout + res.stderr)
        raise RuntimeError(f"nvcc failed on {src}")
    if verbose:
        sys.stdout.write(res.stderr)
    return obj


def build(force: bool = False, verbose: bool = False) -> str:
    """Compile and link; returns the path of lib/libkunlunk200.so.0."""
    os.makedirs(BUILD, exist_ok=True)
    os.makedirs(LIBDIR, exist_ok=True)
    srcs = _sources()
    with cf.ThreadPoolExecutor(max_workers=min(8, len(srcs))) as ex:
        objs = list(ex.map(lambda s: _compile(s, force, verbose), srcs))
    real = os.path.join(LIBDIR, REALNAME)
    if force or not os.path.exists(real) or os.path.getmtime(real) < max(os.path.getmtime(o) for o in objs):
        cmd = [nvcc(), *ARCH, "-shared", "-o", real, *objs, "-Xlinker", f"-soname={SONAME}", "-lpthread"]
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            sys.stderr.write(res.stdout + res.stderr)
            raise RuntimeError("link failed")
    for link in (SONAME, "libkunlunk200.so"):
        p = os.path.join(LIBDIR, link)
        if os.path.islink(p) or os.path.exists(p):
            os.remove(p)
        os.symlink(REALNAME if link == SONAME else SONAME, p)
    return os.path.join(LIBDIR, SONAME)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    a = ap.parse_args()
    print(build(force=a.force, verbose=a.verbose))


if __name__ == "__main__":
    main()
