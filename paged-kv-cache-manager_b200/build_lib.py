"""Build recipe of libkvpage_b200.so (CUDA kernels for sm_100a + C ABI + C++17 host control plane).

Compiles every source in csrc/ with nvcc (host code through the system C++ compiler) into
_build/*.o and links the shared library next to this file.  Incremental: a source is rebuilt when it or
any header is newer than its object.  Usable as `python build_lib.py [--force]`.
"""
from __future__ import annotations

import concurrent.futures as cf
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "libkvpage_b200.so")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON = ["-std=c++17", "-O3", "-DNDEBUG", "-I", os.path.join(ROOT, "include"), "-I", CSRC]
CU_FLAGS = ARCH + COMMON + ["-lineinfo", "--expt-relaxed-constexpr", "-Xcompiler", "-fPIC,-fvisibility=hidden",
                            "-Xptxas", "-warn-spills"]
CPP_FLAGS = ARCH + COMMON + ["-Xcompiler", "-fPIC,-fvisibility=hidden,-Wall,-Wextra"]


def _sources():
    out = []
    for d, _, files in os.walk(CSRC):
        for f in sorted(files):
            if f.endswith((".cu", ".cpp")):
                out.append(os.path.join(d, f))
    return out


def _headers():
    hs = []
    for base in (CSRC, os.path.join(ROOT, "include")):
        for d, _, files in os.walk(base):
            hs += [os.path.join(d, f) for f in files if f.endswith((".h", ".cuh"))]
    return hs


def _obj(src):
    rel = os.path.relpath(src, CSRC).replace(os.sep, "_")
    return os.path.join(BUILD, rel + ".o")


def _compile(src, verbose):
    obj = _obj(src)
    flags = CU_FLAGS if src.endswith(".cu") else CPP_FLAGS
    cmd = [NVCC] + flags + ["-c", src, "-o", obj]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if verbose or r.returncode:
        sys.stderr.write(" ".join(cmd) + "\n" + r.stdout + r.stderr)
    else:
        # register spills are a performance bug worth seeing in every build
        for line in r.stderr.splitlines():
            if "spill" in line:
                sys.stderr.write(f"{os.path.basename(src)}: {line.strip()}\n")
    if r.returncode:
        raise RuntimeError(f"compilation failed: {src}")
    return obj


def build(force: bool = False, verbose: bool = False) -> str:
    """Compiles what changed and links libkvpage_b200.so; returns the library path."""
    os.makedirs(BUILD, exist_ok=True)
    srcs = _sources()
    newest_header = max((os.path.getmtime(h) for h in _headers()), default=0.0)
    todo = []
    for s in srcs:
        o = _obj(s)
        if force or not os.path.exists(o) or os.path.getmtime(o) < max(os.path.getmtime(s), newest_header):
            todo.append(s)
    if todo:
        with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 2)) as ex:
            list(ex.map(lambda s: _compile(s, verbose), todo))
    objs = [_obj(s) for s in srcs]
    if force or todo or not os.path.exists(LIB) or os.path.getmtime(LIB) < max(os.path.getmtime(o) for o in objs):
        tmp = LIB + ".tmp"
        cmd = [NVCC] + ARCH + ["-shared", "-o", tmp] + objs + ["-Xlinker", "--exclude-libs,ALL",
                                                                "-Xlinker", "-Bsymbolic", "-lpthread", "-ldl"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if verbose or r.returncode:
            sys.stderr.write(" ".join(cmd) + "\n" + r.stdout + r.stderr)
        if r.returncode:
            raise RuntimeError("link failed")
        os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
