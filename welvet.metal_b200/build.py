"""Build recipe of libwelvet_b200.so (sm_100a) — run as `python build.py` or via
__graft_entry__.build(). Compiles every .cu/.cpp under csrc/ and host/ with nvcc
(`-gencode arch=compute_100a,code=sm_100a -lineinfo`) into objects under
_build/ and links the shared library in-tree (lib/libwelvet_b200.so), so it
travels with the repository snapshot. Incremental: a source is recompiled when
it or any header of the package is newer than its object."""
from __future__ import annotations

import concurrent.futures as cf
import glob
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
BUILD = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "lib", "libwelvet_b200.so")
# the MHA wire tool (WVM1 / WMV1 readers, tools/welvet_dense_fwd.cpp), linked to LIB
TOOL = os.path.join(HERE, "lib", "welvet_dense_fwd")
TOOL_SRC = os.path.join(HERE, "tools", "welvet_dense_fwd.cpp")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON = ["-std=c++17", "-O3", "-lineinfo", "-Xcompiler", "-fPIC,-fvisibility=hidden",
          f"-I{os.path.join(ROOT, 'include')}"]


def _sources():
    out = []
    for sub in ("csrc", "host"):
        out += sorted(glob.glob(os.path.join(HERE, sub, "*.cu")))
        out += sorted(glob.glob(os.path.join(HERE, sub, "*.cpp")))
    return out


def _headers():
    hs = []
    for sub in ("csrc", "host"):
        for ext in ("*.h", "*.hpp", "*.cuh"):
            hs += glob.glob(os.path.join(HERE, sub, ext))
    hs += glob.glob(os.path.join(ROOT, "include", "*.h"))
    hs += glob.glob(os.path.join(ROOT, "include", "welvet", "*.hpp"))
    hs += glob.glob(os.path.join(ROOT, "include", "welvet", "runtime", "*.hpp"))
    return hs


def _obj(src):
    rel = os.path.relpath(src, HERE).replace(os.sep, "_")
    return os.path.join(BUILD, rel + ".o")


def _compile(src, verbose=False):
    obj = _obj(src)
    cmd = [NVCC] + ARCH + COMMON + ["-c", src, "-o", obj]
    if src.endswith(".cu"):
        cmd += ["-Xptxas", "-v"] if verbose else []
    else:
        cmd += ["-x", "cu"]  # host files include CUDA headers; nvcc drives g++
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed on {src}:\n{r.stdout}\n{r.stderr}")
    return obj, r.stderr


def build(verbose: bool = False, jobs: int | None = None) -> str:
    os.makedirs(BUILD, exist_ok=True)
    os.makedirs(os.path.dirname(LIB), exist_ok=True)
    srcs = _sources()
    newest_header = max((os.path.getmtime(h) for h in _headers()), default=0)
    todo = [s for s in srcs if not os.path.exists(_obj(s))
            or os.path.getmtime(_obj(s)) < max(os.path.getmtime(s), newest_header)]
    if todo:
        with cf.ThreadPoolExecutor(max_workers=jobs or min(8, os.cpu_count() or 4)) as ex:
            for obj, log in ex.map(lambda s: _compile(s, verbose), todo):
                if verbose and log:
                    print(log, file=sys.stderr)
    objs = [_obj(s) for s in srcs]
    if todo or not os.path.exists(LIB) or os.path.getmtime(LIB) < max(os.path.getmtime(o) for o in objs):
        cmd = [NVCC] + ARCH + ["-shared", "-cudart", "static", "-o", LIB] + objs + ["-lpthread", "-ldl", "-lrt"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    if not os.path.exists(TOOL) or os.path.getmtime(TOOL) < max(os.path.getmtime(LIB), os.path.getmtime(TOOL_SRC),
                                                                newest_header):
        cmd = [os.environ.get("CXX", "g++"), "-std=c++17", "-O2", f"-I{os.path.join(ROOT, 'include')}", TOOL_SRC,
               "-o", TOOL, f"-L{os.path.dirname(LIB)}", "-lwelvet_b200", "-Wl,-rpath,$ORIGIN"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"tool build failed:\n{r.stdout}\n{r.stderr}")
    return LIB


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv))
