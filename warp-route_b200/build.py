"""Build the warp-route B200 native code in-tree (sm_100a only).

Outputs, next to the Python package so they travel with the source tree:
  warp_route/libwarp_route_b200.so   CUDA kernels + the C ABI (include/warp_route_b200.h)
  warp_route/_C.<abi>.so             torch binding over that C ABI (same names and
                                     signatures as warp-route's src/bindings.cpp)

Usage: python warp-route_b200/build.py [--force] [--jobs N] [--no-binding]
Rebuilds only what is out of date (source, header or flag changes).
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import hashlib
import os
import subprocess
import sys
import sysconfig

PKG_ROOT = os.path.dirname(os.path.abspath(__file__))
REPO_ROOT = os.path.dirname(PKG_ROOT)
CSRC = os.path.join(PKG_ROOT, "csrc")
OUT_DIR = os.path.join(PKG_ROOT, "warp_route")
OBJ_DIR = os.path.join(PKG_ROOT, "_build")
INCLUDE = os.path.join(REPO_ROOT, "include")
LIB_NAME = "libwarp_route_b200.so"

NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC",
                     "-Xcompiler", "-fvisibility=hidden", "--expt-relaxed-constexpr",
                     "-I" + INCLUDE, "-I" + CSRC]
KERNEL_SOURCES = ["wr_api.cu", "wr_fused.cu", "wr_naive.cu", "wr_noalloc.cu", "wr_comm.cu",
                  "wr_grouped.cu", "wr_pack.cu"]
HEADERS = ["wr_common.cuh", "wr_router.cuh", "wr_internal.h"]


def _sig(paths, flags) -> str:
    h = hashlib.sha1(" ".join(flags).encode())
    for p in paths:
        with open(p, "rb") as f:
            h.update(f.read())
    return h.hexdigest()


def _stale(target: str, sig: str) -> bool:
    stamp = target + ".sig"
    if not os.path.exists(target) or not os.path.exists(stamp):
        return True
    with open(stamp) as f:
        return f.read().strip() != sig


def _stamp(target: str, sig: str) -> None:
    with open(target + ".sig", "w") as f:
        f.write(sig)


def _run(cmd, verbose):
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        sys.stderr.write(r.stdout + r.stderr)
        raise RuntimeError(f"build step failed: {cmd[0]} ... {cmd[-1]}")
    if verbose and (r.stdout or r.stderr):
        sys.stdout.write(r.stdout + r.stderr)
    return r


def build_library(force=False, jobs=4, verbose=False, extra_flags=()) -> str:
    os.makedirs(OBJ_DIR, exist_ok=True)
    flags = NVCC_FLAGS + list(extra_flags)
    hdrs = [os.path.join(CSRC, h) for h in HEADERS] + [os.path.join(INCLUDE, "warp_route_b200.h")]
    objs, todo = [], []
    for src in KERNEL_SOURCES:
        sp = os.path.join(CSRC, src)
        obj = os.path.join(OBJ_DIR, src + ".o")
        sig = _sig([sp] + hdrs, flags)
        objs.append(obj)
        if force or _stale(obj, sig):
            todo.append((sp, obj, sig))

    def compile_one(item):
        sp, obj, sig = item
        _run([NVCC] + flags + ["-c", sp, "-o", obj], verbose)
        _stamp(obj, sig)

    with cf.ThreadPoolExecutor(max_workers=max(1, jobs)) as ex:
        list(ex.map(compile_one, todo))
    lib = os.path.join(OUT_DIR, LIB_NAME)
    lsig = _sig(objs, flags)
    if force or todo or _stale(lib, lsig):
        _run([NVCC] + ARCH + ["-shared", "-o", lib] + objs + ["-lcudart"], verbose)
        _stamp(lib, lsig)
    return lib


def build_binding(force=False, verbose=False) -> str:
    import torch
    from torch.utils import cpp_extension as ce

    src = os.path.join(CSRC, "wr_bindings.cpp")
    suffix = sysconfig.get_config_var("EXT_SUFFIX") or ".so"
    out = os.path.join(OUT_DIR, "_C" + suffix)
    inc = ce.include_paths(device_type="cuda") + [INCLUDE, sysconfig.get_paths()["include"]]
    libdirs = ce.library_paths(device_type="cuda")
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    flags = ["-O2", "-std=c++17", "-fPIC", "-shared", f"-D_GLIBCXX_USE_CXX11_ABI={abi}",
             "-DTORCH_EXTENSION_NAME=_C", "-DTORCH_API_INCLUDE_EXTENSION_H"]
    flags += ["-I" + p for p in inc]
    flags += ["-I/usr/local/cuda/include"]
    libs = ["-L" + p for p in libdirs] + ["-L" + OUT_DIR, "-L/usr/local/cuda/lib64"]
    libs += ["-Wl,-rpath,$ORIGIN"] + ["-Wl,-rpath," + p for p in libdirs]
    libs += ["-lwarp_route_b200", "-lc10", "-lc10_cuda", "-ltorch", "-ltorch_cpu", "-ltorch_cuda",
             "-ltorch_python", "-lcudart"]
    sig = _sig([src, os.path.join(INCLUDE, "warp_route_b200.h")], flags + libs)
    if force or _stale(out, sig):
        _run(["g++"] + flags + [src, "-o", out] + libs, verbose)
        _stamp(out, sig)
    return out


def build(force=False, jobs=4, verbose=False, binding=True):
    lib = build_library(force=force, jobs=jobs, verbose=verbose)
    outs = [lib]
    if binding:
        outs.append(build_binding(force=force, verbose=verbose))
    return outs


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--jobs", type=int, default=4)
    ap.add_argument("--no-binding", action="store_true")
    ap.add_argument("-v", "--verbose", action="store_true")
    a = ap.parse_args()
    for p in build(force=a.force, jobs=a.jobs, verbose=a.verbose, binding=not a.no_binding):
        print(p)


if __name__ == "__main__":
    main()
