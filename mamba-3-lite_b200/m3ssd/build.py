"""Build libm3ssd.so in-tree with nvcc for sm_100a.

    python mamba-3-lite_b200/m3ssd/build.py            # build if sources are newer
    python mamba-3-lite_b200/m3ssd/build.py --force
    python mamba-3-lite_b200/m3ssd/build.py --trace    # measurement build (m3ssd.trace)

The shared library is written next to this file (``m3ssd/libm3ssd.so``) so it travels with the
source tree; the CUDA runtime is linked statically so the library does not depend on which
libcudart the host process loaded first.
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
PKG_ROOT = os.path.dirname(PKG)
REPO = os.path.dirname(PKG_ROOT)
CSRC = os.path.join(PKG_ROOT, "csrc")
INCLUDE = os.path.join(REPO, "include")
BUILD_DIR = os.path.join(REPO, "_build")
LIB_NAME = "libm3ssd.so"
LIB_PATH = os.path.join(PKG, LIB_NAME)
# measurement build: the same sources with -DM3SSD_TRACE (per-phase clock stamps of the
# tensor-core kernels, read by m3ssd.trace); never loaded by the operator itself
TRACE_LIB_PATH = os.path.join(PKG, "libm3ssd_trace.so")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + ["-O3", "-lineinfo", "-std=c++17", "--expt-relaxed-constexpr",
                     "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
                     "-I", INCLUDE, "-I", CSRC]


def nvcc_path():
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def sources():
    return sorted(os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith(".cu"))


def headers():
    hs = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cuh", ".h"))]
    hs.append(os.path.join(INCLUDE, "m3ssd.h"))
    return hs


def _newest(paths):
    return max(os.path.getmtime(p) for p in paths)


def needs_build():
    if not os.path.exists(LIB_PATH):
        return True
    return _newest(sources() + headers() + [__file__]) > os.path.getmtime(LIB_PATH)


def _compile(nvcc, src, extra, build_dir):
    obj = os.path.join(build_dir, os.path.basename(src) + ".o")
    cmd = [nvcc, *NVCC_FLAGS, *extra, "-c", src, "-o", obj]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src}:\n{res.stdout}\n{res.stderr}")
    return obj, res.stderr


def build(force=False, verbose=False, extra_flags=(), trace=False):
    lib_path = TRACE_LIB_PATH if trace else LIB_PATH
    if not force and not trace and not needs_build():
        return LIB_PATH
    nvcc = nvcc_path()
    build_dir = os.path.join(BUILD_DIR, "trace") if trace else BUILD_DIR
    os.makedirs(build_dir, exist_ok=True)
    flags = list(extra_flags) + (["-DM3SSD_TRACE"] if trace else [])
    srcs = sources()
    with cf.ThreadPoolExecutor(max_workers=min(8, len(srcs))) as ex:
        outs = list(ex.map(lambda s: _compile(nvcc, s, flags, build_dir), srcs))
    if verbose:
        for _, err in outs:
            if err.strip():
                print(err, file=sys.stderr)
    tmp = lib_path + ".tmp"
    cmd = [nvcc, *ARCH, "-shared", "-o", tmp, *[o for o, _ in outs]]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"link failed:\n{res.stdout}\n{res.stderr}")
    os.replace(tmp, lib_path)
    return lib_path


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--ptxas-v", action="store_true", help="print register/smem usage")
    ap.add_argument("--trace", action="store_true",
                    help="build the measurement library libm3ssd_trace.so (-DM3SSD_TRACE)")
    args = ap.parse_args()
    extra = ["-Xptxas", "-v"] if args.ptxas_v else []
    print(build(force=args.force or args.ptxas_v, verbose=args.verbose or args.ptxas_v,
                extra_flags=extra, trace=args.trace))
