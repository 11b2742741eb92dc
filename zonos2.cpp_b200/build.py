"""Build recipe for the in-tree shared libraries (nvcc / g++, no torch extension machinery).

libz2b.so        the decode-step library: GGUF loader, tile repack, sm_100a kernels,
                 batch runtime and the C ABI declared in include/z2b.h; the DAC decoder
                 (include/z2b_dac.h).
libz2b_synth.so  host-only synthetic GGUF writer (include/z2b_tools.h).

Objects go to zonos2.cpp_b200/_build/ and are rebuilt when a source or header is newer.
"""
from __future__ import annotations

import concurrent.futures as cf
import os
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
BUILD = os.path.join(PKG, "_build")
INCLUDE = os.path.join(ROOT, "include")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]

LIB = os.path.join(PKG, "libz2b.so")
SYNTH_LIB = os.path.join(PKG, "libz2b_synth.so")

HOST_COMMON = ["gguf.cpp", "quant.cpp"]
Z2B_HOST = ["repack.cpp", "model.cpp", "runtime.cpp", "capi.cpp", "dac.cpp", "capi_dac.cpp", "prompt.cpp"]
Z2B_CUDA = ["k_gemv.cu", "k_gemm.cu", "k_attn.cu", "k_router.cu", "k_misc.cu", "k_test.cu", "k_dac.cu"]


def _headers():
    hs = []
    for d in (CSRC, INCLUDE):
        for f in os.listdir(d):
            if f.endswith((".h", ".cuh", ".hpp")):
                hs.append(os.path.join(d, f))
    return hs


def _stale(out, srcs):
    if not os.path.exists(out):
        return True
    t = os.path.getmtime(out)
    return any(os.path.getmtime(s) > t for s in srcs)


def _run(cmd):
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError("build failed:\n" + " ".join(cmd) + "\n" + r.stdout + r.stderr)
    return r.stdout + r.stderr


def _obj(src, kind, verbose=False):
    os.makedirs(BUILD, exist_ok=True)
    path = os.path.join(CSRC, src)
    out = os.path.join(BUILD, src + ".o")
    if not _stale(out, [path] + _headers()):
        return out, ""
    inc = ["-I" + CSRC, "-I" + INCLUDE]
    if kind == "cuda":
        cmd = [NVCC, *ARCH, "-O3", "-lineinfo", "-std=c++17", "--expt-relaxed-constexpr",
               "-Xcompiler", "-fPIC", "-Xcompiler", "-ffp-contract=off", *inc, "-c", path, "-o", out]
        if verbose:
            cmd.insert(1, "-Xptxas=-v")
    else:
        cmd = ["g++", "-O2", "-std=c++17", "-fPIC", "-fopenmp", "-ffp-contract=off",
               "-I/usr/local/cuda/include", *inc, "-c", path, "-o", out]
    return out, _run(cmd)


def build_synth():
    srcs = ["synth.cpp"] + HOST_COMMON
    objs = [_obj(s, "host")[0] for s in srcs]
    if _stale(SYNTH_LIB, objs):
        _run(["g++", "-shared", "-fopenmp", "-o", SYNTH_LIB, *objs])
    return SYNTH_LIB


def build_z2b(verbose=False):
    jobs = [(s, "host") for s in HOST_COMMON + Z2B_HOST] + [(s, "cuda") for s in Z2B_CUDA]
    logs = []
    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as ex:
        futs = [ex.submit(_obj, s, k, verbose) for s, k in jobs]
        objs = []
        for f in futs:
            o, log = f.result()
            objs.append(o)
            logs.append(log)
    if _stale(LIB, objs):
        _run([NVCC, *ARCH, "-shared", "-Xcompiler", "-fopenmp", "-o", LIB, *objs, "-lcuda"])
    if verbose:
        print("".join(logs))
    return LIB


def build_all(verbose=False):
    build_synth()
    build_z2b(verbose)


if __name__ == "__main__":
    which = sys.argv[1] if len(sys.argv) > 1 else "all"
    v = "-v" in sys.argv
    {"synth": build_synth, "z2b": lambda: build_z2b(v), "all": lambda: build_all(v)}[which]()
    print("ok")
