"""Build recipe for the in-tree shared libraries.

    python -m tinytrain_b200.build            # libttk.so + libtinytrain.so
    python -m tinytrain_b200.build --oracle --reference DIR   # + oracle/_ref (the checker)

Outputs (git-ignored, shipped with the tree):
  tinytrain_b200/lib/libttk.so        CUDA kernels + runtime, C ABI (include/ttk.h)
  tinytrain_b200/lib/libtinytrain.so  C++20 tt:: Tensor/ops/nn/optim/model API and
                                      the trainer C ABI (include/tt_trainer.h),
                                      linked against libttk.so
Every .cu file is compiled for sm_100a only.
"""
from __future__ import annotations

import argparse
import glob
import hashlib
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "tinytrain_b200")
CSRC = os.path.join(PKG, "csrc")
HOST = os.path.join(PKG, "host")
LIBDIR = os.path.join(PKG, "lib")
BUILD = os.path.join(ROOT, "_build")
INCLUDE = os.path.join(ROOT, "include")
CUDA_HOME = os.environ.get("CUDA_HOME", "/usr/local/cuda")
NVCC = os.path.join(CUDA_HOME, "bin", "nvcc")
HOSTCXX = "/usr/bin/g++" if os.path.exists("/usr/bin/g++") else "g++"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def _run(cmd, verbose):
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        sys.stderr.write(r.stdout + r.stderr)
        raise RuntimeError(f"build failed: {' '.join(cmd[:3])} ...")
    return r.stdout + r.stderr


def _stamp(paths, extra=""):
    h = hashlib.sha256(extra.encode())
    for p in sorted(paths):
        with open(p, "rb") as f:
            h.update(p.encode())
            h.update(f.read())
    return h.hexdigest()


def _up_to_date(out, stamp):
    sf = out + ".stamp"
    return os.path.exists(out) and os.path.exists(sf) and open(sf).read() == stamp


def _write_stamp(out, stamp):
    with open(out + ".stamp", "w") as f:
        f.write(stamp)


def build_ttk(verbose=False, force=False, jobs=8):
    os.makedirs(LIBDIR, exist_ok=True)
    os.makedirs(BUILD, exist_ok=True)
    srcs = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    deps = srcs + glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(CSRC, "*.h")) + \
        [os.path.join(INCLUDE, "ttk.h")]
    out = os.path.join(LIBDIR, "libttk.so")
    flags = ["-std=c++17", "-O3", "-lineinfo", "-rdc=true", "-Xcompiler", "-fPIC", "-ccbin", HOSTCXX,
             "-I" + INCLUDE, "-I" + CSRC] + ARCH
    stamp = _stamp(deps, " ".join(flags))
    if not force and _up_to_date(out, stamp):
        return out
    objs = []
    procs = []
    for s in srcs:
        o = os.path.join(BUILD, os.path.basename(s) + ".o")
        objs.append(o)
        cmd = [NVCC] + flags + ["-c", s, "-o", o]
        if verbose:
            print(" ".join(cmd), flush=True)
        procs.append((cmd, subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT,
                                            text=True)))
        if len(procs) >= jobs:
            _drain(procs)
    _drain(procs)
    _run([NVCC, "-shared", "-rdc=true", "-ccbin", HOSTCXX] + ARCH + objs +
         ["-o", out, "-lcudart_static", "-ldl", "-lpthread", "-lrt"], verbose)
    _write_stamp(out, stamp)
    return out


def _drain(procs):
    while procs:
        cmd, p = procs.pop(0)
        outp, _ = p.communicate()
        if p.returncode != 0:
            sys.stderr.write(outp)
            raise RuntimeError(f"nvcc failed on {cmd[-3]}")


def build_host(verbose=False, force=False):
    srcs = sorted(glob.glob(os.path.join(HOST, "*.cpp")))
    if not srcs:
        return None
    hdrs = glob.glob(os.path.join(INCLUDE, "**", "*.h"), recursive=True) + \
        glob.glob(os.path.join(HOST, "*.h"))
    out = os.path.join(LIBDIR, "libtinytrain.so")
    flags = ["-std=c++20", "-O2", "-fPIC", "-march=x86-64-v3", "-I" + INCLUDE, "-I" + HOST]
    stamp = _stamp(srcs + hdrs + [os.path.join(LIBDIR, "libttk.so")], " ".join(flags))
    if not force and _up_to_date(out, stamp):
        return out
    _run([HOSTCXX] + flags + ["-shared", "-o", out] + srcs +
         ["-L" + LIBDIR, "-lttk", "-Wl,-rpath,$ORIGIN", "-lpthread"], verbose)
    _write_stamp(out, stamp)
    return out


def build_oracle(verbose=False, ref=None):
    """Builds the checker (oracle/_ref) from the reference sources at `ref`
    (or $TT_REFERENCE); does nothing when neither names the sources."""
    ref = ref or os.environ.get("TT_REFERENCE")
    if not ref or not os.path.isdir(os.path.join(ref, "src")):
        return None
    _run(["make", "-s", "-C", os.path.join(ROOT, "oracle"), f"REF={ref}"], verbose)
    return os.path.join(ROOT, "oracle", "_ref", "libttref.so")


def build_all(verbose=False, force=False, oracle=True, ref=None):
    build_ttk(verbose, force)
    build_host(verbose, force)
    if oracle:
        build_oracle(verbose, ref)


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--oracle", action="store_true")
    ap.add_argument("--reference", default=None,
                    help="reference source directory for --oracle (default $TT_REFERENCE)")
    ap.add_argument("-v", "--verbose", action="store_true")
    a = ap.parse_args()
    build_all(a.verbose, a.force, a.oracle, a.reference)
    print("built:", LIBDIR)
