"""Builds libhmb.so in-tree with nvcc for sm_100a (B200). No GPU needed: nvcc cross-compiles.

    python -m heteromega_b200.build [--verbose] [--ptxas-info] [--reference DIR]

Objects go to heteromega_b200/_build/, the library to heteromega_b200/libhmb.so. Sources
are compiled in parallel and only when they (or the headers) changed. With the reference
checkout given (--reference, or $HETEROMEGA_REF), the C++ drop-in of its FFN interface
(cpp/gpu_ffn_dropin.cpp -> libhmb_dropin.so) and its C++ self-test are built against the
reference's own headers as well.
"""
import argparse
import concurrent.futures as cf
import glob
import os
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
BUILD = os.path.join(PKG, "_build")
LIB = os.path.join(PKG, "libhmb.so")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-Xcompiler", "-O2", "--expt-relaxed-constexpr",
         "-I" + os.path.join(REPO, "include"), "-I" + CSRC]


def _sources():
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")))


def _headers():
    return sorted(glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(REPO, "include", "*.h")))


def _stale(target, deps):
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def _compile(src, ptxas_info, verbose):
    obj = os.path.join(BUILD, os.path.basename(src) + ".o")
    if not _stale(obj, [src] + _headers()):
        return obj, ""
    cmd = [NVCC] + ARCH + FLAGS + (["-Xptxas", "-v"] if ptxas_info else []) + ["-c", src, "-o", obj]
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed on {src}:\n{r.stdout}\n{r.stderr}")
    return obj, r.stderr


def build(verbose=False, ptxas_info=False, force=False):
    os.makedirs(BUILD, exist_ok=True)
    srcs = _sources()
    if force:
        for o in glob.glob(os.path.join(BUILD, "*.o")):
            os.remove(o)
    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as ex:
        results = list(ex.map(lambda s: _compile(s, ptxas_info, verbose), srcs))
    for _, log in results:
        if log and (ptxas_info or verbose):
            print(log)
    objs = [o for o, _ in results]
    if _stale(LIB, objs) or force:
        cmd = [NVCC] + ARCH + ["-shared", "-o", LIB] + objs
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
    return LIB


def build_dropin(reference):
    """libhmb_dropin.so and tests/cpp/_build/dropin_selftest, compiled against the reference's headers."""
    for folder in (os.path.join(PKG, "cpp"), os.path.join(REPO, "tests", "cpp")):
        subprocess.run(["make", "-s", "-C", folder, f"REF={reference}", f"PY={sys.executable}"], check=True)
    return os.path.join(PKG, "libhmb_dropin.so")


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--ptxas-info", action="store_true")
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--reference", default=os.environ.get("HETEROMEGA_REF", ""))
    args = ap.parse_args()
    print(build(args.verbose, args.ptxas_info, args.force))
    if args.reference:
        print(build_dropin(args.reference))
    sys.exit(0)
