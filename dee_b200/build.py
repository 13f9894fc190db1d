"""Build the in-tree CUDA library ``dee_b200/libdee_b200.so`` for sm_100a.

The library exports the C ABI declared in ``include/dee_b200.h``.  The CUDA
runtime is linked statically so the library loads (and exports its symbols)
on machines without a GPU driver; CUDA calls then fail with an error code.

    python -m dee_b200.build            # build if sources are newer
    python -m dee_b200.build --force    # rebuild
"""
from __future__ import annotations

import argparse
import glob
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
LIB = os.path.join(HERE, "libdee_b200.so")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def sources() -> list[str]:
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")) + glob.glob(os.path.join(CSRC, "*.cpp")))


def deps() -> list[str]:
    return sources() + sorted(glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(CSRC, "*.h"))) + [
        os.path.join(ROOT, "include", "dee_b200.h")]


def up_to_date() -> bool:
    if not os.path.exists(LIB):
        return False
    t = os.path.getmtime(LIB)
    return all(os.path.getmtime(p) <= t for p in deps())


def build(force: bool = False, verbose: bool = False, ptxas_info: bool = False) -> str:
    if not force and up_to_date():
        return LIB
    cmd = [nvcc(), *ARCH, "-O3", "-lineinfo", "-std=c++17", "--expt-relaxed-constexpr",
           "-Xcompiler", "-fPIC,-fvisibility=hidden", "-shared", "-cudart", "static",
           "-I", os.path.join(ROOT, "include"), "-o", LIB + ".tmp", *sources()]
    if ptxas_info:
        cmd.insert(1, "-Xptxas=-v")
    if verbose:
        print(" ".join(cmd), file=sys.stderr)
    subprocess.run(cmd, check=True)
    os.replace(LIB + ".tmp", LIB)
    return LIB


PYDEE_SRC = os.path.join(HERE, "pybind", "pydee.cpp")


def pydee_path() -> str:
    import sysconfig
    return os.path.join(HERE, "_pydee" + sysconfig.get_config_var("EXT_SUFFIX"))


def build_pydee(force: bool = False, verbose: bool = False) -> str:
    """The pybind11 module dee_b200._pydee (pydee.Engine's methods over the
    C ABI), linked against the in-tree libdee_b200.so through an $ORIGIN
    rpath.  Needs the library built first."""
    import sysconfig

    import pybind11
    out = pydee_path()
    srcs = [PYDEE_SRC, os.path.join(ROOT, "include", "dee_b200.h"), LIB]
    if not force and os.path.exists(out) and all(os.path.getmtime(p) <= os.path.getmtime(out) for p in srcs):
        return out
    cxx = os.environ.get("CXX") or shutil.which("g++") or "g++"
    cmd = [cxx, "-O2", "-std=c++17", "-shared", "-fPIC", "-fvisibility=hidden",
           "-I", pybind11.get_include(), "-I", sysconfig.get_paths()["include"], "-I", os.path.join(ROOT, "include"),
           "-o", out + ".tmp", PYDEE_SRC, "-L", HERE, "-l:libdee_b200.so", "-Wl,-rpath,$ORIGIN"]
    if verbose:
        print(" ".join(cmd), file=sys.stderr)
    subprocess.run(cmd, check=True)
    os.replace(out + ".tmp", out)
    return out


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--ptxas-info", action="store_true")
    args = ap.parse_args()
    print(build(force=args.force, verbose=True, ptxas_info=args.ptxas_info))
    print(build_pydee(force=args.force, verbose=True))


if __name__ == "__main__":
    main()
