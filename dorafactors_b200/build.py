"""Build libdora_b200.so in-tree with nvcc for sm_100a.

The library is a plain C-ABI shared object (no PyTorch headers or types), so it
is compiled with nvcc directly: each .cu file to an object with relocatable
device code, then one device link and a shared link.  The CUDA runtime is
linked statically; the driver API entry point used for TMA descriptors is
resolved at run time through cudaGetDriverEntryPoint, so no -lcuda is needed.

    python -m dorafactors_b200.build [--force] [--verbose]
"""

from __future__ import annotations

import argparse
import hashlib
import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
BUILD = os.path.join(PKG, "_build")
LIB = os.path.join(PKG, "libdora_b200.so")
SOURCES = ["capi.cu", "compose.cu", "compose_ch.cu", "backward.cu", "norm_simt.cu", "norm_tc.cu", "norm_tc2.cu", "norm_sk.cu", "norm_sk2.cu", "norm.cu", "shard.cu", "peer.cu", "selftest.cu"]
HEADERS = ["dora_common.cuh", "norm_internal.cuh", "tc_common.cuh"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-rdc=true", "--expt-relaxed-constexpr"]


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found: the DoRA sm_100a library cannot be built")


def _fingerprint() -> str:
    h = hashlib.sha256()
    for f in SOURCES + HEADERS:
        with open(os.path.join(CSRC, f), "rb") as fh:
            h.update(f.encode() + b"\0" + fh.read())
    with open(os.path.join(ROOT, "include", "dora_b200.h"), "rb") as fh:
        h.update(fh.read())
    h.update(" ".join(ARCH + FLAGS).encode())
    return h.hexdigest()


def build(force: bool = False, verbose: bool = False, ptxas_verbose: bool = False) -> str:
    """Compile the library if its sources changed; return the .so path."""
    stamp = os.path.join(BUILD, "fingerprint")
    fp = _fingerprint()
    if not force and os.path.exists(LIB) and os.path.exists(stamp):
        with open(stamp) as f:
            if f.read().strip() == fp:
                return LIB
    os.makedirs(BUILD, exist_ok=True)
    nvcc = _nvcc()
    objs = []
    extra = ["-Xptxas", "-v"] if ptxas_verbose else []
    for src in SOURCES:
        obj = os.path.join(BUILD, src.replace(".cu", ".o"))
        cmd = [nvcc, *ARCH, *FLAGS, *extra, "-c", os.path.join(CSRC, src), "-o", obj]
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
        objs.append(obj)
    dlink = os.path.join(BUILD, "dlink.o")
    cmd = [nvcc, *ARCH, "-Xcompiler", "-fPIC", "-dlink", *objs, "-o", dlink]
    subprocess.run(cmd, check=True)
    tmp = LIB + ".tmp"
    cmd = [nvcc, *ARCH, "-shared", "-Xcompiler", "-fPIC", *objs, dlink, "-o", tmp, "-cudart", "static"]
    if verbose:
        print(" ".join(cmd), flush=True)
    subprocess.run(cmd, check=True)
    os.replace(tmp, LIB)
    with open(stamp, "w") as f:
        f.write(fp)
    return LIB


def main(argv=None) -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--ptxas-verbose", action="store_true", help="print registers / spills / smem per kernel")
    a = ap.parse_args(argv)
    print(build(force=a.force, verbose=a.verbose, ptxas_verbose=a.ptxas_verbose))


if __name__ == "__main__":
    main(sys.argv[1:])
