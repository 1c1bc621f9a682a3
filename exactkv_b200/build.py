"""Builds libexactkv_b200.so (sm_100a) in-tree with nvcc.

    python exactkv_b200/build.py            # compile if a source is newer than the library
    python exactkv_b200/build.py --force    # always recompile
    python exactkv_b200/build.py --ptxas-v  # also print ptxas register/spill/smem report

Run it as a script (or through __graft_entry__.build()): importing the
exactkv_b200 package loads the library, so the package cannot build itself.
"""
import argparse
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
LIB = os.path.join(HERE, "libexactkv_b200.so")
SOURCES = ["exk_host.cu", "exk_attention.cu", "exk_codec.cu", "exk_noalloc.cu"]
HEADERS = ["exk_device.cuh", "exk_host.h", os.path.join("..", "..", "include", "exactkv_b200.h")]

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-Xcompiler", "-fPIC", "-shared",
    "--expt-relaxed-constexpr",
]


def _nvcc():
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", "nvcc"):
        if cand and (os.path.sep not in cand or os.path.exists(cand)):
            return cand
    raise RuntimeError("nvcc not found")


def sources():
    return [os.path.join(CSRC, s) for s in SOURCES if os.path.exists(os.path.join(CSRC, s))]


def stale():
    if not os.path.exists(LIB):
        return True
    t = os.path.getmtime(LIB)
    deps = sources() + [os.path.join(CSRC, h) for h in HEADERS]
    return any(os.path.getmtime(d) > t for d in deps if os.path.exists(d))


def build(force=False, ptxas_verbose=False, quiet=False):
    """Compile every CUDA source into one shared library next to this file."""
    if not force and not stale():
        return LIB
    cmd = [_nvcc(), *NVCC_FLAGS]
    if ptxas_verbose:
        cmd += ["-Xptxas", "-v"]
    cmd += ["-o", LIB + ".tmp", *sources(), "-lcudart_static", "-ldl", "-lpthread", "-lrt"]
    if not quiet:
        print(" ".join(cmd), flush=True)
    subprocess.run(cmd, check=True, cwd=ROOT)
    os.replace(LIB + ".tmp", LIB)
    return LIB


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--ptxas-v", action="store_true")
    a = ap.parse_args(argv)
    build(force=a.force or a.ptxas_v, ptxas_verbose=a.ptxas_v)
    return 0


if __name__ == "__main__":
    sys.exit(main())
