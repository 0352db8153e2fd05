"""Build the sm_100a shared library in-tree with nvcc.

``python -m kvboost_b200._build`` (or ``__graft_entry__.build()``) compiles
``kvboost_b200/csrc/*.cu`` into ``kvboost_b200/_kvb_attn.so`` for
``compute_100a/sm_100a`` only.  The library exports the C ABI declared in
``include/kvb_attn.h``; nothing here depends on torch.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG_DIR)
CSRC = os.path.join(PKG_DIR, "csrc")
INCLUDE = os.path.join(ROOT, "include")
LIB_NAME = "_kvb_attn.so"
LIB_PATH = os.path.join(PKG_DIR, LIB_NAME)
SOURCES = ["kvb_prefill_sm100.cu", "kvb_noalloc_sm100.cu", "kvb_kvstore_sm100.cu",
           "kvb_peer_sm100.cu"]

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-lineinfo", "-O3", "-std=c++17",
    "-Xcompiler", "-fPIC", "-shared",
    "-Xptxas", "-v",
]


def nvcc_path() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found; set NVCC or install the CUDA toolkit")


def sources():
    return [os.path.join(CSRC, s) for s in SOURCES]


def needs_build() -> bool:
    if not os.path.exists(LIB_PATH):
        return True
    t = os.path.getmtime(LIB_PATH)
    deps = sources() + [os.path.join(CSRC, f) for f in os.listdir(CSRC)] + \
        [os.path.join(INCLUDE, f) for f in os.listdir(INCLUDE)]
    return any(os.path.getmtime(d) > t for d in deps)


def build(force: bool = False, verbose: bool = True) -> str:
    if not force and not needs_build():
        return LIB_PATH
    tmp = LIB_PATH + ".tmp"
    cmd = [nvcc_path(), *NVCC_FLAGS, "-I", INCLUDE, "-I", CSRC, "-o", tmp, *sources()]
    if verbose:
        print(" ".join(cmd), file=sys.stderr)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError("nvcc failed:\n" + res.stdout + res.stderr)
    if verbose:
        lines = [l for l in (res.stdout + res.stderr).splitlines()
                 if "registers" in l or "spill" in l or "error" in l]
        print("\n".join(lines), file=sys.stderr)
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


def build_traced(out_path: str) -> str:
    """A copy of the library with the kernels' phase timestamps compiled in
    (``-DKVB_TRACE``; clock64 and global-timer stamps per CTA into a buffer set with
    ``kvb_debug_set_trace``), for pipeline studies only (``kvboost_b200._trace``)."""
    flags = [f for f in NVCC_FLAGS if f not in ("-Xptxas", "-v")]
    cmd = [nvcc_path(), *flags, "-DKVB_TRACE", "-I", INCLUDE, "-I", CSRC, "-o", out_path,
           *sources()]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError("nvcc failed:\n" + res.stdout + res.stderr)
    return out_path


if __name__ == "__main__":
    build(force="--force" in sys.argv)
    print(LIB_PATH)
