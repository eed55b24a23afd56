"""Build libb200attn.so (the C-ABI CUDA library) in-tree for sm_100a.

    python llm-inference_b200/build.py [--force] [--verbose]

Each CUDA translation unit under csrc/ is compiled by nvcc with
``-gencode arch=compute_100a,code=sm_100a`` into _build/, then linked with the
static CUDA runtime into b200attn/libb200attn.so. ptxas resource usage
(registers, spills, shared memory) is kept in _build/ptxas.log.

Freshness is decided by content, not file times: the SHA-256 of the sources,
headers, flags and nvcc version is written to libb200attn.so.sha256 after a
link, and a build whose hash differs (or has none) compiles again. build()
prints whether it compiled or reused the library.
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import hashlib
import os
import shutil
import subprocess
import sys

PKG_ROOT = os.path.dirname(os.path.abspath(__file__))
REPO_ROOT = os.path.dirname(PKG_ROOT)
CSRC = os.path.join(PKG_ROOT, "csrc")
BUILD = os.path.join(PKG_ROOT, "_build")
INCLUDE = os.path.join(REPO_ROOT, "include")
LIB = os.path.join(PKG_ROOT, "b200attn", "libb200attn.so")
# source hash of the linked library (written after a successful link)
STAMP = LIB + ".sha256"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-std=c++17", "-O3", "-lineinfo", *ARCH, "-Xcompiler", "-fPIC,-O3",
              "-Xptxas", "-v", f"-I{INCLUDE}", f"-I{CSRC}"]


def _nvcc() -> str:
    for cand in (shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found: the b200attn CUDA library cannot be built")


def sources() -> list[str]:
    return sorted(os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith(".cu"))


def _headers() -> list[str]:
    hs = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".h", ".cuh"))]
    hs += [os.path.join(INCLUDE, "b200attn.h")]
    return hs


def _compile(src: str, verbose: bool) -> tuple[str, str]:
    obj = os.path.join(BUILD, os.path.basename(src) + ".o")
    cmd = [_nvcc(), *NVCC_FLAGS, "-c", src, "-o", obj]
    if verbose:
        print(" ".join(cmd), flush=True)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed on {os.path.basename(src)}:\n{res.stdout}\n{res.stderr}")
    return obj, res.stderr


def _nvcc_version() -> str:
    res = subprocess.run([_nvcc(), "--version"], capture_output=True, text=True)
    return res.stdout.strip().splitlines()[-1] if res.returncode == 0 and res.stdout else "unknown"


def source_hash() -> str:
    """SHA-256 over every source and header (path and bytes), the compile and
    link flags, this script and the nvcc version: the identity of a build."""
    h = hashlib.sha256()
    for p in sorted(sources() + _headers() + [os.path.abspath(__file__)]):
        h.update(os.path.relpath(p, REPO_ROOT).encode())
        with open(p, "rb") as f:
            h.update(f.read())
    # flags with this checkout's paths made relative, so the same tree hashes
    # the same on every machine it is copied to
    h.update(" ".join(f.replace(REPO_ROOT, ".") for f in NVCC_FLAGS + ARCH).encode())
    h.update(_nvcc_version().encode())
    return h.hexdigest()


def built_hash() -> str | None:
    """The source hash recorded when the library in the tree was linked."""
    try:
        with open(STAMP) as f:
            return f.read().strip() or None
    except OSError:
        return None


def needs_build() -> bool:
    return not os.path.exists(LIB) or built_hash() != source_hash()


def build(force: bool = False, verbose: bool = False, quiet: bool = False) -> str:
    """Compile and link when the library is missing or its recorded source
    hash differs from the tree's; otherwise reuse it. Prints which (unless
    quiet), so a run on another machine shows whether it rebuilt."""
    want = source_hash()
    if not force and os.path.exists(LIB) and built_hash() == want:
        if not quiet:
            print(f"b200attn build: reused {os.path.relpath(LIB, REPO_ROOT)} (sources {want[:16]})", flush=True)
        return LIB
    os.makedirs(BUILD, exist_ok=True)
    srcs = sources()
    with cf.ThreadPoolExecutor(max_workers=min(8, len(srcs))) as ex:
        results = list(ex.map(lambda s: _compile(s, verbose), srcs))
    with open(os.path.join(BUILD, "ptxas.log"), "w") as f:
        for (obj, log), src in zip(results, srcs):
            f.write(f"== {os.path.basename(src)}\n{log}\n")
    tmp = LIB + f".tmp{os.getpid()}"
    cmd = [_nvcc(), "-shared", *ARCH, "-o", tmp, *[o for o, _ in results]]
    if verbose:
        print(" ".join(cmd), flush=True)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"link failed:\n{res.stdout}\n{res.stderr}")
    os.replace(tmp, LIB)
    stamp_tmp = STAMP + f".tmp{os.getpid()}"
    with open(stamp_tmp, "w") as f:
        f.write(want + "\n")
    os.replace(stamp_tmp, STAMP)
    if not quiet:
        print(f"b200attn build: compiled {os.path.relpath(LIB, REPO_ROOT)} (sources {want[:16]})", flush=True)
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    args = ap.parse_args()
    print(build(force=args.force, verbose=args.verbose))
    sys.exit(0)
