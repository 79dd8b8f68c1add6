"""Build the C-ABI shared library ``_lib/libbsattn_b200.so`` with nvcc.

    python -m blocksparsefa_reorder_b200.build [--force] [--verbose]

Every CUDA source under ``csrc/`` is compiled for sm_100a
(``-gencode arch=compute_100a,code=sm_100a -lineinfo -O3``) in parallel into
``_build/`` and linked into one shared library next to the package, so the
built file travels with the source tree.  Objects are rebuilt only when their
source or a header is newer.
"""

from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
INCLUDE = PKG.parent / "include"
BUILD_DIR = PKG / "_build"
LIB_DIR = PKG / "_lib"
LIB_PATH = LIB_DIR / "libbsattn_b200.so"
SOURCES = ["api.cu", "preprocess.cu", "attn_simt.cu", "tma_maps.cu", "attn_tcp.cu", "attn_bwd.cu",
           "plan_noalloc.cu"]
ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
CFLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
          "--expt-relaxed-constexpr"]


def _nvcc() -> str:
    for cand in (shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found; the CUDA toolkit is required to build the extension")


def _headers() -> list:
    return list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h")) + list(INCLUDE.glob("*.h"))


def up_to_date() -> bool:
    if not LIB_PATH.exists():
        return False
    t = LIB_PATH.stat().st_mtime
    return all(p.stat().st_mtime <= t for p in [*(CSRC / s for s in SOURCES), *_headers()])


def _obj_stale(src: Path, obj: Path) -> bool:
    if not obj.exists():
        return True
    t = obj.stat().st_mtime
    return any(p.stat().st_mtime > t for p in [src, *_headers()])


def build(force: bool = False, verbose: bool = False) -> Path:
    if not force and up_to_date():
        return LIB_PATH
    nvcc = _nvcc()
    BUILD_DIR.mkdir(exist_ok=True)
    LIB_DIR.mkdir(exist_ok=True)
    procs, objs = [], []
    for src in SOURCES:
        obj = BUILD_DIR / (Path(src).stem + ".o")
        objs.append(obj)
        if not force and not _obj_stale(CSRC / src, obj):
            continue
        cmd = [nvcc, *ARCH_FLAGS, *CFLAGS, "-I", str(INCLUDE), "-c", str(CSRC / src), "-o", str(obj)]
        if verbose:
            cmd.insert(1, "-Xptxas=-v")
            print(" ".join(cmd), flush=True)
        procs.append((src, subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True)))
    failed = []
    for src, p in procs:
        out, _ = p.communicate()
        if verbose and out:
            print(out)
        if p.returncode != 0:
            failed.append((src, out))
    if failed:
        raise RuntimeError("nvcc failed:\n" + "\n".join(f"--- {s}\n{o}" for s, o in failed))
    tmp = LIB_PATH.with_suffix(".so.tmp")
    r = subprocess.run([nvcc, *ARCH_FLAGS, "-shared", "-o", str(tmp), *map(str, objs)], capture_output=True,
                       text=True)
    if r.returncode != 0:
        raise RuntimeError(f"link failed:\n{r.stdout}{r.stderr}")
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    a = ap.parse_args(argv)
    print(build(force=a.force, verbose=a.verbose))
    return 0


if __name__ == "__main__":
    sys.exit(main())
