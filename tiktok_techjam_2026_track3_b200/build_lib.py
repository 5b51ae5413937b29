"""Compile the sm_100a CUDA sources into the in-tree shared library.

    python -m tiktok_techjam_2026_track3_b200.build_lib [--verbose]

Produces ``tiktok_techjam_2026_track3_b200/libttj_attn_sm100.so`` with nvcc
directly (no torch extension machinery: the library's ABI is plain C, see
``include/ttj_attn.h``).  Each translation unit is compiled in parallel, then
linked; the CUDA runtime is linked statically so the library does not depend
on which libcudart the host process loaded first.
"""

from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
LIB_NAME = "libttj_attn_sm100.so"
LIB_PATH = PKG / LIB_NAME
BUILD_DIR = PKG.parent / "_build"

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON_FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC",
                "--expt-relaxed-constexpr", "-I", str(PKG.parent / "include")]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found; the CUDA toolkit is required to build the library")


def sources():
    return sorted(CSRC.glob("*.cu"))


def _needs_rebuild() -> bool:
    if not LIB_PATH.exists():
        return True
    t = LIB_PATH.stat().st_mtime
    deps = list(CSRC.glob("*")) + list((PKG.parent / "include").glob("*.h"))
    return any(p.stat().st_mtime > t for p in deps)


def build(force: bool = False, verbose: bool = False, ptxas_info: bool = False) -> Path:
    if not force and not _needs_rebuild():
        return LIB_PATH
    BUILD_DIR.mkdir(exist_ok=True)
    cc = nvcc()
    extra = ["-Xptxas", "-v"] if ptxas_info else []

    def compile_one(src: Path) -> Path:
        obj = BUILD_DIR / (src.stem + ".o")
        cmd = [cc, *ARCH_FLAGS, *COMMON_FLAGS, *extra, "-c", str(src), "-o", str(obj)]
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"nvcc failed on {src.name}:\n{res.stderr}")
        if verbose or ptxas_info:
            sys.stderr.write(res.stderr)
        return obj

    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as ex:
        objs = list(ex.map(compile_one, sources()))
    tmp = LIB_PATH.with_suffix(".so.tmp")
    cmd = [cc, *ARCH_FLAGS, "-shared", "-o", str(tmp), *map(str, objs)]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"link failed:\n{res.stderr}")
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--ptxas-info", action="store_true", help="print registers / spills / smem")
    args = ap.parse_args()
    print(build(force=args.force, verbose=args.verbose, ptxas_info=args.ptxas_info))
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
