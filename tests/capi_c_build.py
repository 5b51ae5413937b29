"""Compile tests/c/layer_check.c (the attention layer driven from C through the
C ABI) against the in-tree library and the CUDA runtime.  Shared by the CPU
test (it builds and links) and the GPU test (it runs and passes)."""

import shutil
import subprocess
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent
SRC = ROOT / "tests" / "c" / "layer_check.c"
LIBDIR = ROOT / "tiktok_techjam_2026_track3_b200"
CUDA = Path("/usr/local/cuda")


def toolchain_available() -> bool:
    return (shutil.which("gcc") is not None and (CUDA / "include" / "cuda_runtime_api.h").exists()
            and (LIBDIR / "libttj_attn_sm100.so").exists())


def build(out_dir: Path) -> Path:
    exe = out_dir / "layer_check"
    cmd = ["gcc", "-std=c11", "-O2", "-Wall", "-Wextra", "-Werror",
           f"-I{ROOT / 'include'}", f"-I{CUDA / 'include'}", str(SRC), "-o", str(exe),
           f"-L{LIBDIR}", "-lttj_attn_sm100", f"-L{CUDA / 'lib64'}", "-lcudart", "-lm",
           f"-Wl,-rpath,{LIBDIR}:{CUDA / 'lib64'}"]
    subprocess.run(cmd, check=True)
    return exe
