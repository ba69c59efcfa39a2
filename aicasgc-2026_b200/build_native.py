"""Build recipe of `libaicas_decode.so` (in-tree, sm_100a only).

    python aicasgc-2026_b200/build_native.py

nvcc cross-compiles without a GPU.  The CUDA runtime is linked statically so
the library has no dependency on which libcudart the host process loaded.
"""
from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
REPO = HERE.parent
SOURCES = [HERE / "csrc" / "decode_program.cu", HERE / "csrc" / "decode_batch.cu", HERE / "csrc" / "small_ops.cu",
           HERE / "csrc" / "op_kernels.cu", HERE / "csrc" / "prefill_kernels.cu", HERE / "csrc" / "attn_op.cu",
           HERE / "csrc" / "prefill_attn_tc.cu"]
HEADERS = [REPO / "include" / "aicas_decode.h", REPO / "include" / "aicas_phase_program.h",
           HERE / "csrc" / "aicas_device.cuh"]
OUT = HERE / "libaicas_decode.so"

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-lineinfo", "-O3", "-std=c++17",
    "-Xcompiler", "-fPIC,-fvisibility=hidden",
    "-shared", "-cudart", "static",
]


def nvcc_path() -> str:
    cand = Path(os.environ.get("CUDA_HOME", "/usr/local/cuda")) / "bin" / "nvcc"
    return str(cand) if cand.exists() else "nvcc"


def up_to_date() -> bool:
    if not OUT.exists():
        return False
    t = OUT.stat().st_mtime
    return all(p.stat().st_mtime <= t for p in SOURCES + HEADERS)


def build(force: bool = False, verbose: bool = False) -> Path:
    if not force and up_to_date():
        return OUT
    cmd = [nvcc_path(), *NVCC_FLAGS, f"-I{REPO / 'include'}", "-o", str(OUT), *map(str, SOURCES)]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
        print(" ".join(cmd))
    tmp = OUT.with_suffix(".so.tmp")
    cmd[cmd.index(str(OUT))] = str(tmp)
    subprocess.run(cmd, check=True)
    os.replace(tmp, OUT)
    return OUT


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
