"""Build recipe for libleafq.so (sm_100a), in-tree.

    python -m leaf_b200.build

compiles every CUDA source under leaf_b200/csrc into leaf_b200/libleafq.so
with nvcc for sm_100a only.  The library is built in place so that it ships
with the repository snapshot; nothing is installed into site-packages.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PACKAGE = Path(__file__).resolve().parent
CSRC = PACKAGE / "csrc"
LIBRARY = PACKAGE / "libleafq.so"
SOURCES = ["act_quant.cu", "gemv_w8a8.cu", "gemv_w4a32.cu", "linear_generic.cu", "gemm_tc.cu",
           "gemm_grouped_tc.cu", "graph_gemm.cu", "api.cu", "static_scratch.cu", "decode_persistent.cu",
           "peer_allgather.cu", "decoder_ops.cu", "decode_model.cu"]
GENCODE = "arch=compute_100a,code=sm_100a"


def nvcc() -> str:
    for candidate in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if candidate and Path(candidate).exists():
            return candidate
    raise RuntimeError("nvcc not found: libleafq.so cannot be built")


def command(output: Path = LIBRARY) -> list[str]:
    return [nvcc(), "-O3", "-std=c++17", "-gencode", GENCODE, "-lineinfo", "-rdc=true",
            "-Xcompiler", "-fPIC", "-shared", "-o", str(output),
            *(str(CSRC / name) for name in SOURCES)]


def stale(output: Path = LIBRARY) -> bool:
    if not output.exists():
        return True
    built = output.stat().st_mtime
    inputs = [CSRC / name for name in SOURCES] + list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h"))
    inputs.append(PACKAGE.parent / "include" / "leafq.h")
    return any(path.stat().st_mtime > built for path in inputs)


def build(force: bool = False) -> Path:
    if force or stale():
        tmp = LIBRARY.with_suffix(".so.partial")
        subprocess.run(command(tmp), check=True, cwd=CSRC)
        tmp.replace(LIBRARY)
    return LIBRARY


if __name__ == "__main__":
    build(force="--force" in sys.argv)
    print(LIBRARY)
