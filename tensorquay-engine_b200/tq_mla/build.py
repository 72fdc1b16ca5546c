"""Build libtq_mla.so in-tree with nvcc for sm_100a (run: ``python -m tq_mla.build``)."""

import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG.parent / "csrc"
SOURCES = ["tq_mla_kernels.cu", "tq_kv_write.cu", "tq_prologue.cu", "tq_proj.cu", "tq_peer_merge.cu",
           "tq_contracts.cpp", "tq_comm.cpp"]
HEADERS = ["tq_ptx.cuh", "tq_mla_layout.h", "tq_contracts.h"]
TARGET = PKG / "libtq_mla.so"
NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-Xcompiler", "-fPIC,-O3",
    "-shared",
]


def nvcc():
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found")


def up_to_date():
    if not TARGET.exists():
        return False
    built = TARGET.stat().st_mtime
    deps = [CSRC / s for s in SOURCES + HEADERS] + [PKG.parent.parent / "include" / "tq_mla.h"]
    return all(d.stat().st_mtime <= built for d in deps)


BENCH = PKG / "tq_bench"
BENCH_SOURCE = CSRC / "tq_bench.cpp"


def build_bench(force=False):
    """The native benchmark binary: links libtq_mla.so (found next to it) and the CUDA runtime."""
    deps = [BENCH_SOURCE, PKG.parent.parent / "include" / "tq_mla.h", TARGET]
    if not force and BENCH.exists() and all(d.stat().st_mtime <= BENCH.stat().st_mtime
                                            for d in deps):
        return BENCH
    cmd = [nvcc(), "-O2", "-std=c++17", "-Wno-deprecated-gpu-targets", "-Xcompiler", "-O2", "-o",
           str(BENCH), str(BENCH_SOURCE),
           f"-L{PKG}", "-ltq_mla", "-Xlinker", "-rpath,$ORIGIN"]
    subprocess.run(cmd, check=True)
    return BENCH


def build(force=False, verbose=False):
    if force or not up_to_date():
        cmd = [nvcc(), *NVCC_FLAGS, "-o", str(TARGET), *[str(CSRC / s) for s in SOURCES], "-ldl"]
        if verbose:
            cmd.insert(1, "-Xptxas=-v")
            print(" ".join(cmd))
        subprocess.run(cmd, check=True)
    build_bench(force=force)
    return TARGET


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
