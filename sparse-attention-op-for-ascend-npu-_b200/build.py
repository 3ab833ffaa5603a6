"""Build recipe for the in-tree native libraries.

* ``libtpsa.so``        the sm_100a kernel + C ABI (nvcc, static cudart)
* ``_tpsa_torch.so``    the PyTorch op adapter, linked against libtpsa.so

Both land next to this file so that they travel with the source tree.
Run ``python -m`` style: ``python sparse-attention-op-for-ascend-npu-_b200/build.py``.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
CSRC = PKG_DIR / "csrc"
INCLUDE = PKG_DIR.parent / "include"
LIB = PKG_DIR / "libtpsa.so"
ADAPTER = PKG_DIR / "_tpsa_torch.so"

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
]


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found")


def _cuda_home() -> Path:
    return Path(_nvcc()).resolve().parent.parent


def _newer(target: Path, sources: list[Path]) -> bool:
    return target.exists() and all(target.stat().st_mtime >= s.stat().st_mtime for s in sources)


def _run(cmd: list[str]) -> None:
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"build step failed ({' '.join(cmd[:3])} ...):\n{res.stdout}\n{res.stderr}")


# Spill limit in bytes of spill stores (see _check_ptxas_report).
MAX_SPILL_BYTES = 16


def _check_ptxas_report(text: str) -> None:
    """Every instantiation of tpsa_paged_kernel (<false, false> for
    batch-one calls, <false, true> for packed ragged batches, <true, false>
    recording visited keys) stays within MAX_SPILL_BYTES of local-memory
    spill stores.  The softmax keeps a whole 128-key row of scores in
    registers; the allocation stores 8 bytes to local memory, which measured
    faster than loading half of the row twice without any spill."""
    import re

    found = re.findall(r"Compiling entry function '\w*tpsa_paged_kernelILb([01])ELb([01])E\w*' "
                       r"for 'sm_100a'\n(?:.*\n)*?\s*(\d+) bytes stack frame, (\d+) bytes spill stores",
                       text)
    kinds = {visit + varlen: int(st) for visit, varlen, _, st in found}
    if set(kinds) != {"00", "01", "10"}:
        raise RuntimeError("could not read the ptxas report of tpsa_paged_kernel")
    for kind, spilled in kinds.items():
        if spilled > MAX_SPILL_BYTES:
            raise RuntimeError(f"tpsa_paged_kernel<{kind}> spills registers ({spilled} bytes)")


def build_lib(force: bool = False) -> Path:
    sources = [CSRC / "tpsa_kernel.cu", CSRC / "tpsa_schedule.h", CSRC / "sm100_ptx.cuh",
               INCLUDE / "tpsa.h"]
    if not force and _newer(LIB, sources):
        return LIB
    tmp = LIB.with_suffix(".so.tmp")
    cmd = [_nvcc(), *NVCC_FLAGS, "-Xptxas=-v", "-shared", "-o", str(tmp),
           str(CSRC / "tpsa_kernel.cu")]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed:\n{res.stdout}\n{res.stderr}")
    _check_ptxas_report(res.stdout + res.stderr)
    (PKG_DIR / "ptxas_report.txt").write_text(res.stdout + res.stderr)
    tmp.replace(LIB)
    return LIB


def build_adapter(force: bool = False) -> Path:
    import torch
    from torch.utils import cpp_extension

    sources = [CSRC / "torch_adapter.cpp", INCLUDE / "tpsa.h", LIB]
    if not force and _newer(ADAPTER, sources):
        return ADAPTER
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    incs = cpp_extension.include_paths() + [str(_cuda_home() / "include")]
    libdirs = cpp_extension.library_paths()
    tmp = ADAPTER.with_suffix(".so.tmp")
    cmd = ["g++", "-shared", "-fPIC", "-O2", "-std=c++17", f"-D_GLIBCXX_USE_CXX11_ABI={abi}",
           "-DTORCH_API_INCLUDE_EXTENSION_H", "-DTORCH_EXTENSION_NAME=_tpsa_torch",
           *[f"-I{i}" for i in incs], str(CSRC / "torch_adapter.cpp"), "-o", str(tmp),
           *[f"-L{d}" for d in libdirs], f"-L{PKG_DIR}", "-ltpsa", "-lc10", "-lc10_cuda",
           "-ltorch_cpu", "-ltorch_cuda", "-ltorch", "-Wl,-rpath,$ORIGIN",
           *[f"-Wl,-rpath,{d}" for d in libdirs]]
    _run(cmd)
    tmp.replace(ADAPTER)
    return ADAPTER


def build(force: bool = False) -> tuple[Path, Path]:
    lib = build_lib(force)
    adapter = build_adapter(force)
    return lib, adapter


if __name__ == "__main__":
    force = "--force" in sys.argv
    for p in build(force):
        print(p)
