"""Builds the sm_100a kernels in place.

Outputs (next to the Python package, so they travel with the source tree):

* ``quantem/cuda/libquantem_cuda_b200.so`` — the C-ABI library declared in
  ``include/quantem_cuda_b200.h`` (CUDA runtime linked statically, no libtorch);
* ``quantem/cuda/_core<ext-suffix>`` — the pybind11 binding used by the torch
  op layer, linked against the library above through ``$ORIGIN``.

Run ``python build_ext.py`` (or ``__graft_entry__.build()``). Objects are
rebuilt only when a source or header is newer than its output.
"""

from __future__ import annotations

import os
import subprocess
import sys
import sysconfig
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

HERE = Path(__file__).resolve().parent
REPO = HERE.parent
CSRC = HERE / "csrc"
INCLUDE = REPO / "include"
PKG = HERE / "quantem" / "cuda"
OBJ = HERE / "_build"

CUDA_HOME = Path(os.environ.get("CUDA_HOME", "/usr/local/cuda"))
NVCC = str(CUDA_HOME / "bin" / "nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    "-O3",
    "-std=c++17",
    "-lineinfo",
    "-Xcompiler",
    "-fPIC",
    "-Xptxas",
    "-v",
    *ARCH,
    f"-I{INCLUDE}",
    f"-I{CSRC}",
]

CU_SOURCES = ["status.cu", "tv_sweep.cu", "kplanes_tilted.cu", "kplanes_probe.cu", "peer_mem.cu", "peer_reduce.cu"]
HEADERS = [INCLUDE / "quantem_cuda_b200.h", CSRC / "qc_common.cuh"]

LIB = PKG / "libquantem_cuda_b200.so"
# The same library with every computed global index checked against its buffer
# (QC_DEBUG_BOUNDS): out-of-range accesses are skipped and reported in the
# device fault word. A sanitizer substitute for debugging, never loaded by the
# torch ops.
DEBUG_LIB = PKG / "libquantem_cuda_b200_debug.so"
OBJ_DEBUG = HERE / "_build_debug"
CORE = PKG / ("_core" + sysconfig.get_config_var("EXT_SUFFIX"))


def _stale(out: Path, deps: list[Path]) -> bool:
    if not out.exists():
        return True
    t = out.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def _run(cmd: list[str], log: Path | None = None) -> None:
    res = subprocess.run(cmd, capture_output=True, text=True)
    if log is not None:
        log.write_text(res.stdout + res.stderr)
    if res.returncode != 0:
        sys.stderr.write(res.stdout + res.stderr)
        raise RuntimeError(f"build step failed: {' '.join(cmd[:3])} ... (exit {res.returncode})")


def _compile_cu(name: str, debug: bool = False) -> Path:
    src = CSRC / name
    out_dir = OBJ_DEBUG if debug else OBJ
    obj = out_dir / (Path(name).stem + ".o")
    if _stale(obj, [src, *HEADERS]):
        flags = [*NVCC_FLAGS, "-DQC_DEBUG_BOUNDS"] if debug else NVCC_FLAGS
        _run([NVCC, *flags, "-c", str(src), "-o", str(obj)], out_dir / (Path(name).stem + ".ptxas.txt"))
    return obj


def build_debug(verbose: bool = False) -> Path:
    """Builds the bounds-checked library (libquantem_cuda_b200_debug.so)."""
    OBJ_DEBUG.mkdir(exist_ok=True)
    with ThreadPoolExecutor(max_workers=len(CU_SOURCES)) as ex:
        objs = list(ex.map(lambda n: _compile_cu(n, debug=True), CU_SOURCES))
    if _stale(DEBUG_LIB, objs):
        _run([NVCC, *ARCH, "-shared", "-o", str(DEBUG_LIB), *map(str, objs)])
    if verbose:
        print(f"built {DEBUG_LIB.name} in {PKG}")
    return DEBUG_LIB


def build(verbose: bool = False) -> tuple[Path, Path]:
    OBJ.mkdir(exist_ok=True)
    with ThreadPoolExecutor(max_workers=len(CU_SOURCES)) as ex:
        objs = list(ex.map(_compile_cu, CU_SOURCES))
    if _stale(LIB, objs):
        _run([NVCC, *ARCH, "-shared", "-o", str(LIB), *map(str, objs)])
    core_src = CSRC / "pybind_core.cpp"
    if _stale(CORE, [core_src, LIB, *HEADERS]):
        import pybind11

        py_inc = sysconfig.get_paths()["include"]
        _run(
            [
                "g++",
                "-O2",
                "-std=c++17",
                "-shared",
                "-fPIC",
                "-fvisibility=hidden",
                f"-I{INCLUDE}",
                f"-I{CUDA_HOME / 'include'}",
                f"-I{pybind11.get_include()}",
                f"-I{py_inc}",
                str(core_src),
                "-o",
                str(CORE),
                f"-L{PKG}",
                "-lquantem_cuda_b200",
                "-Wl,-rpath,$ORIGIN",
            ]
        )
    if verbose:
        print(f"built {LIB.name} and {CORE.name} in {PKG}")
    return LIB, CORE


if __name__ == "__main__":
    build(verbose=True)
    if "--debug-bounds" in sys.argv:
        build_debug(verbose=True)
