"""The C ABI from plain C: include/quantem_cuda_b200.h compiles as C11 and a C
program links against libquantem_cuda_b200.so and calls the entry points that
need no GPU (what a cgo or FFI binding would do first)."""

from __future__ import annotations

import shutil
import subprocess
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parents[1]
INCLUDE = REPO / "include"
PKG = REPO / "quantem-cuda_b200" / "quantem" / "cuda"
CUDA_INC = Path("/usr/local/cuda/include")

PROGRAM = r"""
#include <stdio.h>
#include <string.h>
#include "quantem_cuda_b200.h"

int main(void) {
    /* status strings and the compiled CUDA runtime version need no device */
    if (strlen(quantem_cuda_status_string(QC_ERR_INVALID_ARGUMENT)) == 0) return 2;
    if (quantem_cuda_cudart_version() < 12000) return 3;
    /* the fixed TV workspace size and the peer block sizes */
    size_t ws = tv_loss_3d_workspace_bytes(4, 256, 256, 256);
    if (ws == 0 || ws != tv_loss_3d_workspace_bytes(1, 2, 2, 2)) return 4;
    if (tv_peer_comm_bytes() == 0 || peer_allreduce_comm_bytes() == 0) return 5;
    /* argument checks run before any CUDA call */
    int st = kplanes_tilted_fuse_cuda(NULL, NULL, NULL, NULL, 16, 2, 8, 4, 4, (cudaStream_t)0);
    if (st != QC_ERR_INVALID_ARGUMENT) return 6;
    if (strlen(quantem_cuda_last_error()) == 0) return 7;
    printf("ok %zu\n", ws);
    return 0;
}
"""


@pytest.mark.skipif(shutil.which("gcc") is None, reason="needs gcc")
def test_header_is_c_and_the_library_links_from_c(tmp_path):
    lib = PKG / "libquantem_cuda_b200.so"
    if not lib.exists():
        pytest.skip("library not built")
    src = tmp_path / "abi.c"
    src.write_text(PROGRAM)
    exe = tmp_path / "abi"
    cmd = ["gcc", "-std=c11", "-Wall", "-Werror", f"-I{INCLUDE}", f"-I{CUDA_INC}", str(src), "-o", str(exe),
           f"-L{PKG}", "-lquantem_cuda_b200", f"-Wl,-rpath,{PKG}"]
    res = subprocess.run(cmd, capture_output=True, text=True)
    assert res.returncode == 0, res.stderr
    run = subprocess.run([str(exe)], capture_output=True, text=True, timeout=60)
    assert run.returncode == 0, (run.returncode, run.stdout, run.stderr)
    assert run.stdout.startswith("ok ")
