"""B200-native (sm_100a) kernels for quantem's data-parallel hot path.

Drop-in for the reference package's hot path (quantem-cuda,
src/quantem/cuda/__init__.py): the same import path ``quantem.cuda``, the same
public functions and the same ``torch.library`` ops (``quantem_cuda::*``),
backed by hand-written CUDA for sm_100a behind a torch-free C ABI
(``include/quantem_cuda_b200.h``).

Submodules:
    quantem.cuda.core       3-D total-variation losses (+ single-sweep fwd+grad)
    quantem.cuda.core.ml    fused tilted K-Planes interpolation
    quantem.cuda.sharded    multi-GPU forms (K-Planes point sharding, TV D-slabs)
"""

from importlib.metadata import PackageNotFoundError, version

from quantem.cuda import core as core
from quantem.cuda._common import cudart_version as cudart_version

try:  # the reference reads dist metadata unconditionally (cuda/__init__.py:23)
    __version__ = version("quantem-cuda")
except PackageNotFoundError:
    __version__ = "0.1.0+b200"
