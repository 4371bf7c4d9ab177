"""CUDA kernels accelerating quantem.core.ml (K-Planes models).
Mirrors the reference's src/quantem/cuda/core/ml/__init__.py for the hot path."""

from quantem.cuda.core.ml._ops import kplanes_tilted_fuse as kplanes_tilted_fuse
from quantem.cuda.core.ml._ops import kplanes_tilted_tv_fuse as kplanes_tilted_tv_fuse
from quantem.cuda.core.ml._ops import kplanes_tilted_fuse_levels as kplanes_tilted_fuse_levels
