"""vdit: B200-native (sm_100a) sparse-voxel DiT (lat_dit) forward path.

Drop-in for the reference's hot path behind its plugin contract:
``solution.Solution`` (``LatDitGenerator.from_pretrained`` / ``generate_impl``),
``fast_flow.OptimizedLatDitRunner`` and ``fast_sampler`` (exact subset).
The kernels live in ``libvdit.so`` (C ABI, ``include/vdit.h``).
"""
from . import _lib
from .fast_sampler import SolverConfig, build_schedule
from .model import LatDitArch, LatDitModel
from .runtime import FlowMatchSamplingParams, LatDitConditioning, LatDitGenerator, resolve

__all__ = ["_lib", "SolverConfig", "build_schedule", "LatDitArch", "LatDitModel", "FlowMatchSamplingParams",
           "LatDitConditioning", "LatDitGenerator", "resolve"]
