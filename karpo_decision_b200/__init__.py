"""B200-native (sm_100a) packed prefill forward of karpo-decision: hand-written CUDA kernels behind a C ABI
(libkd_b200.so, include/kd_b200.h), with a drop-in ``Packed`` / ``Readout`` for the reference's
``family.Packed`` / ``model.readout.Readout``."""

from . import ops, profile
from .pack import Pack, from_arrays, pack
from .packed import Packed, Readout
from .synthetic import CONFIGS, Spec

__all__ = ["CONFIGS", "Pack", "Packed", "Readout", "Spec", "from_arrays", "ops", "pack", "profile"]
