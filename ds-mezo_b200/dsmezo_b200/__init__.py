"""B200-native (sm_100a) DS-MeZO optimizer hot path.

* ``dsmezo_b200.kernels`` - drop-in for the reference module ``ds_mezo.kernels``
  (zo_muon_update, fused_power_iter, fused_agzo_perturbation, fused_perturb_dual).
* ``dsmezo_b200.AdapterSet`` / ``ZOController`` - the whole optimizer step over every
  adapter of every layer as grouped launches (one sequence per phase).
* ``dsmezo_b200.sharding`` - layer-sharded step over ranks (NCCL).
* ``dsmezo_b200.calibration`` - first-step basis width (optimal hard threshold) and the
  batched randomized SVD of the bases (``AdapterSet.calibrate``).

All compute runs in libdsmezo.so (C ABI in include/dsmezo.h); there is no CPU path.
"""
from . import calibration  # noqa: F401
from . import kernels  # noqa: F401
from . import scoring  # noqa: F401
from ._lib import DsmzError, lib  # noqa: F401
from .adapter_set import (AdapterSet, BasisShape, ModuleShape, ShrinkageRLOO, ZOController,  # noqa: F401
                          device_layout, draw_increments, eps_from_norms, kalman_beta_q, rloo_direction_scalars,
                          transformer_adapter_shapes)
from .calibration import calibration_rank  # noqa: F401
from .sharding import ShardedStep, ShardLayout, partition_layers, shard_layout  # noqa: F401

__all__ = ["kernels", "rloo_direction_scalars", "AdapterSet", "ZOController", "ModuleShape", "BasisShape", "transformer_adapter_shapes",
           "draw_increments", "device_layout", "kalman_beta_q", "DsmzError", "lib", "ShardedStep", "ShardLayout",
           "partition_layers", "shard_layout", "ShrinkageRLOO", "eps_from_norms", "calibration",
           "calibration_rank"]
