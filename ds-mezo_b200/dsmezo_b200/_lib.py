"""ctypes binding of libdsmezo.so (declarations in include/dsmezo.h).

The library is built in-tree (``python -m dsmezo_b200.build``) next to this file. There
is no fallback: when the shared library is missing, every entry point raises.
"""
from __future__ import annotations

import ctypes
import os
from ctypes import POINTER, c_char_p, c_double, c_float, c_int32, c_int64, c_size_t, c_uint32, c_uint64, c_void_p

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libdsmezo.so")

ABI_VERSION = 3              # DSMZ_ABI_VERSION of the structs below
DSMZ_F32 = 0
DSMZ_BF16 = 1
MAX_RANK = 128
MAX_NS_ITERS = 16


class DsmzError(RuntimeError):
    """A libdsmezo entry point returned an error status."""


class NSSchedule(ctypes.Structure):
    _fields_ = [("iters", c_int32), ("c", (c_double * 3) * MAX_NS_ITERS)]


class ModuleSpec(ctypes.Structure):
    _fields_ = [
        ("A", c_void_p), ("B", c_void_p),
        ("pos_A", c_void_p), ("pos_B", c_void_p), ("neg_A", c_void_p), ("neg_B", c_void_p),
        ("shadow_A", c_void_p), ("shadow_B", c_void_p),
        ("mu_A", c_void_p), ("mu_B", c_void_p), ("var_A", c_void_p), ("var_B", c_void_p),
        ("z_A", c_void_p), ("z_B", c_void_p),
        ("scratch_A", c_void_p), ("scratch_B", c_void_p),
        ("d_out", c_int64), ("d_in", c_int64), ("r", c_int64),
        ("ld_A", c_int64), ("ld_B", c_int64),
        ("basis", c_int32), ("layer", c_int32),
    ]


class BasisSpec(ctypes.Structure):
    _fields_ = [
        ("H", c_void_p), ("h_dtype", c_int32),
        ("T", c_int64), ("D", c_int64), ("ld_H", c_int64),
        ("V", c_void_p), ("R", c_int64),
    ]


class PlanDesc(ctypes.Structure):
    _fields_ = [
        ("copy_dtype", c_int32),
        ("num_modules", c_int32), ("modules", POINTER(ModuleSpec)),
        ("num_bases", c_int32), ("bases", POINTER(BasisSpec)),
        ("sm_count", c_int32), ("max_threads_per_sm", c_int32),
        ("rng_offset_before", c_uint64),
        ("flags", ctypes.c_uint32),
        ("directions", c_int32), ("pad0", c_int32),
        ("dir_stride_factor", c_int64), ("dir_stride_z", c_int64),
        ("rng_direction_stride", c_uint64),
        ("module_rng_offsets", POINTER(c_uint64)),
    ]


MAX_DIRECTIONS = 32
PI_BASIS_UNCHANGED = 1        # dsmz_step_power_iteration_ex flag (include/dsmezo.h)


PLAN_SIMT_POWER_ITER = 1
PLAN_SINGLE_PASS_POWER_ITER = 2
PLAN_CUDA_CORE_PERTURB = 4


# name -> (restype, argtypes); mirrors include/dsmezo.h
SIGNATURES = {
    "dsmz_last_error": (c_char_p, []),
    "dsmz_abi_version": (c_int32, []),
    "dsmz_ns_schedule_cubic": (c_int32, [POINTER(NSSchedule)]),
    "dsmz_ns_schedule_quintic": (c_int32, [POINTER(NSSchedule)]),
    "dsmz_zo_muon_update_workspace_bytes": (c_size_t, [c_int64, c_int64]),
    "dsmz_zo_muon_update": (c_int32, [c_int32, c_void_p, c_int64, c_int64, c_void_p, c_int64, c_int64,
                                      c_void_p, c_int64, c_int64, c_int64, c_int64, c_float, c_float,
                                      POINTER(NSSchedule), c_void_p, c_size_t, c_void_p]),
    "dsmz_zo_muon_update_noalloc": (c_int32, [c_int32, c_void_p, c_int64, c_int64, c_void_p, c_int64, c_int64,
                                              c_void_p, c_int64, c_int64, c_int64, c_int64, c_float, c_float,
                                              POINTER(NSSchedule), c_void_p]),
    "dsmz_power_iter_workspace_bytes": (c_size_t, [c_int64, c_int64, c_int64]),
    "dsmz_contrastive_loss_workspace_bytes": (c_size_t, [c_int64]),
    "dsmz_contrastive_loss": (c_int32, [c_int32, c_void_p, c_int64, c_int64, c_void_p, c_int64, POINTER(c_int64),
                                        POINTER(c_double), c_int32, c_void_p, c_void_p, c_size_t, c_void_p]),
    "dsmz_activation_load": (c_int32, [c_int32, c_void_p, c_int64, c_int64, c_int64, c_int32, c_void_p,
                                       c_int64, c_int64, c_int64, c_void_p]),
    "dsmz_power_iter": (c_int32, [c_int32, c_void_p, c_int64, c_int64, c_int64, c_int64,
                                  c_void_p, c_int64, c_int64, c_int64, c_void_p, c_int32, c_float,
                                  c_void_p, c_size_t, c_void_p]),
    "dsmz_agzo_perturbation_workspace_bytes": (c_size_t, [c_int64, c_int64, c_int64, c_int64]),
    "dsmz_agzo_perturbation": (c_int32, [c_void_p, c_int64, c_int64, c_int64, c_int64,
                                         c_void_p, c_int64, c_int64, c_int64,
                                         c_void_p, c_void_p, c_int64, c_void_p, c_void_p, c_float, c_float,
                                         c_void_p, c_size_t, c_void_p]),
    "dsmz_perturb_dual": (c_int32, [c_int32, c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_void_p]),
    "dsmz_randn_threads": (c_int64, [c_int64, c_int32, c_int32]),
    "dsmz_randn_offset_increment": (c_uint64, [c_int64, c_int32, c_int32]),
    "dsmz_randn": (c_int32, [c_void_p, c_int64, c_uint64, c_uint64, c_int32, c_int32, c_void_p]),
    "dsmz_plan_create": (c_int32, [POINTER(PlanDesc), POINTER(c_void_p)]),
    "dsmz_plan_destroy": (None, [c_void_p]),
    "dsmz_plan_table_bytes": (c_size_t, [c_void_p]),
    "dsmz_plan_workspace_bytes": (c_size_t, [c_void_p]),
    "dsmz_plan_rng_increment": (c_uint64, [c_void_p]),
    "dsmz_plan_launch_count": (c_int32, [c_void_p, c_int32]),
    "dsmz_plan_bind": (c_int32, [c_void_p, c_void_p, c_size_t, c_void_p, c_size_t, c_void_p]),
    "dsmz_plan_uses_tensor_cores": (c_int32, [c_void_p]),
    "dsmz_plan_directions": (c_int32, [c_void_p]),
    "dsmz_plan_factor_norms": (c_int32, [c_void_p, c_void_p, c_void_p]),
    "dsmz_step_draw": (c_int32, [c_void_p, c_uint64, c_uint64, c_void_p]),
    "dsmz_plan_set_gather_peers": (c_int32, [c_void_p, c_int32, c_void_p, c_void_p, c_void_p]),
    "dsmz_ipc_export": (c_int32, [c_void_p, c_void_p, POINTER(c_int64)]),
    "dsmz_ipc_import": (c_int32, [c_void_p, c_int64, POINTER(c_void_p)]),
    "dsmz_ipc_close": (c_int32, [c_void_p, c_int64]),
    "dsmz_peer_copy": (c_int32, [c_void_p, c_void_p, c_int64, c_void_p]),
    "dsmz_plan_perturb_on_tensor_cores": (c_int32, [c_void_p]),
    "dsmz_plan_calibration_workspace_bytes": (c_size_t, [c_void_p]),
    "dsmz_plan_calibration_rng_increment": (c_uint64, [c_void_p]),
    "dsmz_plan_calibration_launch_count": (c_int32, [c_void_p, c_int32]),
    "dsmz_plan_calibrate": (c_int32, [c_void_p, c_uint64, c_uint64, c_int32, c_float, c_void_p, c_size_t,
                                      c_void_p, c_void_p]),
    "dsmz_step_update_directions": (c_int32, [c_void_p, POINTER(c_float), c_int32, c_float, c_float, c_float,
                                              c_float, POINTER(NSSchedule), c_void_p]),
    "dsmz_plan_device_error": (c_int32, [c_void_p, c_void_p]),
    "dsmz_step_power_iteration": (c_int32, [c_void_p, c_int32, c_float, c_void_p]),
    "dsmz_step_power_iteration_ex": (c_int32, [c_void_p, c_int32, c_float, c_uint32, c_void_p]),
    "dsmz_step_perturb": (c_int32, [c_void_p, c_uint64, c_uint64, c_float, c_float, c_float, c_float, c_void_p]),
    "dsmz_step_kalman_sums": (c_void_p, [c_void_p]),
    "dsmz_step_update": (c_int32, [c_void_p, c_float, c_float, c_float, c_float, c_float, POINTER(NSSchedule),
                                   c_void_p]),
    "dsmz_plan_set_probe": (c_int32, [c_void_p, c_int32, POINTER(c_void_p), POINTER(c_void_p), c_int32]),
    "dsmz_plan_probe_count": (c_int32, [c_void_p, c_int32]),
}

KERNEL_IDS = {"pi_y": 0, "pi_w": 1, "pi_gram": 2, "pi_chol": 3, "pi_apply": 4, "bside": 5, "coef": 6,
              "perturb": 7, "kalman_sum": 8, "gram": 9, "ns_solve": 10, "apply": 11, "pi_split": 12, "draw": 13,
              "kalman_dirs": 14, "pi_fused": 15}

_lib = None


def lib() -> ctypes.CDLL:
    """The loaded library; raises if it has not been built."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(f"libdsmezo.so not found at {LIB_PATH}; build it with "
                              f"`python -m dsmezo_b200.build` (nvcc, sm_100a)")
        handle = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(handle, name)
            fn.restype = res
            fn.argtypes = args
        if handle.dsmz_abi_version() != ABI_VERSION:
            raise ImportError(f"{LIB_PATH} has ABI version {handle.dsmz_abi_version()}, this binding expects "
                              f"{ABI_VERSION}; rebuild it with `python -m dsmezo_b200.build`")
        _lib = handle
    return _lib


def check(status: int, what: str) -> None:
    if status != 0:
        msg = lib().dsmz_last_error()
        raise DsmzError(f"{what} failed (status {status}): {msg.decode() if msg else ''}")


def schedule(name_or_coeffs) -> NSSchedule:
    """'cubic' (reference), 'quintic', or a sequence of (c0, c1, c2) triples."""
    s = NSSchedule()
    if isinstance(name_or_coeffs, str):
        fn = {"cubic": lib().dsmz_ns_schedule_cubic, "quintic": lib().dsmz_ns_schedule_quintic}.get(name_or_coeffs)
        if fn is None:
            raise ValueError(f"unknown Newton-Schulz schedule {name_or_coeffs!r}")
        check(fn(ctypes.byref(s)), "schedule")
        return s
    coeffs = list(name_or_coeffs)
    if len(coeffs) > MAX_NS_ITERS:
        raise ValueError(f"at most {MAX_NS_ITERS} Newton-Schulz iterations")
    s.iters = len(coeffs)
    for i, tr in enumerate(coeffs):
        tr = tuple(tr) + (0.0,) * (3 - len(tr))
        for j in range(3):
            s.c[i][j] = float(tr[j])
    return s
