"""ctypes binding of libphyzb200.so (include/phyzb.h).

Loading fails loudly: there is no CPU fallback for any entry point. The
struct layouts below mirror include/phyzb.h field for field.
"""
from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libphyzb200.so"

PHYZB_OK = 0
ERR_INVALID = -1
ERR_CUDA = -2
ERR_NO_DEVICE = -3
ERR_STATE = -4
ERR_NONFINITE = -5
ERR_TOO_LARGE = -6
ERR_UNSUPPORTED = -7
ERR_COMM = -8
COMM_ID_BYTES = 128
GAE_NOALLOC_MAX_WORLDS = 1 << 24
DEFAULT_CONTACT_SWEEPS = 16
MAX_CONTACT_SWEEPS = 1024

F32 = 0
F64 = 1
HOST_F32 = 0
HOST_F64 = 1
MAX_BODIES = 32
MAX_DOFS = 64
CONTACT_STRIDE = 8

JOINT_REVOLUTE, JOINT_PRISMATIC, JOINT_FIXED, JOINT_BALL, JOINT_FREE = 0, 1, 2, 3, 4
GEOM_NONE, GEOM_SPHERE, GEOM_BOX, GEOM_CAPSULE, GEOM_CYLINDER, GEOM_MESH_AABB = 0, 1, 2, 3, 4, 5


class PhyzbBody(C.Structure):
    _fields_ = [
        ("parent", C.c_int32),
        ("joint_type", C.c_int32),
        ("mass", C.c_double),
        ("com", C.c_double * 3),
        ("inertia", C.c_double * 6),
        ("ptj_rot", C.c_double * 9),
        ("ptj_pos", C.c_double * 3),
        ("axis", C.c_double * 3),
        ("damping", C.c_double),
        ("stiffness", C.c_double),
        ("spring_ref", C.c_double),
        ("armature", C.c_double),
        ("has_limits", C.c_int32),
        ("limit_lower", C.c_double),
        ("limit_upper", C.c_double),
        ("limit_stiffness", C.c_double),
        ("limit_damping", C.c_double),
        ("friction_loss", C.c_double),
        ("geom_type", C.c_int32),
        ("geom_params", C.c_double * 6),
        ("geom_origin_pos", C.c_double * 3),
        ("geom_origin_rot", C.c_double * 9),
    ]


class PhyzbModel(C.Structure):
    _fields_ = [
        ("nbodies", C.c_int32),
        ("gravity", C.c_double * 3),
        ("dt", C.c_double),
        ("bodies", C.POINTER(PhyzbBody)),
    ]


class PhyzbHeightfield(C.Structure):
    _fields_ = [("origin", C.c_double * 3), ("cell", C.c_double), ("nx", C.c_int32), ("ny", C.c_int32),
                ("heights", C.POINTER(C.c_float))]


class PhyzbBodyPlane(C.Structure):
    _fields_ = [("body", C.c_int32), ("offset", C.c_double), ("max_depth", C.c_double), ("half_x", C.c_double),
                ("half_y", C.c_double), ("exclude", C.POINTER(C.c_int32)), ("n_exclude", C.c_int32)]


class PhyzbPdDof(C.Structure):
    _fields_ = [
        ("q_index", C.c_int32),
        ("v_index", C.c_int32),
        ("kp", C.c_double),
        ("kd", C.c_double),
        ("max_force", C.c_double),
    ]


class PhyzbDeviceView(C.Structure):
    _fields_ = [
        ("q", C.c_void_p),
        ("v", C.c_void_p),
        ("ctrl", C.c_void_p),
        ("qdd", C.c_void_p),
        ("nworld", C.c_int64),
        ("nv", C.c_int32),
        ("nbodies", C.c_int32),
        ("precision", C.c_int32),
        ("device", C.c_int32),
        ("stream", C.c_void_p),
    ]


class PhyzbPolicySpec(C.Structure):
    _fields_ = [
        ("n_obs", C.c_int32),
        ("obs_ops", C.POINTER(C.c_float)),
        ("n_aux", C.c_int32),
        ("obs_aux", C.POINTER(C.c_float)),
        ("hidden", C.c_int32),
        ("n_act", C.c_int32),
        ("act_slots", C.POINTER(C.c_int32)),
        ("act_clamp", C.c_double),
        ("act_clamp_slots", C.POINTER(C.c_double)),
        ("noise_rho", C.c_double),
        ("input_noise", C.POINTER(C.c_double)),
        ("history_steps", C.c_int32),
    ]


class PhyzbNetDims(C.Structure):
    _fields_ = [("n_in", C.c_int32), ("n_h", C.c_int32), ("n_out", C.c_int32)]


class PhyzbAdamCfg(C.Structure):
    _fields_ = [("lr", C.c_double), ("beta1", C.c_double), ("beta2", C.c_double), ("eps", C.c_double),
                ("weight_decay", C.c_double)]


class PhyzbPpoCfg(C.Structure):
    _fields_ = [("clip", C.c_double), ("entropy_coef", C.c_double), ("vdelta", C.c_double),
                ("minibatch", C.c_int32), ("epochs", C.c_int32), ("target_kl", C.c_double),
                ("kl_scale", C.c_double), ("kl_mode", C.c_int32)]


class PhyzbUpdateStats(C.Structure):
    _fields_ = [("policy_loss", C.c_double), ("value_loss", C.c_double), ("kl", C.c_double),
                ("grad_steps", C.c_int32), ("stopped_early", C.c_int32)]


class PhyzbBatchCol(C.Structure):
    _fields_ = [("base", C.c_void_p), ("block", C.c_int64), ("features", C.c_int32)]


class PhyzbPolicyHistory(C.Structure):
    _fields_ = [("obs", C.c_void_p), ("out", C.c_void_p), ("n_obs", C.c_int32), ("n_act", C.c_int32),
                ("nworld", C.c_int64), ("steps", C.c_int32)]


class PhyzbReturnCfg(C.Structure):
    _fields_ = [("reward_coef", C.POINTER(C.c_double)), ("action_penalty", C.c_double), ("gamma", C.c_double),
                ("lambda_", C.c_double), ("steps", C.c_int32), ("normalize", C.c_int32)]


KINEMATICS_STRIDE = 18

_P = C.c_void_p
_D = C.POINTER(C.c_double)
_I32P = C.POINTER(C.c_int32)
_FP = C.POINTER(C.c_float)

# name -> (restype, argtypes)
SIGNATURES = {
    "phyzb_last_error": (C.c_char_p, []),
    "phyzb_abi_version": (C.c_int, []),
    "phyzb_device_count": (C.c_int, []),
    "phyzb_create": (C.c_int, [C.POINTER(PhyzbModel), C.c_int64, C.c_int, C.c_int, C.POINTER(_P)]),
    "phyzb_destroy": (C.c_int, [_P]),
    "phyzb_set_model": (C.c_int, [_P, C.POINTER(PhyzbModel)]),
    "phyzb_enable_ground_contact": (C.c_int, [_P, C.c_double, C.c_double, C.c_double, C.c_double, _I32P]),
    "phyzb_enable_ground_contact_per_body": (C.c_int, [_P, C.c_double, C.c_double, _D, _D, _I32P]),
    "phyzb_enable_contact_impulse": (C.c_int, [_P, C.c_double, C.c_double, _D, _D, _P, _P, _I32P]),
    "phyzb_enable_contact_terrain": (C.c_int, [_P, C.c_double, C.c_double, _D, _D, _P, _P, _I32P]),
    "phyzb_set_heightfield": (C.c_int, [_P, _P]),
    "phyzb_set_contact_sweeps": (C.c_int, [_P, C.c_int32]),
    "phyzb_disable_contact": (C.c_int, [_P]),
    "phyzb_collidable_bodies": (C.c_int, [_P]),
    "phyzb_enable_pd": (C.c_int, [_P, C.POINTER(PhyzbPdDof), C.c_int32]),
    "phyzb_set_position_targets": (C.c_int, [_P, _D]),
    "phyzb_load_states": (C.c_int, [_P, _D, _D, _D]),
    "phyzb_set_controls": (C.c_int, [_P, _D]),
    "phyzb_step": (C.c_int, [_P, C.c_int32]),
    "phyzb_step_with_controls": (C.c_int, [_P, _P, C.c_int, C.c_int32]),
    "phyzb_sync": (C.c_int, [_P]),
    "phyzb_status": (C.c_int, [_P]),
    "phyzb_clear_status": (C.c_int, [_P]),
    "phyzb_readback_states": (C.c_int, [_P, _D, _D]),
    "phyzb_readback_qdd": (C.c_int, [_P, _D]),
    "phyzb_readback_contacts": (C.c_int, [_P, _D]),
    "phyzb_device_view_get": (C.c_int, [_P, C.POINTER(PhyzbDeviceView)]),
    "phyzb_set_stream": (C.c_int, [_P, _P]),
    "phyzb_load_states_device": (C.c_int, [_P, _P, _P, _P]),
    "phyzb_step_device_controls": (C.c_int, [_P, _P, C.c_int64, C.c_int32]),
    "phyzb_objective_device": (C.c_int, [_P, C.c_int, _P]),
    "phyzb_flops_per_world_step": (C.c_int, [_P, _D, _D]),
    "phyzb_flops_executed": (C.c_int, [_P, _D, _D, _D, C.c_int64, C.c_int32, C.c_int32, _D, _D]),
    "phyzb_set_world_lanes": (C.c_int, [_P, C.c_int32]),
    "phyzb_reduce_objective_device": (C.c_int, [_P, _P, C.c_int, _P]),
    "phyzb_comm_sync": (C.c_int, [_P, _P, C.c_double]),
    "phyzb_get_world_lanes": (C.c_int, [_P, C.POINTER(C.c_int32), C.POINTER(C.c_int32)]),
    "phyzb_launch_info": (C.c_int, [_P, _I32P, _I32P, _I32P, _I32P, _I32P]),
    "phyzb_slice_plan": (C.c_int, [_P, C.c_int32, _I32P, _I32P, _I32P]),
    "phyzb_set_kernel_specialization": (C.c_int, [_P, C.c_int32]),
    "phyzb_get_kernel_specialization": (C.c_int, [_P, _I32P, _I32P]),
    "phyzb_enable_policy": (C.c_int, [_P, C.POINTER(PhyzbPolicySpec)]),
    "phyzb_set_policy_weights": (C.c_int, [_P, _D, C.c_int64]),
    "phyzb_set_policy_std": (C.c_int, [_P, _D, C.c_int32]),
    "phyzb_set_policy_base_targets": (C.c_int, [_P, _D]),
    "phyzb_seed_policy": (C.c_int, [_P, C.c_uint64]),
    "phyzb_run_policy": (C.c_int, [_P, C.c_int32]),
    "phyzb_policy_rollout": (C.c_int, [_P, C.c_int32, C.c_int32, C.c_int32]),
    "phyzb_readback_policy_history": (C.c_int, [_P, C.c_int32, C.c_int32, _FP, _FP]),
    "phyzb_readback_targets": (C.c_int, [_P, _D]),
    "phyzb_readback_kinematics": (C.c_int, [_P, _D]),
    "phyzb_trainer_create": (C.c_int, [C.c_int32, PhyzbNetDims, PhyzbNetDims, C.c_int64, C.c_int32,
                                       C.POINTER(_P)]),
    "phyzb_trainer_destroy": (C.c_int, [_P]),
    "phyzb_trainer_set_adam": (C.c_int, [_P, C.POINTER(PhyzbAdamCfg), C.POINTER(PhyzbAdamCfg)]),
    "phyzb_trainer_set_params": (C.c_int, [_P, C.c_int32, _D, C.c_int64]),
    "phyzb_trainer_params": (C.c_int, [_P, C.c_int32, _D, C.c_int64]),
    "phyzb_trainer_upload_batch": (C.c_int, [_P, C.c_int64, _FP, _FP, _FP, _FP, _FP, _FP]),
    "phyzb_trainer_update": (C.c_int, [_P, C.POINTER(C.c_uint32), C.c_int32, C.POINTER(PhyzbPpoCfg),
                                       C.POINTER(PhyzbUpdateStats)]),
    "phyzb_trainer_set_batch_device": (C.c_int, [_P, C.c_int64, C.POINTER(PhyzbBatchCol)]),
    "phyzb_trainer_update_shuffled": (C.c_int, [_P, C.POINTER(PhyzbPpoCfg), C.c_uint64,
                                                C.POINTER(PhyzbUpdateStats)]),
    "phyzb_trainer_evaluate": (C.c_int, [_P, C.c_int32, PhyzbBatchCol, C.c_int64, C.c_void_p]),
    "phyzb_trainer_set_comm": (C.c_int, [_P, _P]),
    "phyzb_policy_history_view": (C.c_int, [_P, C.POINTER(PhyzbPolicyHistory)]),
    "phyzb_policy_advantages": (C.c_int, [_P, _P, _P, C.POINTER(PhyzbReturnCfg), C.c_void_p, C.c_void_p, _D]),
    "phyzb_policy_sync_from_trainer": (C.c_int, [_P, _P]),
    "phyzb_gae_noalloc": (C.c_int, [_P, _P, C.c_int64, C.c_int32, C.c_double, C.c_double, C.c_int32, C.c_int32, _P,
                                    _P, _P, _D]),
    "phyzb_enable_state_history": (C.c_int, [_P, C.c_int32]),
    "phyzb_record_state": (C.c_int, [_P, C.c_int32]),
    "phyzb_readback_state_history": (C.c_int, [_P, C.c_int32, C.c_int32, _D, _D]),
    "phyzb_comm_unique_id": (C.c_int, [C.POINTER(C.c_uint8)]),
    "phyzb_comm_init": (C.c_int, [C.POINTER(C.c_uint8), C.c_int32, C.c_int32, C.c_int32, C.c_double,
                                  C.POINTER(_P)]),
    "phyzb_comm_destroy": (C.c_int, [_P]),
    "phyzb_reduce_objective": (C.c_int, [_P, _P, C.c_int, C.c_double, C.POINTER(C.c_double)]),
    "phyzb_measure_fma_peak": (C.c_int, [C.c_int, _D]),
}

_lib = None


def load() -> C.CDLL:
    """Load the library (built by phyz_b200.build). Raises if it is missing."""
    global _lib
    if _lib is not None:
        return _lib
    if not LIB_PATH.exists():
        raise RuntimeError(
            f"{LIB_PATH} is missing: build it with `python -m phyz_b200.build` "
            "(there is no CPU fallback for the stepper)"
        )
    lib = C.CDLL(str(LIB_PATH))
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


class PhyzbError(RuntimeError):
    """A failing libphyzb200 call: `code` is the PHYZB_ERR_* value."""

    def __init__(self, code: int, message: str):
        super().__init__(f"[{code}] {message}")
        self.code = code
        self.message = message


def check(code: int) -> int:
    if code < 0:
        msg = load().phyzb_last_error().decode("utf-8", "replace")
        raise PhyzbError(code, msg)
    return code


def dptr(a) -> C.POINTER(C.c_double):
    """Pointer to a C-contiguous float64 numpy array."""
    return a.ctypes.data_as(_D)


def lib_path() -> str:
    return os.fspath(LIB_PATH)
