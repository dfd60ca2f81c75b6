"""ctypes binding of libmmn_optim_cuda.so (declarations in include/mmn_optim.h).

Loading fails loudly when the library has not been built: there is no CPU
fallback for any entry point.
"""
from __future__ import annotations

import ctypes
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "_lib", "libmmn_optim_cuda.so")

MMN_OK = 0
MMN_E_INVALID, MMN_E_SHAPE, MMN_E_CUDA, MMN_E_NO_DEVICE = -1, -2, -3, -4
MMN_E_STATE, MMN_E_OOM, MMN_E_TIMEOUT, MMN_E_UNSUPPORTED = -5, -6, -7, -8
MEM_HOST, MEM_DEVICE = 0, 1
DTYPE_F32, DTYPE_BF16 = 0, 1
ROUTE_AUTO, ROUTE_MUON, ROUTE_ADAMW = 0, 1, 2
NS_REFERENCE, NS_BF16, NS_TF32, NS_FP32 = 0, 1, 2, 3


class MmnError(RuntimeError):
    """Base error of the optimizer library (mirrors crates/mmn-core/src/error.rs)."""

    def __init__(self, code: int, message: str):
        super().__init__(f"[{code}] {message}")
        self.code = code


class CUDAError(MmnError):
    """CUDA requested but unusable (MmnError::Cuda, crates/mmn-core/src/error.rs:84-90;
    surfaced to Python as CUDAError by crates/mmn-py/src/errors.rs:27)."""


class ShapeError(MmnError):
    """Shape differs from the registered state (the reference panics here)."""


class KernelTimeoutError(MmnError):
    """A kernel gave up a bounded wait and reported it instead of hanging."""


_ERRORS = {MMN_E_NO_DEVICE: CUDAError, MMN_E_SHAPE: ShapeError, MMN_E_TIMEOUT: KernelTimeoutError}


class AdamWConfigC(ctypes.Structure):
    _fields_ = [("lr", ctypes.c_float), ("beta1", ctypes.c_float), ("beta2", ctypes.c_float),
                ("eps", ctypes.c_float), ("weight_decay", ctypes.c_float)]


class MuonConfigC(ctypes.Structure):
    _fields_ = [("lr", ctypes.c_float), ("momentum", ctypes.c_float),
                ("nesterov", ctypes.c_int32), ("ns_steps", ctypes.c_int32)]


class OptimConfigC(ctypes.Structure):
    _fields_ = [("adamw", AdamWConfigC), ("muon", MuonConfigC), ("use_hybrid", ctypes.c_int32),
                ("ns_mode", ctypes.c_int32), ("fresh_state", ctypes.c_int32),
                ("grad_dtype", ctypes.c_int32), ("bf16_param_shadow", ctypes.c_int32),
                ("loss_scaling", ctypes.c_int32), ("loss_scale_init", ctypes.c_float),
                ("growth_interval", ctypes.c_int32), ("rank", ctypes.c_int32),
                ("world_size", ctypes.c_int32), ("use_graph", ctypes.c_int32),
                ("reduce_grads", ctypes.c_int32), ("scan_shard", ctypes.c_int32)]


class GatherLayoutC(ctypes.Structure):
    _fields_ = [("adamw_param", ctypes.c_void_p), ("adamw_param_bf16", ctypes.c_void_p),
                ("adamw_region", ctypes.c_int64), ("muon_param", ctypes.c_void_p),
                ("muon_param_bf16", ctypes.c_void_p), ("muon_region", ctypes.c_int64)]


_vp = ctypes.c_void_p
_i = ctypes.c_int
_u64 = ctypes.c_uint64
_i64 = ctypes.c_int64
_f = ctypes.c_float
_i64p = ctypes.POINTER(ctypes.c_int64)

# name -> (restype, argtypes); every name is declared in include/mmn_optim.h
SIGNATURES = {
    "mmn_cuda_is_available": (_i, []),
    "mmn_require_cuda": (_i, [_i]),
    "mmn_last_error": (ctypes.c_char_p, []),
    "mmn_abi_version": (_i, []),
    "mmn_selftest_bounded_wait": (_i, [_i, _u64]),
    "mmn_adamw_config_default": (AdamWConfigC, []),
    "mmn_muon_config_default": (MuonConfigC, []),
    "mmn_adamw_create": (_i, [ctypes.POINTER(AdamWConfigC), _i, _vp, ctypes.POINTER(_vp)]),
    "mmn_adamw_destroy": (_i, [_vp]),
    "mmn_adamw_step_param": (_i, [_vp, _u64, _vp, _vp, _i64p, _i, _f, _i]),
    "mmn_adamw_get_step": (_i, [_vp, ctypes.POINTER(_u64)]),
    "mmn_adamw_set_step": (_i, [_vp, _u64]),
    "mmn_adamw_export_state": (_i, [_vp, _u64, _i, _vp, _i64, _i]),
    "mmn_adamw_import_state": (_i, [_vp, _u64, _i, _vp, _i64, _i]),
    "mmn_muon_create": (_i, [ctypes.POINTER(MuonConfigC), _i, _i, _vp, ctypes.POINTER(_vp)]),
    "mmn_muon_destroy": (_i, [_vp]),
    "mmn_muon_register": (_i, [_vp, _u64, _i64p, _i]),
    "mmn_muon_step_matrix": (_i, [_vp, _u64, _vp, _vp, _i64p, _i, _f, _i]),
    "mmn_muon_export_velocity": (_i, [_vp, _u64, _vp, _i64, _i]),
    "mmn_muon_import_velocity": (_i, [_vp, _u64, _vp, _i64, _i]),
    "mmn_newton_schulz5": (_i, [_vp, _i64p, _i, _i, _i, _vp, _i, _vp, _i]),
    "mmn_newton_schulz5_noalloc": (_i, [_vp, _i64, _i64, _i, _i, _vp, _i, _vp]),
    "mmn_newton_schulz_iteration": (_i, [_vp, _i64, _i64, _f, _i, _vp, _vp, _vp, _i]),
    "mmn_hybrid_classify_param": (_i, [_i64p, _i]),
    "mmn_hybrid_create": (_i, [ctypes.POINTER(MuonConfigC), ctypes.POINTER(AdamWConfigC), _i, _i,
                               _vp, ctypes.POINTER(_vp)]),
    "mmn_hybrid_destroy": (_i, [_vp]),
    "mmn_hybrid_step": (_i, [_vp, _u64, _vp, _vp, _i64p, _i, _i, _f, _i]),
    "mmn_hybrid_adamw": (_vp, [_vp]),
    "mmn_hybrid_muon": (_vp, [_vp]),
    "mmn_optim_config_default": (OptimConfigC, []),
    "mmn_optim_create": (_i, [ctypes.POINTER(OptimConfigC), _i, _vp, ctypes.POINTER(_vp)]),
    "mmn_optim_destroy": (_i, [_vp]),
    "mmn_optim_add_param": (_i, [_vp, _u64, _i64p, _i, _i, ctypes.POINTER(_i)]),
    "mmn_optim_finalize": (_i, [_vp]),
    "mmn_optim_slot_ptrs": (_i, [_vp, _i, ctypes.POINTER(_vp), ctypes.POINTER(_vp),
                                 ctypes.POINTER(_vp)]),
    "mmn_optim_set_param": (_i, [_vp, _i, _vp, _i]),
    "mmn_optim_get_param": (_i, [_vp, _i, _vp, _i]),
    "mmn_optim_set_grad": (_i, [_vp, _i, _vp, _i]),
    "mmn_optim_set_state": (_i, [_vp, _i, _i, _vp, _i]),
    "mmn_optim_get_state": (_i, [_vp, _i, _i, _vp, _i]),
    "mmn_optim_set_adamw_step": (_i, [_vp, _u64]),
    "mmn_optim_get_adamw_step": (_i, [_vp, ctypes.POINTER(_u64)]),
    "mmn_optim_step": (_i, [_vp, _f]),
    "mmn_optim_step_host": (_i, [_vp, ctypes.POINTER(_vp), ctypes.POINTER(_vp), _f]),
    "mmn_optim_sync": (_i, [_vp]),
    "mmn_optim_loss_scale": (_i, [_vp, ctypes.POINTER(_f), ctypes.POINTER(_i64)]),
    "mmn_optim_get_loss_state": (_i, [_vp, ctypes.POINTER(_f), ctypes.POINTER(_i64),
                                      ctypes.POINTER(ctypes.c_int32)]),
    "mmn_optim_set_loss_state": (_i, [_vp, _f, _i64, ctypes.c_int32]),
    "mmn_optim_slot_owner": (_i, [_vp, _i, ctypes.POINTER(_i)]),
    "mmn_optim_get_gather_layout": (_i, [_vp, ctypes.POINTER(GatherLayoutC)]),
    "mmn_optim_param_counts": (_i, [_vp, _i64p, _i64p, _i64p]),
    "mmn_optim_export_ipc": (_i, [_vp, _vp]),
    "mmn_optim_connect_peers": (_i, [_vp, ctypes.c_char_p]),
    "mmn_optim_reduce_grads": (_i, [_vp]),
    "mmn_optim_scan_grads": (_i, [_vp, _vp]),
    "mmn_grad_reduce": (_i, [ctypes.POINTER(_vp), _i, _vp, _i64, _i, _vp, _i, _vp]),
    "mmn_grad_nonfinite_scan": (_i, [_vp, _i64, _i, ctypes.POINTER(_vp), _i, _i, _vp]),
    "mmn_optim_plan": (_i, [_i64p, ctypes.POINTER(_i), ctypes.POINTER(_i), _i, _i, _i, _i,
                            ctypes.POINTER(_i), _i64p, _i64p, _i64p]),
    "mmn_optim_ns_flops": (_i, [_vp, ctypes.POINTER(ctypes.c_double)]),
    "mmn_optim_kernel_launches": (_i, [_vp, _i64p, _i64p]),
    "mmn_optim_enable_timing": (_i, [_vp, _i]),
    "mmn_optim_last_timing": (_i, [_vp, ctypes.POINTER(_f)]),
    "mmn_optim_last_timing_ex": (_i, [_vp, ctypes.POINTER(_f)]),
}

_lib = None


def lib() -> ctypes.CDLL:
    """The loaded library. Raises if it has not been built."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(
                f"{LIB_PATH} is missing: build it with `python -m magicmindnet_b200.build` "
                "(nvcc, sm_100a). There is no CPU fallback.")
        L = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def check(rc: int) -> None:
    if rc != MMN_OK:
        msg = lib().mmn_last_error().decode(errors="replace")
        raise _ERRORS.get(rc, MmnError)(rc, msg)


def shape_array(shape) -> ctypes.Array:
    shape = tuple(int(s) for s in shape)
    return (ctypes.c_int64 * max(len(shape), 1))(*shape)
