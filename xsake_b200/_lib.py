"""ctypes binding of libxsake_hads.so (the C ABI declared in include/xsake_hads.h).

This module is the only place that loads the native library.  There is no fallback: if the
library is missing or no CUDA device is present, every operator raises ``XsakeError``.
"""

from __future__ import annotations

import ctypes as C
import os
import threading

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "lib", "libxsake_hads.so")

XSAKE_OK, XSAKE_EINVAL, XSAKE_EUNSUPPORTED, XSAKE_ECUDA, XSAKE_ETIMEOUT, XSAKE_EDEVICE = range(6)
XSAKE_F32, XSAKE_BF16 = 0, 1
ABI_VERSION = 1


class XsakeError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"[xsake status {code}] {msg}")
        self.code = code


class MaskDims(C.Structure):
    _fields_ = [("batch", C.c_int32), ("heads", C.c_int32), ("seq", C.c_int32),
                ("mask_batch", C.c_int32), ("mask_heads", C.c_int32),
                ("block_size", C.c_int32), ("causal", C.c_int32)]


class PlanOptions(C.Structure):
    _fields_ = [("units_dev", C.c_void_p), ("n_units", C.c_int32), ("workers", C.c_int32),
                ("forward_pairing", C.c_int32)]


class PlanInfo(C.Structure):
    _fields_ = [("active_blocks", C.c_int64), ("computed_tiles", C.c_int64), ("empty_qblocks", C.c_int64),
                ("work_items", C.c_int32), ("selected_units", C.c_int32), ("pairing", C.c_int32),
                ("split_items", C.c_int32), ("split_slots", C.c_int32), ("split_cap", C.c_int32),
                ("workers", C.c_int32), ("reserved", C.c_int32)]


class AttnDesc(C.Structure):
    _fields_ = [("dtype", C.c_int32), ("batch", C.c_int32), ("heads", C.c_int32),
                ("seq", C.c_int32), ("head_dim", C.c_int32), ("block_size", C.c_int32),
                ("causal", C.c_int32), ("mask_batch", C.c_int32), ("mask_heads", C.c_int32),
                ("scale", C.c_float),
                ("q_stride", C.c_int64 * 3), ("k_stride", C.c_int64 * 3),
                ("v_stride", C.c_int64 * 3), ("o_stride", C.c_int64 * 3)]


# name -> (restype, argtypes)
_VP, _SZ, _I32, _I64, _F = C.c_void_p, C.c_size_t, C.c_int32, C.c_int64, C.c_float
_SIGS = {
    "xsake_abi_version": (C.c_int, []),
    "xsake_last_error": (C.c_char_p, []),
    "xsake_device_error": (C.c_int, [_VP, C.POINTER(_I32)]),
    "xsake_mask_plan_bytes": (C.c_int, [C.POINTER(MaskDims), C.POINTER(_SZ)]),
    "xsake_mask_compile": (C.c_int, [C.POINTER(MaskDims), _VP, _VP, _SZ, _VP]),
    "xsake_mask_compile_ex": (C.c_int, [C.POINTER(MaskDims), C.POINTER(PlanOptions), _VP, _VP, _SZ, _VP]),
    "xsake_mask_plan_stats": (C.c_int, [_VP, _VP, C.POINTER(_I64)]),
    "xsake_mask_plan_info": (C.c_int, [_VP, _VP, C.POINTER(PlanInfo)]),
    "xsake_attn_fwd_workspace_size": (C.c_int, [C.POINTER(AttnDesc), C.POINTER(_SZ)]),
    "xsake_attn_fwd": (C.c_int, [C.POINTER(AttnDesc), _VP, _VP, _VP, _VP, _VP, _VP, _VP, _SZ, _VP]),
    "xsake_attn_bwd_workspace_size": (C.c_int, [C.POINTER(AttnDesc), C.POINTER(_SZ)]),
    "xsake_attn_bwd": (C.c_int, [C.POINTER(AttnDesc), _VP, _VP, _VP, _VP, _VP, _VP, _VP, _VP, _VP,
                                 _VP, _VP, _SZ, _VP]),
    "xsake_softmax_fwd": (C.c_int, [_I32, _I64, _I64, _VP, _VP, _VP]),
    "xsake_softmax_bwd": (C.c_int, [_I32, _I64, _I64, _VP, _VP, _VP, _VP]),
    "xsake_layernorm_fwd": (C.c_int, [_I32, _I64, _I64, _VP, _VP, _VP, _F, _VP, _VP, _VP, _VP]),
    "xsake_layernorm_bwd_workspace_size": (C.c_int, [_I64, _I64, C.POINTER(_SZ)]),
    "xsake_xent_fwd": (C.c_int, [_I32, _I64, _I64, _I64, _VP, _VP, _I64, _VP, _VP, _VP]),
    "xsake_xent_bwd": (C.c_int, [_I32, _I64, _I64, _I64, _VP, _VP, _I64, _VP, _VP, _VP, _VP]),
    "xsake_layernorm_bwd": (C.c_int, [_I32, _I64, _I64, _VP, _VP, _VP, _VP, _VP, _VP, _VP, _VP,
                                      _VP, _SZ, _VP]),
    "xsake_entropy_workspace_size": (C.c_int, [_I64, _I64, _I64, C.POINTER(_SZ)]),
    "xsake_entropy_rows": (C.c_int, [_VP, _I64, _I64, _I64, _I64, _VP, _VP, _SZ, _VP]),
    "xsake_entropy_rows_noalloc": (C.c_int, [_VP, _I64, _I64, _I64, _I64, _VP, _VP]),
    "xsake_attn_probs": (C.c_int, [C.POINTER(AttnDesc), _VP, _VP, _VP, _VP, _VP]),
    "xsake_attn_probs_workspace_size": (C.c_int, [C.POINTER(AttnDesc), C.POINTER(_SZ)]),
    "xsake_attn_probs_ex": (C.c_int, [C.POINTER(AttnDesc), _VP, _VP, _VP, _VP, _VP, _SZ, _VP]),
    "xsake_attn_entropy": (C.c_int, [C.POINTER(AttnDesc), _VP, _VP, _VP, _VP, _VP, _SZ, _VP]),
    "xsake_entropy_qk_workspace_size": (C.c_int, [_I64, _I64, _I64, C.POINTER(_SZ)]),
    "xsake_entropy_qk": (C.c_int, [_I32, _VP, _VP, _I64, _I64, _I64, _I64, _F, _VP, _VP, _SZ, _VP]),
    "xsake_comm_unique_id": (C.c_int, [_VP]),
    "xsake_comm_init": (C.c_int, [_VP, C.c_int, C.c_int, C.POINTER(_VP)]),
    "xsake_comm_init_ex": (C.c_int, [_VP, C.c_int, C.c_int, C.c_int, C.POINTER(_VP)]),
    "xsake_comm_wait": (C.c_int, [_VP, _VP, C.c_int]),
    "xsake_comm_allreduce_sum_f64": (C.c_int, [_VP, _VP, _SZ, _VP]),
    "xsake_comm_destroy": (C.c_int, [_VP]),
}

_lib = None
_lock = threading.Lock()


def exported_symbols():
    return sorted(_SIGS)


def load():
    """Load the library (once).  Raises XsakeError when it is missing or incompatible."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(LIB_PATH):
            raise XsakeError(XSAKE_ECUDA, f"{LIB_PATH} is missing; build it with "
                                          "`python -m xsake_b200.build`")
        lib = C.CDLL(LIB_PATH)
        for name, (res, args) in _SIGS.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        v = lib.xsake_abi_version()
        if v != ABI_VERSION:
            raise XsakeError(XSAKE_EUNSUPPORTED, f"ABI version {v}, expected {ABI_VERSION}")
        _lib = lib
        return lib


def check(status: int):
    if status != XSAKE_OK:
        msg = load().xsake_last_error().decode(errors="replace")
        if status in (XSAKE_EINVAL,):
            raise ValueError(f"xsake: {msg}")
        raise XsakeError(status, msg)


def device_error(stream) -> int:
    code = C.c_int32(0)
    check(load().xsake_device_error(stream, C.byref(code)))
    return code.value
