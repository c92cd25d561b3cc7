"""ctypes loader for libvdttfs.so (the C ABI declared in include/vdttfs.h).

The engine is native code only: if the library is missing this raises instead
of falling back to anything else.
"""
from __future__ import annotations

import ctypes as C
import os

PKG_DIR = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIB_PATH = os.path.join(PKG_DIR, "libvdttfs.so")

VDT_OK = 0


class VdtError(RuntimeError):
    def __init__(self, status: int, what: str, detail: str):
        super().__init__(f"{what}: status {status} ({detail})")
        self.status = status


class TimeCfg(C.Structure):
    _fields_ = [("T", C.c_int), ("delta", C.c_int), ("fire_start", C.c_float),
                ("vth_init", C.c_float), ("inf_time", C.c_float), ("lut_mode", C.c_int),
                ("decay_len", C.c_int), ("lut_source", C.c_int)]


class LayerDesc(C.Structure):
    _fields_ = [("kind", C.c_int), ("k", C.c_int), ("pad", C.c_int),
                ("pool_after", C.c_int), ("out", C.c_int)]


class NetDesc(C.Structure):
    _fields_ = [("in_h", C.c_int), ("in_w", C.c_int), ("in_c", C.c_int),
                ("tc_in", C.c_float), ("td_in", C.c_float), ("encoder", C.c_int),
                ("readout", C.c_int)]


class DvsDesc(C.Structure):
    _fields_ = [("in_c", C.c_int), ("H", C.c_int), ("W", C.c_int), ("T", C.c_int), ("delta", C.c_int),
                ("c1", C.c_int), ("c2", C.c_int), ("c3", C.c_int), ("k", C.c_int), ("hidden", C.c_int),
                ("classes", C.c_int), ("decay_conv", C.c_float), ("th_conv", C.c_float),
                ("decay_fc", C.c_float), ("th_fc", C.c_float)]


# every function the header declares: name -> (restype, argtypes)
_vp, _fp, _ip = C.c_void_p, C.POINTER(C.c_float), C.POINTER(C.c_int)
SIGNATURES = {
    "vdt_version": (C.c_char_p, []),
    "vdt_strerror": (C.c_char_p, [C.c_int]),
    "vdt_last_error": (C.c_char_p, []),
    "vdt_model_load_blob": (C.c_int, [C.c_void_p, C.c_size_t, C.POINTER(LayerDesc), C.c_int,
                                      C.POINTER(NetDesc), C.POINTER(TimeCfg), C.c_int,
                                      C.POINTER(C.c_void_p)]),
    "vdt_model_load_dvs_flat": (C.c_int, [C.c_void_p, C.c_size_t, C.POINTER(DvsDesc), C.c_int,
                                          C.POINTER(C.c_void_p)]),
    "vdt_model_destroy": (None, [_vp]),
    "vdt_model_info": (C.c_int, [_vp, _ip, _ip, C.POINTER(C.c_size_t)]),
    "vdt_model_luts": (C.c_int, [_vp, C.c_int, _vp, _vp]),
    "vdt_ctx_create": (C.c_int, [_vp, C.c_int, _vp, C.POINTER(C.c_void_p)]),
    "vdt_ctx_destroy": (None, [_vp]),
    "vdt_ctx_set_graphs": (C.c_int, [_vp, C.c_int]),
    "vdt_ctx_set_counting": (C.c_int, [_vp, C.c_int]),
    "vdt_ctx_counters": (C.c_int, [_vp, C.POINTER(C.c_ulonglong), C.POINTER(C.c_ulonglong)]),
    "vdt_ctx_layer_counters": (C.c_int, [_vp, C.c_int, _vp, _vp]),
    "vdt_ctx_set_profiling": (C.c_int, [_vp, C.c_int]),
    "vdt_ctx_layer_times": (C.c_int, [_vp, C.c_int, _vp, _vp, _vp, _ip]),
    "vdt_infer": (C.c_int, [_vp, _vp, C.c_int, C.c_int, _vp, _vp]),
    "vdt_infer_host": (C.c_int, [_vp, _vp, C.c_int, C.c_int, _vp, _vp]),
    "vdt_infer_host_batches": (C.c_int, [_vp, C.c_int, _vp, C.c_int, C.c_int, _vp, _vp]),
    "vdt_infer_trace": (C.c_int, [_vp, _vp, C.c_int, C.c_int, C.POINTER(C.c_void_p), _vp, _vp]),
    "vdt_build_luts": (C.c_int, [C.c_int, C.c_int, C.c_float, C.c_float, C.c_float, C.c_float,
                                 C.c_float, _vp, _vp, _vp]),
    "vdt_encode": (C.c_int, [_vp, _vp, C.c_int64, C.c_int, C.c_float, C.c_float, C.c_int,
                             C.c_float, _vp]),
    "vdt_bucketize": (C.c_int, [_vp, C.c_int64, C.c_int, C.c_int, C.c_int64, C.POINTER(TimeCfg),
                                C.c_int, _vp, _vp, _vp, _vp]),
    "vdt_conv_bucketed": (C.c_int, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, C.c_int, C.c_int, C.c_int,
                                    C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int,
                                    C.c_int, C.c_int, C.POINTER(TimeCfg), _vp, _vp]),
    "vdt_layer_vmem": (C.c_int, [_vp, _vp, _vp, _vp, C.c_int, C.c_int, C.c_int,
                                 C.POINTER(TimeCfg), _vp, _vp]),
    "vdt_pool_min": (C.c_int, [_vp, _vp, C.c_int, C.c_int, C.c_int, C.c_int, C.c_float, _vp]),
    "vdt_readout": (C.c_int, [_vp, C.c_int, C.c_int, C.c_int, C.c_float, _vp, _vp]),
    "vdt_ctx_layer_kernels": (C.c_int, [_vp, C.c_int, _vp]),
    "vdt_ctx_set_layer_kernel": (C.c_int, [_vp, C.c_int, C.c_int]),
    "vdt_ctx_set_sub_batches": (C.c_int, [_vp, C.c_int]),
    "vdt_dvs_conv1_raw": (C.c_int, [_vp, _vp] + [C.c_int] * 8 + [C.c_float, C.c_float, _vp, _vp]),
    "vdt_dvs_conv_bucketed": (C.c_int, [_vp, _vp, _vp, _vp] + [C.c_int] * 8 +
                              [C.c_float, C.c_float, C.c_int, _vp, _vp]),
    "vdt_dvs_conv_dense": (C.c_int, [_vp, C.c_int, _vp] + [C.c_int] * 8 +
                           [C.c_float, C.c_float, C.c_int, _vp, _vp]),
    "vdt_dvs_pool": (C.c_int, [_vp, _vp] + [C.c_int] * 7 + [C.c_float, C.c_float, _vp]),
    "vdt_dvs_fc1_recurrent": (C.c_int, [_vp] * 5 + [C.c_int] * 5 + [C.c_float, C.c_float, _vp, _vp]),
    "vdt_dvs_fc1_scratch_bytes": (C.c_size_t, [C.c_int] * 4),
    "vdt_dvs_fc1_recurrent_ws": (C.c_int, [_vp] * 5 + [C.c_int] * 5 + [C.c_float, C.c_float, _vp, _vp,
                                                                       C.c_size_t, _vp]),
    "vdt_dvs_fc2": (C.c_int, [_vp] * 4 + [C.c_int] * 5 + [C.c_float, C.c_float, _vp, _vp]),
    "vdt_oihw_to_hwio": (C.c_int, [_vp, _vp, C.c_int, C.c_int, C.c_int, _vp]),
    "vdt_set_launch_overlap": (C.c_int, [C.c_int]),
    "vdt_measure_peaks": (C.c_int, [C.c_int, C.POINTER(C.c_double), C.POINTER(C.c_double)]),
    "vdt_noalloc_scratch_bytes": (C.c_size_t, []),
    "vdt_conv_layer_noalloc": (C.c_int, [_vp, C.c_int, _vp, _vp, _vp, _vp, C.c_int, C.c_int,
                                         C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int,
                                         C.c_int, C.c_int, C.c_int, C.POINTER(TimeCfg), _vp, _vp]),
}

_lib = None


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"{LIB_PATH} is not built (make -C vd-ttfs_b200); "
                               "the engine has no non-native fallback")
        L = C.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            f = getattr(L, name)
            f.restype = res
            f.argtypes = args
        _lib = L
    return _lib


def check(status: int, what: str):
    if status != VDT_OK:
        L = lib()
        detail = L.vdt_last_error().decode() or L.vdt_strerror(status).decode()
        raise VdtError(status, what, detail)
