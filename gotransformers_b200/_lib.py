"""ctypes binding of libgtmoe.so (include/gtmoe.h).

The library is loaded from this package directory; a missing library is an
error (there is no CPU fallback)."""
from __future__ import annotations

import ctypes
import os
import subprocess
import threading

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libgtmoe.so")
CSRC = os.path.join(_HERE, "csrc")

FLOAT64, FLOAT32, INT8, FP4 = 0, 1, 2, 3
DTYPE_F64, DTYPE_F32, DTYPE_BF16 = 0, 1, 2
SHARED, ROUTED = 0, 1
GATE, UP, DOWN = 0, 1, 2

N_PHASES = 8
PHASES = ["router", "dispatch", "gather", "expert_gate_up", "expert_down", "combine", "ep_send", "ep_return"]

ERRORS = {
    -1: "EINVAL",
    -2: "ENODEVICE",
    -3: "ECUDA",
    -4: "ENOTREADY",
    -5: "ENOMEM",
    -6: "ETIMEOUT",
    -7: "ENCCL",
}

# Every entry point declared in include/gtmoe.h.
EXPORTS = [
    "gtmoe_version",
    "gtmoe_last_error",
    "gtmoe_create",
    "gtmoe_ep_unique_id",
    "gtmoe_create_ep",
    "gtmoe_ep_set_replicas",
    "gtmoe_destroy",
    "gtmoe_set_stream",
    "gtmoe_set_graphs",
    "gtmoe_set_router",
    "gtmoe_set_balance",
    "gtmoe_get_balance",
    "gtmoe_set_expert_layer",
    "gtmoe_forward",
    "gtmoe_last_expert_load",
    "gtmoe_update_balance",
    "gtmoe_set_timing",
    "gtmoe_read_timing",
    "gtmoe_quantize_rows",
    "gtmoe_fill_normal",
    "gtmoe_route_noalloc",
    "gtmoe_bounded_wait_selftest",
    "gtmoe_set_norm",
    "gtmoe_forward_block",
    "gtmoe_set_training",
    "gtmoe_backward",
    "gtmoe_weightfile_open",
    "gtmoe_weightfile_close",
    "gtmoe_weightfile_count",
    "gtmoe_weightfile_info",
    "gtmoe_weightfile_set_expert_layer",
    "gtmoe_weightfile_set_router",
]


class GtmoeError(RuntimeError):
    def __init__(self, code: int, message: str):
        super().__init__(f"{ERRORS.get(code, code)}: {message}")
        self.code = code


class Config(ctypes.Structure):
    """gtmoe_config."""

    _fields_ = [
        ("d_model", ctypes.c_int32),
        ("hidden", ctypes.c_int32),
        ("n_shared", ctypes.c_int32),
        ("n_routed", ctypes.c_int32),
        ("experts_per_token", ctypes.c_int32),
        ("hash_routing", ctypes.c_int32),
        ("clamped", ctypes.c_int32),
        ("weight_precision", ctypes.c_int32),
        ("clamp_limit", ctypes.c_double),
    ]


def build(jobs: int = 8) -> str:
    """Compile libgtmoe.so for sm_100a with nvcc (no GPU needed)."""
    subprocess.run(["make", "-s", "-j", str(jobs), "-C", CSRC], check=True)
    return LIB_PATH


_lock = threading.Lock()
_lib = None


def lib():
    global _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise RuntimeError(f"{LIB_PATH} is not built; run gotransformers_b200._lib.build() (needs nvcc)")
            L = ctypes.CDLL(LIB_PATH)
            vp, i32, i64, d = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_double
            L.gtmoe_version.restype = i32
            L.gtmoe_last_error.restype = ctypes.c_char_p
            L.gtmoe_create.argtypes = [ctypes.POINTER(Config), i32, ctypes.POINTER(vp)]
            L.gtmoe_ep_unique_id.argtypes = [vp]
            L.gtmoe_create_ep.argtypes = [ctypes.POINTER(Config), i32, i32, i32, vp, ctypes.POINTER(vp)]
            L.gtmoe_ep_set_replicas.argtypes = [vp, i32, vp]
            L.gtmoe_destroy.argtypes = [vp]
            L.gtmoe_destroy.restype = None
            L.gtmoe_set_stream.argtypes = [vp, vp]
            L.gtmoe_set_graphs.argtypes = [vp, i32]
            L.gtmoe_set_router.argtypes = [vp, i32, vp, vp, vp]
            L.gtmoe_set_balance.argtypes = [vp, vp]
            L.gtmoe_get_balance.argtypes = [vp, vp]
            L.gtmoe_set_expert_layer.argtypes = [vp, i32, i32, i32, i32, vp, vp, i32, i32, vp]
            L.gtmoe_forward.argtypes = [vp, vp, i32, i64, vp, vp, vp, i32, vp, vp, vp, vp]
            L.gtmoe_last_expert_load.argtypes = [vp, vp]
            L.gtmoe_update_balance.argtypes = [vp, d]
            L.gtmoe_set_timing.argtypes = [vp, i32]
            L.gtmoe_read_timing.argtypes = [vp, vp, i32, vp, vp]
            L.gtmoe_quantize_rows.argtypes = [i32, vp, i64, i32, vp, vp]
            L.gtmoe_route_noalloc.argtypes = [vp, vp, i32, i64, vp, vp, vp]
            L.gtmoe_bounded_wait_selftest.argtypes = [i32]
            L.gtmoe_fill_normal.argtypes = [vp, i32, i64, ctypes.c_uint64, ctypes.c_uint64, i64, d]
            L.gtmoe_set_norm.argtypes = [vp, vp, d]
            L.gtmoe_forward_block.argtypes = [vp, vp, i32, i64, vp, vp, i32, vp, vp, vp, vp]
            L.gtmoe_set_training.argtypes = [vp, i32]
            L.gtmoe_backward.argtypes = [vp, vp, i32, vp, i32, vp, vp]
            L.gtmoe_weightfile_open.argtypes = [ctypes.c_char_p, ctypes.POINTER(vp)]
            L.gtmoe_weightfile_close.argtypes = [vp]
            L.gtmoe_weightfile_close.restype = None
            L.gtmoe_weightfile_count.argtypes = [vp]
            L.gtmoe_weightfile_info.argtypes = [vp, i32, ctypes.POINTER(ctypes.c_char_p), ctypes.POINTER(i32),
                                                ctypes.POINTER(i32), ctypes.POINTER(i64), ctypes.POINTER(i64),
                                                ctypes.POINTER(i64)]
            L.gtmoe_weightfile_set_expert_layer.argtypes = [vp, vp, i32, i32, i32, ctypes.c_char_p, ctypes.c_char_p]
            L.gtmoe_weightfile_set_router.argtypes = [vp, vp, ctypes.c_char_p, ctypes.c_char_p]
            for name in EXPORTS:
                if name not in ("gtmoe_destroy", "gtmoe_weightfile_close"):
                    fn = getattr(L, name)
                    if fn.restype is not ctypes.c_char_p:
                        fn.restype = i32
            _lib = L
    return _lib


def check(rc: int) -> None:
    if rc != 0:
        msg = lib().gtmoe_last_error()
        raise GtmoeError(rc, msg.decode() if msg else "")
