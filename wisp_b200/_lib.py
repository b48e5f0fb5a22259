"""ctypes binding of ``libwisp_b200.so`` (the C ABI in ``include/wisp_b200.h``).

There is no fallback: importing this module without the built library raises
``ImportError`` naming the build command, and every failing call raises a
``WispError`` carrying the library's status code and message.
"""
from __future__ import annotations

import ctypes
import os

LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "lib", "libwisp_b200.so")

WISP_OK = 0
WISP_ERR_INVALID = 1
WISP_ERR_OVERFLOW = 2
WISP_ERR_BAD_EXPERT = 3
WISP_ERR_CUDA = 4
WISP_ERR_TIMEOUT = 5
WISP_ERR_NOMEM = 6
WISP_ERR_UNSUPPORTED = 7

MODE_PAGED = 0
MODE_RESIDENT = 1

CFG_ASYNC = 1
CFG_WAIT_NS = 2
CFG_DROP_PAGEINS = 4
CFG_TRACE_BUFFER = 5
CFG_TC_MIN_PAIRS = 6
CFG_COMPUTE_CLASS = 7
PREFILL_MIN_PAIRS = 513     # calls from this size always run on the tensor cores (token-major GEMMs)

_c_int32 = ctypes.c_int32
_c_int64 = ctypes.c_int64
_vp = ctypes.c_void_p
_p32 = ctypes.POINTER(ctypes.c_int32)
_p64 = ctypes.POINTER(ctypes.c_int64)
_pf = ctypes.c_void_p

# name -> (restype, argtypes); every symbol declared in include/wisp_b200.h
SIGNATURES = {
    "wisp_version": (ctypes.c_char_p, []),
    "wisp_last_error": (ctypes.c_char_p, []),
    "wisp_layer_create": (ctypes.c_int, [_c_int32, _c_int32, _c_int32, _c_int32, _c_int64, _c_int64,
                                         _vp, _vp, _c_int32, _c_int32, ctypes.POINTER(_vp)]),
    "wisp_layer_destroy": (ctypes.c_int, [_vp]),
    "wisp_layer_create_fp8": (ctypes.c_int, [_c_int32, _c_int32, _c_int32, _c_int32, _c_int32, _c_int32,
                                             _vp, _vp, _vp, _vp, _c_int32, _c_int32, ctypes.POINTER(_vp)]),
    "wisp_layer_scale_buffers": (ctypes.c_int, [_vp, ctypes.POINTER(_vp), ctypes.POINTER(_vp)]),
    "wisp_moe_forward": (ctypes.c_int, [_vp, _vp, _pf, _vp, _c_int32, _c_int32, _c_int32, _vp, _vp]),
    "wisp_route_topk": (ctypes.c_int, [_vp, _c_int32, _c_int32, _c_int32, _c_int32, _c_int32, _vp, _vp, _vp]),
    "wisp_ensure_resident": (ctypes.c_int, [_vp, _vp, _c_int32, _c_int32, _vp]),
    "wisp_pager_step": (ctypes.c_int, [_vp, _vp, _c_int32, _c_int32, _c_int32, _vp, _vp]),
    "wisp_prefetch_async": (ctypes.c_int, [_vp, _p32, _c_int32, _vp]),
    "wisp_prime_identity": (ctypes.c_int, [_vp, _vp]),
    "wisp_resize_cap": (ctypes.c_int, [_vp, _c_int32, _vp]),
    "wisp_get_state": (ctypes.c_int, [_vp, _p32, _p64, _p64, _p64, _p32, _p32]),
    "wisp_set_stats": (ctypes.c_int, [_vp, _p64]),
    "wisp_layer_buffers": (ctypes.c_int, [_vp, ctypes.POINTER(_vp), ctypes.POINTER(_vp),
                                          ctypes.POINTER(_vp)]),
    "wisp_get_telemetry": (ctypes.c_int, [_vp, _p64]),
    "wisp_get_launch_count": (ctypes.c_int, [_vp, _p64]),
    "wisp_get_last_unique_experts": (ctypes.c_int, [_vp, _p32, _c_int32, _p32]),
    "wisp_layer_sync": (ctypes.c_int, [_vp]),
    "wisp_layer_reserve": (ctypes.c_int, [_vp, _c_int32, _c_int32]),
    "wisp_cooccur_create": (ctypes.c_int, [ctypes.POINTER(_vp)]),
    "wisp_cooccur_destroy": (ctypes.c_int, [_vp]),
    "wisp_cooccur_observe_step": (ctypes.c_int, [_vp, _c_int32, _p32, _p32, _p32]),
    "wisp_cooccur_predict": (ctypes.c_int, [_vp, _c_int32, _p32, _p32, _p32, _c_int32, _c_int32, _c_int32,
                                            ctypes.c_double, _c_int32, _p32, _p32]),
    "wisp_cooccur_set_pair": (ctypes.c_int, [_vp, _c_int32, _c_int32, _c_int32, _c_int32, _c_int64]),
    "wisp_cooccur_set_marginal": (ctypes.c_int, [_vp, _c_int32, _c_int32, _c_int64]),
    "wisp_cooccur_set_steps": (ctypes.c_int, [_vp, _c_int64]),
    "wisp_cooccur_sizes": (ctypes.c_int, [_vp, _p64, _p64, _p64, _p64]),
    "wisp_cooccur_export": (ctypes.c_int, [_vp, _p64, _c_int64, _p64, _p64, _c_int64, _p64]),
    "wisp_layer_config": (ctypes.c_int, [_vp, _c_int32, _c_int64]),
    "wisp_layer_query": (ctypes.c_int, [_vp, _c_int32, ctypes.POINTER(_c_int64)]),
    "wisp_expert_compute_noalloc": (ctypes.c_int, [_c_int32, _vp, _vp, _vp, _c_int32, _vp, _vp,
                                                   _c_int32, _c_int32, _c_int32, _c_int32, _vp, _vp]),
    "wisp_ep_group_create": (ctypes.c_int, [_c_int32, _c_int32, _c_int32, _c_int32, _c_int32,
                                            ctypes.POINTER(_vp)]),
    "wisp_ep_group_ipc_handle": (ctypes.c_int, [_vp, _vp]),
    "wisp_ep_group_connect": (ctypes.c_int, [_vp, _vp]),
    "wisp_ep_group_connect_local": (ctypes.c_int, [_vp, ctypes.POINTER(_vp)]),
    "wisp_ep_group_destroy": (ctypes.c_int, [_vp]),
    "wisp_ep_group_buffers": (ctypes.c_int, [_vp, ctypes.POINTER(_vp), ctypes.POINTER(_vp),
                                             ctypes.POINTER(_vp), ctypes.POINTER(_vp)]),
    "wisp_ep_group_config": (ctypes.c_int, [_vp, _c_int64]),
    "wisp_ep_dispatch": (ctypes.c_int, [_vp, _vp, _vp, _c_int32, _vp, _c_int32, _c_int32, _c_int32, _vp]),
    "wisp_ep_receive": (ctypes.c_int, [_vp, _c_int32, _vp, _p32, _p32, _p32]),
    "wisp_ep_return": (ctypes.c_int, [_vp, _vp]),
    "wisp_ep_combine": (ctypes.c_int, [_vp, _c_int32, _c_int32, _vp, _vp]),
    "wisp_ep_sync": (ctypes.c_int, [_vp]),
}


class WispError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(msg)
        self.code = code


class WispOverflowError(WispError):
    """A single call's working set exceeds the cap; same condition (and the
    same 'sub-batch' wording) as the reference's RuntimeError at
    src/wisp/integrations/vllm/fused_moe.py:313-327."""


_lib = None


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(f"wisp_b200 native library missing at {LIB_PATH}; "
                              "build it with `python -m wisp_b200.build`")
        handle = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(handle, name)
            fn.restype = res
            fn.argtypes = args
        _lib = handle
    return _lib


def check(rc: int, what: str = "") -> None:
    if rc == WISP_OK:
        return
    msg = lib().wisp_last_error().decode(errors="replace")
    if rc == WISP_ERR_OVERFLOW:
        raise WispOverflowError(rc, f"wisp.vllm: {msg}. The forward path failed to sub-batch "
                                    f"correctly (working set exceeds cap_experts)")
    raise WispError(rc, f"{what}: {msg} (status {rc})" if what else f"{msg} (status {rc})")


def stream_ptr(stream) -> int:
    """cudaStream_t of a torch stream (0 for the legacy default stream)."""
    return int(stream.cuda_stream) if stream is not None else 0
