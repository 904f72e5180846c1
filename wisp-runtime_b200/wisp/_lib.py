"""ctypes binding of libwisp_b200.so (the C ABI in include/wisp_b200.h).

There is no fallback: if the library is missing or a call fails, a WispError is raised.  The library
loads without a GPU (its host-only entry points work on CPU machines); every compute entry point needs
CUDA device pointers.
"""

from __future__ import annotations

import ctypes
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.environ.get("WISP_B200_LIB", os.path.join(os.path.dirname(_HERE), "lib", "libwisp_b200.so"))

WISP_OK, WISP_ERR_INVALID, WISP_ERR_CUDA, WISP_ERR_UNSUPPORTED = 0, 1, 2, 3
STATUS_BAD_SLOT, STATUS_BAD_POS, STATUS_WAIT_TIMEOUT, STATUS_BAD_ROUTE, STATUS_RANGE = 0x1, 0x2, 0x4, 0x8, 0x10
DTYPE_F32, DTYPE_BF16, DTYPE_F16 = 0, 1, 2
MOE_NOALLOC_MAX_SCRATCH = 65536  # WISP_MOE_NOALLOC_MAX_SCRATCH: fp32 values of k*I
ARGMAX_WORKSPACE = 256  # WISP_ARGMAX_WORKSPACE: u64 entries

_P = ctypes.c_void_p
_I = ctypes.c_int
_L = ctypes.c_int64
_F = ctypes.c_float

# name -> (restype, argtypes); mirrors include/wisp_b200.h one to one
SIGNATURES = {
    "wisp_version": (_I, []),
    "wisp_last_error": (ctypes.c_char_p, []),
    "wisp_device_status": (_I, [_I, _I, ctypes.POINTER(ctypes.c_uint32)]),
    "wisp_expert_nbytes": (_L, [_L, _I, _I]),
    "wisp_quantize": (_I, [_P, _I, _L, _L, _I, _I, _P, _P]),
    "wisp_dequant": (_I, [_P, _L, _L, _P, _L, _L, _I, _I, _P, _P]),
    "wisp_unpack_codes": (_I, [_P, _L, _L, _P, _L, _L, _I, _P, _P]),
    "wisp_moe_scratch_floats": (_L, [_I, _L, _L, _I, _I]),
    "wisp_moe_decode": (_I, [_P, _L, _L, _P, _I, _P, _L, _L, _I, _I, _P, _L, _P, _P]),
    "wisp_moe_decode_variant": (_I, [_P, _L, _L, _P, _I, _P, _L, _L, _I, _I, _P, _L, _P, _I, _P]),
    "wisp_moe_decode_routed": (_I, [_P, _L, _L, _P, _I, _I, _I, _P, _L, _P, _P, _L, _L, _I, _I, _P, _L, _P, _P]),
    "wisp_moe_decode_paged": (_I, [_P, _L, _L, _P, _I, _I, _I, _P, _L, _P, _L, _P, _P, _P, _L, _L, _I, _I, _P, _L, _P, _P]),
    "wisp_moe_batched_workspace_bytes": (_L, [_I, _I, _L, _L]),
    "wisp_moe_batched": (_I, [_P, _L, _L, _P, _I, _I, _P, _L, _L, _I, _I, _P, _L, _P, _P]),
    "wisp_moe_batched_variant": (_I, [_P, _L, _L, _P, _I, _I, _P, _L, _L, _I, _I, _P, _L, _P, _I, _P]),
    "wisp_moe_gptoss_workspace_bytes": (_L, [_I, _I, _L, _L]),
    "wisp_moe_gptoss": (_I, [_P, _L, _L, _P, _P, _I, _I, _P, _L, _L, _I, _I, _P, _P, _P, _L, _P, _P]),
    "wisp_ep_dispatch": (_I, [_P, _I, _L, _P, _I, _I, _I, _L, _L, _P, _P, _P, _P]),
    "wisp_ep_combine": (_I, [_P, _I, _I, _L, _P, _P, _P, _P]),
    "wisp_ipc_alloc": (_I, [_L, ctypes.POINTER(ctypes.c_void_p), ctypes.c_char_p]),
    "wisp_ipc_open": (_I, [ctypes.c_char_p, ctypes.POINTER(ctypes.c_void_p)]),
    "wisp_ipc_close": (_I, [_P]),
    "wisp_ipc_free": (_I, [_P]),
    "wisp_ep_p2p_bytes": (_L, [_I, _L, _L]),
    "wisp_ep_dispatch_p2p": (_I, [_P, _I, _L, _P, _I, _I, _I, _I, _L, _L, _I, ctypes.POINTER(ctypes.c_void_p), _P, _P]),
    "wisp_ep_wait": (_I, [_P, _I, _L, _L, _I, _P]),
    "wisp_ep_return_p2p": (_I, [_P, _I, _I, _L, _L, _I, ctypes.POINTER(ctypes.c_void_p), _P]),
    "wisp_ep_combine_p2p": (_I, [_P, _I, _L, _L, _I, _I, _I, _P, _P, _P, _P]),
    "wisp_moe_decode_noalloc": (_I, [_P, _L, _L, _P, _I, _P, _L, _L, _I, _I, _P, _P]),
    "wisp_rope_decode": (_I, [_P, _L, _I, _P, _L, _I, _I, _P, _P, _P, _P, _P]),
    "wisp_gemv": (_I, [_P, _L, _L, _P, _P, _P, _P, _F, _P, _P, _P, _P]),
    "wisp_gemv_bias": (_I, [_P, _L, _L, _P, _P, _P, _P, _F, _P, _P, _P, _P, _P]),
    "wisp_qk_norm_rope_kv": (_I, [_P, _I, _I, _I, _P, _P, _F, _P, _P, _P, _L, _P, _P, _P, _P]),
    "wisp_qk_norm_rope_kv_rows": (_I, [_P, _I, _L, _I, _I, _I, _P, _P, _F, _P, _P, _P, _L, _P, _P, _P, _P]),
    "wisp_attn_workspace_floats": (_L, [_I, _I, _I, _L]),
    "wisp_qk_norm_rope_kv_batched": (_I, [_P, _I, _L, _I, _I, _I, _P, _P, _F, _P, _P, _P, _L, _P, _P, _P, _P]),
    "wisp_attn_batched_workspace_floats": (_L, [_I, _I, _I, _I, _L]),
    "wisp_gqa_decode_attn_batched": (_I, [_P, _I, _I, _I, _I, _P, _P, _L, _P, _I, _P, _F, _P, _L, _P, _P]),
    "wisp_attn_decode_batched": (_I, [_P, _L, _I, _I, _I, _I, _P, _P, _F, _P, _P, _P, _P, _L, _P, _I, _P, _F, _P, _L, _P, _P]),
    "wisp_gqa_decode_attn": (_I, [_P, _I, _I, _I, _P, _P, _L, _P, _F, _P, _P, _P]),
    "wisp_attn_decode": (_I, [_P, _I, _I, _I, _P, _P, _F, _P, _P, _P, _L, _P, _P, _F, _P, _P]),
    "wisp_router_topk": (_I, [_P, _I, _I, _I, _P, _L, _P, _P, _P]),
    "wisp_router_rows": (_I, [_P, _I, _L, _P, _F, _P, _P, _P, _I, _I, _I, _P, _L, _P, _P, _P, _P]),
    "wisp_router_rows_ws": (_I, [_P, _I, _L, _P, _F, _P, _P, _P, _I, _I, _I, _P, _L, _P, _P, _P, _P, _L, _P]),
    "wisp_router_workspace_bytes": (_L, [_I, _I]),
    "wisp_embed": (_I, [_P, _L, _L, _P, _P, _P]),
    "wisp_argmax": (_I, [_P, _L, _P, _P, _P]),
    "wisp_rmsnorm": (_I, [_P, _P, _P, _P, _L, _L, _F, _P, _P]),
}


class WispError(RuntimeError):
    """A libwisp_b200 entry point returned an error code."""


_lib = None


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise WispError(
                f"{LIB_PATH} is missing: build it with `python wisp-runtime_b200/build.py` "
                "(there is no fallback implementation)"
            )
        L = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype, fn.argtypes = res, args
        _lib = L
    return _lib


def check(name: str, rc: int) -> None:
    if rc != WISP_OK:
        msg = lib().wisp_last_error().decode(errors="replace")
        raise WispError(f"{name} failed ({rc}): {msg}")


def call(name: str, *args) -> None:
    check(name, getattr(lib(), name)(*args))


def device_status(device: int = 0, clear: bool = True) -> int:
    """Read (and by default clear) the device-side status word (WISP_STATUS_* bits).  Synchronises."""
    v = ctypes.c_uint32(0)
    call("wisp_device_status", device, 1 if clear else 0, ctypes.byref(v))
    return int(v.value)
