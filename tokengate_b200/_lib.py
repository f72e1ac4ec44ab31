"""ctypes binding of the tokengate_b200 C ABI (include/tokengate_b200.h).

The shared library is the only compute path: there is no CPU or eager
fallback. If the library is missing, every call raises with the build
command, mirroring the reference loader's loud failure
(kernels/fa2bias/keybias.py:17-26).
"""
import ctypes
import os
import threading

from .build import LIB_PATH

ABI_VERSION = 1

TG_OK = 0
TG_ERR_INVALID_ARGUMENT = 1
TG_ERR_UNSUPPORTED = 2
TG_ERR_ALIGNMENT = 3
TG_ERR_CUDA = 4


class TokenGateKernelError(RuntimeError):
    """A tokengate_b200 entry point returned a non-zero status."""

    def __init__(self, status: int, message: str):
        super().__init__(f"tokengate_b200 status {status}: {message}")
        self.status = status


class TokenGateArgumentError(TokenGateKernelError, ValueError):
    """Invalid shape, count, pointer or alignment (TG_ERR_INVALID_ARGUMENT / TG_ERR_ALIGNMENT)."""


class TokenGateUnsupportedError(TokenGateKernelError, NotImplementedError):
    """A valid request the kernels do not serve (TG_ERR_UNSUPPORTED)."""


class GatherTensor(ctypes.Structure):
    """Mirror of tg_gather_tensor."""
    _fields_ = [
        ("src", ctypes.c_void_p),
        ("dst", ctypes.c_void_p),
        ("src_batch_stride", ctypes.c_int64),
        ("src_row_stride", ctypes.c_int64),
        ("src_seg_stride", ctypes.c_int64),
        ("dst_batch_stride", ctypes.c_int64),
        ("dst_row_stride", ctypes.c_int64),
        ("dst_seg_stride", ctypes.c_int64),
        ("seg_bytes", ctypes.c_int64),
        ("n_seg", ctypes.c_int32),
        ("reserved", ctypes.c_int32),
    ]


MAX_GATHER_TENSORS = 16

_I64 = ctypes.c_int64
_I32 = ctypes.c_int
_P = ctypes.c_void_p
_F = ctypes.c_float

# name -> argtypes, in header order
_SIGNATURES = {
    "tg_abi_version": [],
    "tg_find_state_span": [_P, _I64, _I64, _I64, _P, _P, _P, _P],
    "tg_last_error": [],
    "tg_device_error": [_P, ctypes.POINTER(ctypes.c_uint), _I32],
    "tg_keybias_attn_fwd": [
        _P, _I64, _I64, _I64,
        _P, _I64, _I64, _I64,
        _P, _I64, _I64, _I64,
        _P, _I64, _I64,
        _P, _I64, _I64,
        _P, _I64, _I64, _I64,
        _P, _I64, _I64,
        _I32, _I32, _I32, _I32, _I32, _I32,
        _F, _I32, _P,
    ],
    "tg_gate_score": [_P, _I64, _I64, _I32, _P, _I32, _P, _P, _P, _I64, _P],
    "tg_topk_select": [_P, _I64, _I32, _P, _P, _P, _P, _I32, _P, _I64, _P, _I64, _I32, _P, _I64, _P],
    "tg_gather_rows": [ctypes.POINTER(GatherTensor), _I32, _P, _I64, _I32, _I32, _P, _P],
    "tg_add_rmsnorm": [_P, _I64, _P, _I64, _P, _I64, _P, _I64, _P, _I64, _I32, _F, _P],
    "tg_qk_norm_rope": [_P, _I64, _I32, _P, _I64, _I32, _I64, _I32, _P, _P, _P, _P, _I64, _I64, _I32,
                        _F, _P],
    "tg_qk_norm_rope_append": [_P, _I64, _I32, _P, _I64, _I32, _P, _I64, _I64, _P, _P, _P, _P, _I64, _I64, _I32,
                               _F, _P, _P, _I64, _I64, _P, _P],
    "tg_silu_mul": [_P, _I64, _P, _I64, _I64, _I64, _P],
    "tg_gemm_swiglu": [_P, _I64, _P, _I64, _P, _I64, _I64, _I32, _I32, _P],
    "tg_gemm_qkv_rope": [_P, _I64, _P, _I64, _P, _I64, _I64, _I32, _I32, _I32, _P, _P, _P, _P, _I64, _I64,
                         _I32, _F, _P],
    "tg_branch_score": [_P, _I64, _I64, _I32, _P, _I32, _P, _P, _P, _I64, _P],
    "tg_gemm_swiglu_readout": [_P, _I64, _P, _I64, _P, _P, _P, _I64, _I32, _I32, _P],
    "tg_phase2_tables": [_P, _I64, _I32, _P, _P, _P, _I64, _P, _I32, _P, _P, _I32, _I32, _F, _F, _P, _P,
                         _P],
    "tg_decode_attn": [_P, _I64, _I64, _P, _I64, _P, _I64, _I64, _I64, _P, _I64, _I64, _I64, _P, _I64, _I64,
                       _P, _I32, _I32, _P, _I64, _I64, _P, ctypes.c_size_t, _I32, _I32, _I32, _I32, _F, _P],
    "tg_decode_attn_ex": [_P, _I64, _I64, _P, _I64, _P, _I64, _I64, _I64, _P, _I64, _I64, _I64, _P, _I64, _I64,
                          _P, _I32, _I32, _P, _P, _I64, _I64, _P, ctypes.c_size_t, _I32, _I32, _I32, _I32, _F,
                          _P],
    "tg_gemv": [_P, _I64, _P, _I64, _P, _I64, _I32, _I32, _I32, _I32, _P],
    "tg_decode_attn_workspace": [_I32, _I32, _I32, ctypes.POINTER(ctypes.c_size_t)],
    "tg_decode_attn_noalloc": [_P, _I64, _I64, _P, _I64, _P, _I64, _I64, _I64, _P, _I64, _I64, _I64, _P, _I64,
                               _I64, _P, _I32, _I32, _P, _I64, _I64, _I32, _I32, _I32, _I32, _F, _P],
}
EXPORTED = tuple(_SIGNATURES)

_lib = None
_lock = threading.Lock()


def available() -> bool:
    return os.path.exists(LIB_PATH)


def lib() -> ctypes.CDLL:
    """Load (once) and return the library; raises if it is not built."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not available():
            raise RuntimeError(
                f"tokengate_b200 kernels are not built ({LIB_PATH} missing): "
                f"build them with `python -m tokengate_b200.build` (needs nvcc)")
        handle = ctypes.CDLL(LIB_PATH)
        for name, argtypes in _SIGNATURES.items():
            fn = getattr(handle, name)
            fn.argtypes = argtypes
            fn.restype = ctypes.c_int
        handle.tg_last_error.restype = ctypes.c_char_p
        abi = handle.tg_abi_version()
        if abi != ABI_VERSION:
            raise RuntimeError(f"{LIB_PATH} is ABI {abi}, this package needs {ABI_VERSION}: "
                               f"rebuild with `python -m tokengate_b200.build --force`")
        _lib = handle
    return _lib


def check(status: int) -> None:
    if status == TG_OK:
        return
    msg = lib().tg_last_error().decode(errors="replace")
    if status in (TG_ERR_INVALID_ARGUMENT, TG_ERR_ALIGNMENT):
        raise TokenGateArgumentError(status, msg)
    if status == TG_ERR_UNSUPPORTED:
        raise TokenGateUnsupportedError(status, msg)
    raise TokenGateKernelError(status, msg)


# C-ABI calls that launched kernels since import (host-side count; each such
# call of the prefill path launches one kernel at up to 64 requests)
LAUNCH_CALLS = 0


def check_launch(status: int) -> None:
    """check() for a call that launches kernels, counted in LAUNCH_CALLS."""
    global LAUNCH_CALLS
    LAUNCH_CALLS += 1
    check(status)


def device_error(stream_handle: int = 0, clear: bool = False) -> int:
    """Bit flags recorded on the current device by kernels whose bounded waits gave up."""
    out = ctypes.c_uint(0)
    check(lib().tg_device_error(stream_handle, ctypes.byref(out), int(clear)))
    return int(out.value)
