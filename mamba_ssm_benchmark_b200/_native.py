"""ctypes binding of libssm_b200.so, the C ABI declared in include/ssm_b200.h.

This module only loads the library and marshals torch tensors into the ABI's plain
(pointer, dtype, strides) views.  There is no fallback: if the library has not been built
(``python -m mamba_ssm_benchmark_b200.build``) every op raises ``NativeLibraryError``.
"""

import ctypes
import os
import threading

import torch

LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "_C", "libssm_b200.so")

SSM_OK, SSM_ERR_INVALID, SSM_ERR_DTYPE, SSM_ERR_WORKSPACE, SSM_ERR_CUDA, SSM_ERR_UNSUPPORTED = range(6)
SSM_F32, SSM_BF16 = 0, 1
METHODS = {"zoh": 0, "euler": 1, "bilinear": 2}
DTYPES = {torch.float32: SSM_F32, torch.bfloat16: SSM_BF16}
ABI_VERSION = 5

# Every symbol include/ssm_b200.h declares (checked by the tests).
EXPORTED = (
    "ssm_abi_version", "ssm_last_error_message", "ssm_read_device_error",
    "ssm_scan_fwd_workspace_size", "ssm_scan_fwd", "ssm_scan_bwd_workspace_size", "ssm_scan_bwd",
    "ssm_scan_fwd_summary", "ssm_scan_fwd_finish", "ssm_state_update", "ssm_scan_bwd_noalloc",
    "ssm_scan_bwd_summary", "ssm_conv1d_fwd", "ssm_conv1d_bwd_workspace_size", "ssm_conv1d_bwd",
    "selective_scan_fwd", "selective_scan_bwd", "selective_state_update", "ssm_scan_fwd_ex", "ssm_scan_bwd_ex",
    "ssm_scan_bwd_plan", "ssm_compose_shards",
)


class NativeLibraryError(ImportError):
    """libssm_b200.so is missing or unusable; the package has no non-CUDA path."""


class SsmView(ctypes.Structure):
    """ssm_view: a (B, rows, cols) tensor with unit stride along cols."""
    _fields_ = [("ptr", ctypes.c_void_p), ("dtype", ctypes.c_int32), ("reserved", ctypes.c_int32),
                ("batch_stride", ctypes.c_int64), ("row_stride", ctypes.c_int64)]


class SsmDeltaOpts(ctypes.Structure):
    """ssm_delta_opts: delta = softplus(delta + bias) inside the scan; dbias out of the backward."""
    _fields_ = [("bias", ctypes.c_void_p), ("softplus", ctypes.c_int32), ("reserved", ctypes.c_int32),
                ("dbias", ctypes.c_void_p)]


_V = SsmView
_P = ctypes.c_void_p
_I64 = ctypes.c_int64
_I32 = ctypes.c_int32
_SZ = ctypes.c_size_t

_SIGNATURES = {
    "ssm_abi_version": (ctypes.c_int, []),
    "ssm_last_error_message": (ctypes.c_char_p, []),
    "ssm_read_device_error": (ctypes.c_int, [ctypes.POINTER(ctypes.c_int32)]),
    "ssm_scan_fwd_workspace_size": (ctypes.c_int, [_I64, _I64, _I64, _I64, ctypes.POINTER(_SZ)]),
    "ssm_scan_bwd_workspace_size": (ctypes.c_int, [_I64, _I64, _I64, _I64, ctypes.POINTER(_SZ)]),
    "ssm_scan_bwd_plan": (ctypes.c_int, [_I64, _I64, _I64, _I64, _I32, ctypes.POINTER(_I32), ctypes.POINTER(_I32)]),
    "ssm_compose_shards": (ctypes.c_int, [_I32, _I64, _I64, _I64, _P, _P, _I64, _P, _I32, _P, _P, _P]),
    "ssm_scan_fwd": (ctypes.c_int, [_I64, _I64, _I64, _I64, _I32, _V, _V, _P, _V, _V, _P, _V, _P,
                                    _V, _V, _P, _P, _P, _SZ, _P]),
    "ssm_scan_fwd_summary": (ctypes.c_int, [_I64, _I64, _I64, _I64, _I32, _V, _V, _P, _V, _P, _P,
                                            _P, _SZ, _P]),
    "ssm_scan_fwd_finish": (ctypes.c_int, [_I64, _I64, _I64, _I64, _I32, _V, _V, _P, _V, _V, _P, _V, _P,
                                           _V, _V, _P, _P, _P, _SZ, _P]),
    "ssm_scan_bwd": (ctypes.c_int, [_I64, _I64, _I64, _I64, _I32, _V, _V, _P, _V, _V, _P, _V, _P,
                                    _P, _V, _V, _P, _V, _V, _P, _V, _V, _P, _V, _P, _P, _SZ, _P]),
    "ssm_state_update": (ctypes.c_int, [_I64, _I64, _I64, _I32, _P, _V, _V, _P, _V, _V, _P, _V, _V, _P]),
    "ssm_scan_bwd_summary": (ctypes.c_int, [_I64, _I64, _I64, _I64, _I32, _V, _P, _V, _V, _V, _P, _P, _P, _SZ,
                                            _P]),
    "ssm_conv1d_fwd": (ctypes.c_int, [_I64, _I64, _I64, _I64, _V, _P, _P, _P, _I32, _V, _P, _P]),
    "ssm_conv1d_bwd_workspace_size": (ctypes.c_int, [_I64, _I64, _I64, _I64, ctypes.POINTER(_SZ)]),
    "ssm_conv1d_bwd": (ctypes.c_int, [_I64, _I64, _I64, _I64, _V, _P, _P, _I32, _V, _V, _P, _P, _P, _SZ, _P]),
    "ssm_scan_bwd_noalloc": (ctypes.c_int, [_I64, _I64, _I64, _I64, _I32, _V, _V, _P, _V, _V, _P, _V, _P,
                                            _P, _V, _V, _P, _V, _V, _P, _V, _V, _P, _V, _P, _P]),
}

_OPTS = ctypes.POINTER(SsmDeltaOpts)
_SIGNATURES["ssm_scan_fwd_ex"] = (ctypes.c_int, _SIGNATURES["ssm_scan_fwd"][1][:17] + [_OPTS] +
                                  _SIGNATURES["ssm_scan_fwd"][1][17:])
_SIGNATURES["ssm_scan_bwd_ex"] = (ctypes.c_int, _SIGNATURES["ssm_scan_bwd"][1][:25] + [_OPTS] +
                                  _SIGNATURES["ssm_scan_bwd"][1][25:])
# the reference-named aliases share their counterparts' signatures
_SIGNATURES["selective_scan_fwd"] = _SIGNATURES["ssm_scan_fwd"]
_SIGNATURES["selective_scan_bwd"] = _SIGNATURES["ssm_scan_bwd"]
_SIGNATURES["selective_state_update"] = _SIGNATURES["ssm_state_update"]

_lib = None
_lock = threading.Lock()


def lib():
    """Loads libssm_b200.so once and declares every signature."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise NativeLibraryError(
                    f"{LIB_PATH} is not built; run `python -m mamba_ssm_benchmark_b200.build` "
                    "(this package has no non-CUDA fallback)")
            try:
                handle = ctypes.CDLL(LIB_PATH)
            except OSError as e:
                raise NativeLibraryError(f"cannot load {LIB_PATH}: {e}") from e
            for name, (res, args) in _SIGNATURES.items():
                fn = getattr(handle, name)
                fn.restype, fn.argtypes = res, args
            if handle.ssm_abi_version() != ABI_VERSION:
                raise NativeLibraryError(f"{LIB_PATH} has ABI {handle.ssm_abi_version()}, expected {ABI_VERSION}")
            _lib = handle
    return _lib


def check(rc, what):
    """Turns a non-OK status into the exception the reference raises for the same problem."""
    if rc == SSM_OK:
        return
    msg = (lib().ssm_last_error_message() or b"").decode(errors="replace")
    if rc in (SSM_ERR_INVALID, SSM_ERR_DTYPE):
        raise ValueError(f"{what}: {msg}")
    raise RuntimeError(f"{what}: {msg} (status {rc})")


NULL_VIEW = SsmView(None, 0, 0, 0, 0)


def view3(t):
    """(B, rows, cols) tensor with unit inner stride -> ssm_view."""
    if t is None:
        return NULL_VIEW
    assert t.dim() == 3 and (t.stride(2) == 1 or t.shape[2] == 1), "inner dimension must be contiguous"
    return SsmView(t.data_ptr(), DTYPES[t.dtype], 0, t.stride(0), t.stride(1))


def view2(t):
    """(B, cols) tensor with unit inner stride -> ssm_view with one row per batch entry."""
    if t is None:
        return NULL_VIEW
    assert t.dim() == 2 and (t.stride(1) == 1 or t.shape[1] == 1), "inner dimension must be contiguous"
    return SsmView(t.data_ptr(), DTYPES[t.dtype], 0, t.stride(0), 0)


def delta_opts(bias, softplus, dbias=None):
    """ssm_delta_opts for the _ex entry points, or None (plain delta)."""
    if not softplus:
        return None
    return ctypes.byref(SsmDeltaOpts(None if bias is None else bias.data_ptr(), 1, 0,
                                     None if dbias is None else dbias.data_ptr()))


def ptr(t):
    return None if t is None else t.data_ptr()


def stream_of(device):
    return torch.cuda.current_stream(device).cuda_stream


def conv_workspace_bytes(B, L, D, K):
    n = _SZ(0)
    check(lib().ssm_conv1d_bwd_workspace_size(B, L, D, K, ctypes.byref(n)), "ssm_conv1d_bwd_workspace_size")
    return n.value


def fwd_workspace_bytes(B, L, D, N):
    n = _SZ(0)
    check(lib().ssm_scan_fwd_workspace_size(B, L, D, N, ctypes.byref(n)), "ssm_scan_fwd_workspace_size")
    return n.value


def bwd_plan(B, L, D, N, dtype):
    """(segments, steps per segment) of the backward's sequence split on the current device."""
    S, n = _I32(0), _I32(0)
    code = SSM_BF16 if dtype == torch.bfloat16 else SSM_F32
    check(lib().ssm_scan_bwd_plan(B, L, D, N, code, ctypes.byref(S), ctypes.byref(n)), "ssm_scan_bwd_plan")
    return S.value, n.value


def bwd_workspace_bytes(B, L, D, N):
    n = _SZ(0)
    check(lib().ssm_scan_bwd_workspace_size(B, L, D, N, ctypes.byref(n)), "ssm_scan_bwd_workspace_size")
    return n.value


def read_device_error():
    """Reads and clears the device error word (synchronises)."""
    v = ctypes.c_int32(0)
    check(lib().ssm_read_device_error(ctypes.byref(v)), "ssm_read_device_error")
    return v.value
