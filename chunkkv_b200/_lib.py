"""ctypes binding of ``libchunkkv_b200.so`` (the C ABI in ``include/chunkkv_b200.h``).

There is no fallback: if the library is missing or cannot be loaded, every
call raises.  Status codes map to the exceptions the reference raises for the
same conditions (ValueError for bad arguments, NotImplementedError for
unsupported shapes, RuntimeError for CUDA / device-side failures).
"""

from __future__ import annotations

import ctypes as C
import threading
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libchunkkv_b200.so"

_p = C.c_void_p
_i32 = C.c_int32
_i64 = C.c_int64
_f32 = C.c_float
_f64 = C.c_double

# name -> argtypes (all return int status unless listed in _RESTYPES)
SIGNATURES: dict[str, list] = {
    "ckv_version": [],
    "ckv_last_error": [],
    "ckv_get_device_error": [_p],
    "ckv_rope_table": [_p, _i32, _i32, _p, _p],
    "ckv_shift_keys": [_p, _p, _i64, _i32, _i32, _i32, _p, _p],
    "ckv_apply_rope": [_p, _p, _i64, _i32, _i32, _i32, _p, _p, _p],
    "ckv_shift_keys_f32": [_p, _p, _i64, _i32, _i32, _i32, _p, _p],
    "ckv_apply_rope_f32": [_p, _p, _i64, _i32, _i32, _i32, _p, _p, _p],
    "ckv_blend_gather_paged": [_p, _i64, _p, _p, _i32, _p, _i32, _p, _p, _i32, _i32, _i32, _i32, _i32,
                               _i32, _p],
    "ckv_blend_gather_dense": [_p, _p, _p, _i32, _p, _i32, _p, _p, _i32, _i32, _i32, _i32, _i32, _p],
    "ckv_pages_write": [_p, _i64, _p, _i32, _p, _p, _i64, _i32, _i32, _i32, _p],
    "ckv_deviation_select": [_p, _p, _i64, _p, _p, _p, _i32, _p, _i32, _p, _i32, _i32, _f64, _i32, _i32,
                             _p, _p, _p, _p, _p, _p, _p, _p, _p],
    "ckv_deviation_select_noalloc": [_p, _p, _i64, _p, _p, _p, _i32, _p, _i32, _p, _i32, _i32, _f64, _i32,
                                     _i32, _p, _p, _p, _p, _p, _p, _p],
    "ckv_deviation_scores": [_p, _p, _i64, _p, _p, _p, _i32, _p, _i32, _i32, _i32, _p, _p, _p],
    "ckv_select_from_scores": [_p, _p, _p, _i32, _p, _i32, _i32, _f64, _p, _p, _p, _p, _p, _p],
    "ckv_apply_selection": [_p, _p, _p, _i32, _p, _p, _p, _p, _i32, _p, _p, _i64, _p, _p, _i32, _i32,
                            _i32, _p],
    "ckv_embed": [_p, _i32, _i32, _p, _p, _i32, _p, _p],
    "ckv_rmsnorm": [_p, _p, _p, _i32, _i32, _f32, _p],
    "ckv_add_rmsnorm": [_p, _p, _p, _p, _i32, _i32, _f32, _p],
    "ckv_linear_partial": [_p, _p, _p, _i32, _i32, _i32, _p, _p, _i32, _i32, _p],
    "ckv_gemv_residual": [_p, _p, _p, _i32, _i32, _i32, _p],
    "ckv_gemv_swiglu": [_p, _p, _p, _i32, _i32, _i32, _p],
    "ckv_gemv_qkv_rope": [_p, _p, _p, _i32, _i32, _i32, _i32, _i32, _p, _p, _i32, _p, _p, _p, _i32, _p],
    "ckv_gemv_swiglu_rmsnorm": [_p, _p, _f32, _p, _p, _i32, _i32, _i32, _p],
    "ckv_gemv_qkv_rope_rmsnorm": [_p, _p, _f32, _p, _p, _i32, _i32, _i32, _i32, _i32, _p, _p, _i32, _p, _p, _p,
                                  _i32, _p],
    "ckv_reduce_add_gather": [_p, _i32, _i32, _i32, _i32, _p, _p, _p, _p, _p, _p, C.c_uint32, _p],
    "ckv_ipc_alloc": [_i64, _p, _p],
    "ckv_ipc_open": [_p, _p],
    "ckv_ipc_close": [_p],
    "ckv_ipc_free": [_p],
    "ckv_linear": [_p, _p, _p, _p, _i32, _i32, _i32, _p],
    "ckv_linear_residual": [_p, _p, _p, _i32, _i32, _i32, _p],
    "ckv_linear_swiglu": [_p, _p, _p, _i32, _i32, _i32, _p],
    "ckv_qkv_rope": [_p, _p, _p, _i32, _i32, _i32, _i32, _i32, _i32, _i32, _p, _p, _i32, _p, _p, _p,
                     _i32, _p, _p, _p],
    "ckv_attention_workspace_size": [_i32, _i32, _i32, _i32, _i32],
    "ckv_attention_launches": [_i32, _i32, _i32, _i32, _i32, _i64],
    "ckv_attention": [_p, _p, _p, _p, _p, _i32, _i32, _i32, _i32, _i32, _f32, _p, _i64, _p],
    "ckv_gemv": [_p, _p, _p, _i32, _i32, _i32, _p],
    "ckv_log_softmax": [_p, _i32, _p, _p],
    "ckv_greedy_next": [_p, _i32, _p, _p, _p],
}
_RESTYPES = {"ckv_version": C.c_char_p, "ckv_last_error": C.c_char_p, "ckv_attention_workspace_size": C.c_int64}

CKV_OK, CKV_ERR_ARG, CKV_ERR_CUDA, CKV_ERR_DEVICE, CKV_ERR_UNSUPPORTED = range(5)
DEV_ERR_BITS = {
    0x1: "a bounded wait (mbarrier or peer counter) ran past its limit",
    0x2: "a page id outside the pool was skipped",
    0x4: "the selection kept a position that was never computed",
    0x8: "a position or index outside its range was skipped",
}

_lock = threading.Lock()
_lib: C.CDLL | None = None


class NativeLibraryError(RuntimeError):
    """The CUDA library is missing or failed to load (there is no CPU fallback)."""


def load() -> C.CDLL:
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not LIB_PATH.exists():
                raise NativeLibraryError(
                    f"{LIB_PATH.name} is not built; run chunkkv_b200._build.build() (nvcc, sm_100a)")
            try:
                lib = C.CDLL(str(LIB_PATH))
            except OSError as e:  # pragma: no cover - depends on the box
                raise NativeLibraryError(f"cannot load {LIB_PATH}: {e}") from e
            for name, argtypes in SIGNATURES.items():
                fn = getattr(lib, name)
                fn.argtypes = argtypes
                fn.restype = _RESTYPES.get(name, C.c_int)
            _lib = lib
    return _lib


def exported_symbols() -> list[str]:
    lib = load()
    return [n for n in SIGNATURES if hasattr(lib, n)]


def last_error() -> str:
    return load().ckv_last_error().decode(errors="replace")


def call(name: str, *args) -> None:
    """Call a status-returning entry point and raise on failure."""
    rc = getattr(load(), name)(*args)
    if rc == CKV_OK:
        return
    msg = f"{name}: {last_error()}"
    if rc == CKV_ERR_ARG:
        raise ValueError(msg)
    if rc == CKV_ERR_UNSUPPORTED:
        raise NotImplementedError(msg)
    raise RuntimeError(msg)


def device_error() -> int:
    """Reads and clears the device error word (synchronises the device)."""
    code = C.c_uint32(0)
    call("ckv_get_device_error", C.byref(code))
    return code.value


def check_device() -> None:
    code = device_error()
    if code:
        what = "; ".join(v for b, v in DEV_ERR_BITS.items() if code & b)
        raise RuntimeError(f"chunkkv_b200 device error 0x{code:x}: {what}")
