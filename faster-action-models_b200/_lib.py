"""ctypes binding of libfam.so (the C ABI declared in include/fam.h).

The library is the product path: there is no fallback.  Loading fails with a
RuntimeError naming the missing file when ``libfam.so`` has not been built,
and every call that returns a non-zero status raises ``FamError`` carrying the
library's own message.
"""
from __future__ import annotations

import ctypes as C
import threading
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libfam.so"

FAM_OK = 0
FAM_DTYPE_BF16 = 0
FAM_DTYPE_F32 = 1
FAM_EPI_STORE = 0
FAM_EPI_PARTIAL = 1
FAM_EPI_RESIDUAL = 2
FAM_ACT_NONE = 0
FAM_ACT_GELU_TANH = 1


class FamError(RuntimeError):
    pass


class GemmDesc(C.Structure):
    _fields_ = [
        ("a", C.c_void_p), ("lda", C.c_int64),
        ("b", C.c_void_p), ("ldb", C.c_int64),
        ("m", C.c_int32), ("n", C.c_int32), ("k", C.c_int32),
        ("splits", C.c_int32), ("tile_n", C.c_int32),
        ("epilogue", C.c_int32), ("activation", C.c_int32), ("out_dtype", C.c_int32),
        ("features_on_a", C.c_int32), ("a_is_const", C.c_int32), ("b_is_const", C.c_int32),
        ("pdl", C.c_int32),
        ("out", C.c_void_p), ("out_stride_a", C.c_int64), ("out_stride_b", C.c_int64),
        ("out_stride_split", C.c_int64),
        ("bias", C.c_void_p), ("gate_w", C.c_void_p), ("gate_t", C.c_void_p),
        ("tokens_per_batch", C.c_int32), ("first_frame_tokens", C.c_int32),
        ("gate_batch_stride", C.c_int64), ("gate_group_stride", C.c_int64),
        ("scratch", C.c_void_p), ("scratch_bytes", C.c_size_t), ("split_round", C.c_int32),
        ("conv_wp", C.c_int32), ("conv_cin", C.c_int32), ("conv_a_rows", C.c_int64), ("pair", C.c_int32),
    ]


_lib = None
_lock = threading.Lock()


def _declare(lib):
    lib.fam_version.argtypes = [C.POINTER(C.c_int)] * 3
    lib.fam_last_error.argtypes = [C.c_char_p, C.c_size_t]
    lib.fam_device_status.argtypes = [C.POINTER(C.c_int), C.c_int, C.c_void_p]
    lib.fam_gemm.argtypes = [C.POINTER(GemmDesc), C.c_void_p]
    lib.fam_gemm_split_round_scratch_bytes.argtypes = [C.POINTER(C.c_size_t)]
    for name in ("fam_version", "fam_last_error", "fam_device_status", "fam_gemm", "fam_gemm_split_round_scratch_bytes"):
        getattr(lib, name).restype = C.c_int
    from . import _abi  # model-level entry points
    _abi.declare(lib)


def lib():
    """The loaded libfam.so (raises when it is missing: there is no fallback)."""
    global _lib
    if _lib is None:
        with _lock:
            if _lib is None:
                if not LIB_PATH.exists():
                    raise RuntimeError(
                        f"libfam.so not found at {LIB_PATH}; build it with "
                        "`python faster-action-models_b200/build.py` (no CPU fallback exists)")
                handle = C.CDLL(str(LIB_PATH))
                _declare(handle)
                _lib = handle
    return _lib


def last_error() -> str:
    buf = C.create_string_buffer(1024)
    lib().fam_last_error(buf, len(buf))
    return buf.value.decode(errors="replace")


def check(rc: int, what: str) -> None:
    if rc != FAM_OK:
        raise FamError(f"{what} failed (status {rc}): {last_error()}")


def version() -> tuple[int, int, int]:
    a, b, c = C.c_int(), C.c_int(), C.c_int()
    check(lib().fam_version(C.byref(a), C.byref(b), C.byref(c)), "fam_version")
    return a.value, b.value, c.value


def device_status(stream_ptr: int = 0, reset: bool = True) -> int:
    code = C.c_int()
    check(lib().fam_device_status(C.byref(code), 1 if reset else 0, C.c_void_p(stream_ptr)),
          "fam_device_status")
    return code.value
