"""ctypes binding of ``libqi4_b200.so`` (the C ABI declared in include/qi4_b200.h).

The library is loaded from this package directory. There is no fallback:
if it is missing or cannot be loaded, every entry point raises RuntimeError.
"""

from __future__ import annotations

import ctypes
import threading
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libqi4_b200.so"

DTYPE_NONE, DTYPE_F16, DTYPE_BF16, DTYPE_F32 = -1, 0, 1, 2
ALGO_AUTO, ALGO_GEMV, ALGO_TC, ALGO_GEMV_FMA = 0, 1, 2, 3
STATUS = {
    -1: "ARGUMENT", -2: "DTYPE", -3: "SHAPE", -4: "ALIGNMENT", -5: "LAUNCH", -6: "DEVICE",
}

# Entry points and their C signatures (must match include/qi4_b200.h).
_p, _i, _i64, _sz = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_size_t
SIGNATURES = {
    "qi4_w4g64_linear": [_p, _i, _i64, _i64, _p, _p, _p, _p, _i, _p, _i64, _p],
    "qi4_w4g64_linear_ex": [_p, _i, _i64, _i64, _p, _p, _p, _p, _i, _p, _i64, _p, _i, _i],
    "qi4_w4g64_dequant_f32": [_p, _p, _p, _p, _i64, _i64, _p],
    "qi4_w4_unpack": [_p, _p, _i64, _p],
    "qi4_w4g64_linear_f32_noalloc": [_p, _i64, _i64, _p, _p, _p, _p, _i, _p, _i64, _p],
    "qi4_gemv_plan_override": [_i, _i, _i, _i],
    "qi4_gemv_mma_plan_override": [_i, _i, _i],
    "qi4_gemm_tc_plan_override": [_i, _i],
    "qi4_w4g64_linear_multi": [_p, _i, _i64, _i64, _i, _p, _p, _p, _p, _i, _p, _p, _p],
    "qi4_w4g64_gate_up_silu": [_p, _i, _i64, _i64, _p, _p, _p, _p, _p, _p, _p, _i64, _p],
    "qi4_w4g64_gate_up_silu_scatter": [_p, _i, _i64, _i64, _p, _p, _p, _p, _p, _p, _i64, _p, _i64, _i64, _p, _i,
                                       _i, ctypes.c_uint32, _p],
    "qi4_peer_flag_wait": [_p, _i, ctypes.c_uint32, ctypes.c_uint64, _p],
    "qi4_ipc_alloc": [_sz, _p, _p],
    "qi4_ipc_open": [_p, _p],
    "qi4_ipc_close": [_p],
    "qi4_ipc_free": [_p],
    "qi4_gemv_mma_plan": [_i64, _i64, _i64, _i, _i, _p],
    "qi4_device_status": [_p],
    "qi4_selftest_bounded_wait": [ctypes.c_uint64, _p],
    "qi4_chain_create": [_p, _i, _i64, _p, ctypes.POINTER(_p)],
    "qi4_chain_run": [_p, _p],
    "qi4_chain_info": [_p, _p],
    "qi4_chain_destroy": [_p],
    "qi4_gqa_decode_attention": [_p, _p, _p, _p, _p, _p, _p, _p, _i64, _i64, _i64, _p, _p, _i64, _p, _i64, _i64,
                                 _i64, _i64, ctypes.c_float, _p],
    "qi4_gqa_decode_attention_workspace": [_i64, _i64, _i64, _i64],
    "qi4_gqa_decode_attention_ex": [_p, _p, _p, _p, _p, _p, _p, _p, _i64, _i64, _i64, _p, _p, _i64, _p, _i64, _i64,
                                    _i64, _i64, ctypes.c_float, _i, _p, _sz, _p],
    "qi4_bf16_gemv_argmax": [_p, _p, _i64, _i64, _i64, _p, _p, _p],
    "qi4_bf16_gemv_argmax_ws": [_p, _p, _i64, _i64, _i64, _p, _p, _p, _p],
    "qi4_bf16_argmax_rows": [_p, _i64, _i64, _i64, _p, _p],
    "qi4_add_rmsnorm": [_p, _p, _i, _p, _p, _i64, _i64, ctypes.c_float, _p],
    "qi4_w4g64_linear_multi_norm": [_p, _i64, _i64, _i, _p, _p, _p, _p, _i, _p, _p, _p],
    "qi4_w4g64_gate_up_silu_norm": [_p, _i64, _i64, _p, _p, _p, _p, _p, _p, _p, _i64, _p],
    "qi4_last_error": [ctypes.c_char_p, _sz],
    "qi4_version": [],
}

# Return types other than the int status.
RESTYPES = {"qi4_gqa_decode_attention_workspace": ctypes.c_size_t}

CHAIN_SWIGLU = 1
ATTN_EARLY_CACHE_READ = 1


class RmsNormPrologue(ctypes.Structure):
    """``qi4_rmsnorm_prologue`` of include/qi4_b200.h."""

    _fields_ = [
        ("h_in", ctypes.c_void_p), ("delta", ctypes.c_void_p), ("delta_dtype", ctypes.c_int32),
        ("eps", ctypes.c_float), ("weight", ctypes.c_void_p), ("h_out", ctypes.c_void_p),
    ]


class ChainStage(ctypes.Structure):
    """``qi4_chain_stage`` of include/qi4_b200.h."""

    _fields_ = [
        ("nmats", ctypes.c_int32), ("flags", ctypes.c_int32), ("K", ctypes.c_int64),
        ("x", ctypes.c_void_p), ("x_dtype", ctypes.c_int32), ("bias_dtype", ctypes.c_int32),
        ("out_dtype", ctypes.c_int32), ("reserved", ctypes.c_int32),
        ("qweight", ctypes.c_void_p * 3), ("scales_f16", ctypes.c_void_p * 3), ("zeros", ctypes.c_void_p * 3),
        ("bias", ctypes.c_void_p * 3), ("out", ctypes.c_void_p * 3), ("N", ctypes.c_int64 * 3),
    ]


_lock = threading.Lock()
_lib: ctypes.CDLL | None = None


def load() -> ctypes.CDLL:
    """Load the shared library once; raise RuntimeError if it is unavailable."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not LIB_PATH.exists():
                raise RuntimeError(
                    f"B200 backend library {LIB_PATH.name} is not built; run the package's "
                    "build step (build.py) - there is no CPU fallback")
            lib = ctypes.CDLL(str(LIB_PATH))
            for name, args in SIGNATURES.items():
                fn = getattr(lib, name)
                fn.argtypes = args
                fn.restype = RESTYPES.get(name, ctypes.c_int)
            _lib = lib
    return _lib


def last_error() -> str:
    lib = load()
    buf = ctypes.create_string_buffer(1024)
    lib.qi4_last_error(buf, len(buf))
    return buf.value.decode(errors="replace")


def check(rc: int, what: str) -> None:
    """Turn a negative status into a Python exception with the library's message."""
    if rc == 0:
        return
    message = f"{what} failed ({STATUS.get(rc, rc)}): {last_error()}"
    if rc in (-1, -3, -4):
        raise ValueError(message)
    if rc == -2:
        raise TypeError(message)
    raise RuntimeError(message)
