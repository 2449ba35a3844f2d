"""B200 (sm_100a) backend for the canonical W4G64 QuantLinear forward.

Drop-in ``b200`` backend for ryanyue-16/qwen2-int4-systems: hand-written CUDA
kernels behind the C ABI ``libqi4_b200.so`` (include/qi4_b200.h), called from
PyTorch through ctypes. The directory name is not a Python identifier, so
import it with ``importlib.import_module("qwen2-int4-systems_b200")``.
"""

from ._lib import ALGO_AUTO, ALGO_GEMV, ALGO_GEMV_FMA, ALGO_TC
from .backends import (
    SUPPORTED_BACKENDS,
    b200_w4g64_linear,
    b200_w4g64_gate_up_silu,
    b200_w4g64_linear_multi,
    dequantize_canonical_w4g64_b200,
    linear_canonical_w4g64_b200,
    set_value_checks,
    unpack_canonical_signed_int4_b200,
)
from .attention import b200_gqa_decode_attention
from .integration import register_with_reference
from .lm_head import b200_lm_head

__all__ = [
    "ALGO_AUTO", "ALGO_GEMV", "ALGO_GEMV_FMA", "ALGO_TC", "SUPPORTED_BACKENDS", "b200_gqa_decode_attention", "b200_lm_head",
    "b200_w4g64_gate_up_silu", "b200_w4g64_linear", "b200_w4g64_linear_multi",
    "dequantize_canonical_w4g64_b200", "linear_canonical_w4g64_b200",
    "register_with_reference", "set_value_checks", "unpack_canonical_signed_int4_b200",
]
