"""CPU oracle for the canonical W4G64 QuantLinear forward (numpy).

TEST INFRASTRUCTURE ONLY. This module is the checker for the CUDA backend:
only ``tests/``, ``__graft_entry__.smoke()`` and the ``cpu_baseline`` /
``--impl reference`` legs of ``bench.py`` may import it. The product path
(the ``qwen2-int4-systems_b200`` package) never calls it and has no CPU
fallback.

Each function restates, in numpy, the algorithm of the reference project
ryanyue-16/qwen2-int4-systems (paths relative to that project's root):

* ``pack_int4`` / ``unpack_int4``      -> src/qwen_int4/quantization.py:30-84
  (CANONICAL branch: element 2i in the low nibble, 2i+1 in the high nibble,
  4-bit two's complement).
* ``quantize_symmetric_rtn``           -> src/qwen_int4/quantization.py:87-111
* ``quantize_asymmetric_rtn``          -> src/qwen_int4/quantization.py:114-162
* ``dequantize_groupwise``             -> src/qwen_int4/quantization.py:221-258
* ``linear``                           -> src/qwen_int4/backends.py:73-98
  (``torch_reference_linear``: full FP32 dequantisation, FP32 matmul, FP32
  bias add, final cast to the activation dtype).

numpy has no bfloat16, so bf16 values travel as uint16 bit patterns;
``bf16_to_f32`` / ``f32_to_bf16_bits`` give the exact conversions (the latter
rounds to nearest-even like ``torch.Tensor.to(torch.bfloat16)``).

Parity is pinned: ``tests/test_oracle_golden.py`` checks every function here
against fixtures produced by running the reference itself
(``tests/golden/make_golden.py``) and against the known-answer vectors of the
reference's own tests.
"""

from __future__ import annotations

import numpy as np

GROUP_SIZE = 64


# ---------------------------------------------------------------------------
# bf16 / fp16 helpers
# ---------------------------------------------------------------------------

def bf16_to_f32(bits: np.ndarray) -> np.ndarray:
    """Exact widening of bf16 bit patterns (uint16) to float32."""
    bits = np.asarray(bits, dtype=np.uint16)
    return (bits.astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16_bits(values: np.ndarray) -> np.ndarray:
    """Round float32 to bf16 (nearest, ties to even); returns uint16 bits."""
    v = np.ascontiguousarray(values, dtype=np.float32)
    u = v.view(np.uint32).astype(np.uint64)
    nan = np.isnan(v)
    rounded = (u + 0x7FFF + ((u >> 16) & 1)) >> 16
    out = rounded.astype(np.uint16)
    out[nan] = 0x7FC0
    return out


def round_to_dtype(values: np.ndarray, dtype: str) -> np.ndarray:
    """Cast float32 values to ``dtype`` and back, as the final ``.to(x.dtype)``."""
    values = np.asarray(values, dtype=np.float32)
    if dtype == "f32":
        return values.copy()
    if dtype == "f16":
        return values.astype(np.float16).astype(np.float32)
    if dtype == "bf16":
        return bf16_to_f32(f32_to_bf16_bits(values))
    raise ValueError(f"unknown dtype {dtype!r}")


# ---------------------------------------------------------------------------
# Packing (reference quantization.py:30-84, CANONICAL branch)
# ---------------------------------------------------------------------------

def pack_int4(codes: np.ndarray) -> np.ndarray:
    """Pack signed INT4 codes: even index -> low nibble, odd -> high nibble."""
    flat = np.asarray(codes).reshape(-1).astype(np.int16)
    if flat.size % 2:
        raise ValueError("INT4 packing requires an even number of elements")
    if flat.size and (flat.min() < -8 or flat.max() > 7):
        raise ValueError("signed INT4 codes must be in [-8, 7]")
    low = flat[0::2] & 0x0F
    high = flat[1::2] & 0x0F
    return (low | (high << 4)).astype(np.uint8)


def unpack_int4(packed: np.ndarray, elements: int | None = None) -> np.ndarray:
    """Decode bytes to int8 codes in [-8, 7], element 2i from the low nibble."""
    byte = np.asarray(packed, dtype=np.uint8).reshape(-1)
    nibbles = np.empty(byte.size * 2, dtype=np.uint8)
    nibbles[0::2] = byte & 0x0F
    nibbles[1::2] = byte >> 4
    # 4-bit two's complement: (n ^ 8) - 8 maps 0..7 -> 0..7 and 8..15 -> -8..-1.
    codes = ((nibbles ^ 0x08).astype(np.int16) - 8).astype(np.int8)
    if elements is not None:
        if elements < 0 or elements > codes.size:
            raise ValueError(
                f"invalid element count {elements} for {codes.size} decoded values"
            )
        codes = codes[:elements]
    return codes


# ---------------------------------------------------------------------------
# Quantisers (data generators; reference quantization.py:87-162)
# ---------------------------------------------------------------------------

def quantize_symmetric_rtn(weight: np.ndarray, group_size: int = GROUP_SIZE):
    """Per-row, per-K-group symmetric RTN to codes in [-7, 7].

    Returns ``(packed uint8 [N*K/2, 1], scales float16 [N, K/group])``.
    """
    w = np.asarray(weight, dtype=np.float32)
    if w.ndim != 2:
        raise ValueError(f"weight must be 2D, got shape={w.shape}")
    n, k = w.shape
    if k % group_size:
        raise ValueError(f"in_features={k} is not divisible by group_size={group_size}")
    grouped = w.reshape(n, k // group_size, group_size)
    scale = (np.abs(grouped).max(axis=-1) / np.float32(7.0)).astype(np.float32)
    scale = np.where(scale == 0, np.float32(1.0), scale).astype(np.float32)
    codes = np.clip(np.round(grouped / scale[..., None]), -7, 7).astype(np.int8)
    return pack_int4(codes).reshape(-1, 1), scale.astype(np.float16)


def quantize_asymmetric_rtn(weight: np.ndarray, group_size: int = GROUP_SIZE):
    """Per-row, per-K-group asymmetric RTN with packed signed zero points.

    Logical codes and zeros live in [0, 15]; both are stored shifted by -8 as
    signed INT4. Returns ``(packed [N*K/2,1], scales f16 [N,G], zeros
    [(N*G+1)//2, 1])``; an odd ``N*G`` is padded with one zero nibble.
    """
    w = np.asarray(weight, dtype=np.float32)
    if w.ndim != 2:
        raise ValueError(f"weight must be 2D, got shape={w.shape}")
    n, k = w.shape
    if k % group_size:
        raise ValueError(f"in_features={k} is not divisible by group_size={group_size}")
    grouped = w.reshape(n, k // group_size, group_size)
    zero_f = np.float32(0.0)
    lo = np.minimum(grouped.min(axis=-1), zero_f)
    hi = np.maximum(grouped.max(axis=-1), zero_f)
    scale = (np.maximum(hi - lo, np.float32(1e-5)) / np.float32(15.0)).astype(np.float32)
    uzero = np.clip(np.round(-lo / scale), 0, 15).astype(np.int16)
    ucode = np.round(grouped / scale[..., None]).astype(np.float32)
    ucode = np.clip(ucode + uzero[..., None].astype(np.float32), 0, 15)
    scodes = (ucode.astype(np.int16) - 8).astype(np.int8)
    szeros = (uzero - 8).astype(np.int8).reshape(-1)
    if szeros.size % 2:
        szeros = np.concatenate([szeros, np.zeros(1, dtype=np.int8)])
    return (
        pack_int4(scodes).reshape(-1, 1),
        scale.astype(np.float16),
        pack_int4(szeros).reshape(-1, 1),
    )


# ---------------------------------------------------------------------------
# Dequantisation and the linear forward
# ---------------------------------------------------------------------------

def dequantize_groupwise(
    qweight: np.ndarray,
    scales: np.ndarray,
    *,
    out_features: int,
    in_features: int,
    group_size: int = GROUP_SIZE,
    zeros: np.ndarray | None = None,
) -> np.ndarray:
    """FP32 weight ``W[n, k] = (code[n,k] - zero[n,g]) * f32(scale[n,g])``.

    ``g = k // group_size``; zero ``n*G + g`` is nibble ``(n*G+g) & 1`` of byte
    ``(n*G+g) >> 1``. The product of a small integer and an fp16 value is
    exact in fp32, so this result is bit-exact by construction.
    """
    if in_features % group_size:
        raise ValueError(
            f"in_features={in_features} is not divisible by group_size={group_size}"
        )
    groups = in_features // group_size
    scales = np.asarray(scales)
    if tuple(scales.shape) != (out_features, groups):
        raise ValueError(
            f"scale shape must be {(out_features, groups)}, got {tuple(scales.shape)}"
        )
    expected = out_features * in_features // 2
    if np.asarray(qweight).size != expected:
        raise ValueError(f"qweight must contain {expected} bytes, got {np.asarray(qweight).size}")
    codes = unpack_int4(qweight).reshape(out_features, groups, group_size)
    if zeros is None:
        zero_values = np.zeros((out_features, groups), dtype=np.int8)
    else:
        expected_zero = (out_features * groups + 1) // 2
        if np.asarray(zeros).size != expected_zero:
            raise ValueError(
                f"zeros must contain {expected_zero} bytes, got {np.asarray(zeros).size}"
            )
        zero_values = unpack_int4(zeros, elements=out_features * groups).reshape(
            out_features, groups
        )
    diff = codes.astype(np.float32) - zero_values.astype(np.float32)[..., None]
    weight = diff * scales.astype(np.float32)[..., None]
    return weight.reshape(out_features, in_features)


def linear(
    x: np.ndarray,
    qweight: np.ndarray,
    scales: np.ndarray,
    zeros: np.ndarray | None,
    bias: np.ndarray | None,
    *,
    out_features: int,
    in_features: int,
    group_size: int = GROUP_SIZE,
    accumulate: str = "f32",
) -> np.ndarray:
    """``(x.float() @ deq(W).T + bias.float())`` before the final dtype cast.

    ``x`` and ``bias`` are float32 arrays holding the exact values of the
    activation / bias dtype. Returns float32 ``[*x.shape[:-1], N]``; callers
    apply ``round_to_dtype`` for the cast the reference performs last.
    ``accumulate='f64'`` gives a higher-precision answer for error budgets.
    """
    x = np.asarray(x, dtype=np.float32)
    w = dequantize_groupwise(
        qweight, scales, out_features=out_features, in_features=in_features,
        group_size=group_size, zeros=zeros,
    )
    x2 = x.reshape(-1, in_features)
    if accumulate == "f64":
        out = (x2.astype(np.float64) @ w.T.astype(np.float64))
        if bias is not None:
            out = out + np.asarray(bias, dtype=np.float64)
        out = out.astype(np.float32)
    else:
        out = x2 @ w.T
        if bias is not None:
            out = out + np.asarray(bias, dtype=np.float32)
    return out.reshape(*x.shape[:-1], out_features)
