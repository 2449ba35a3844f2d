"""The ``b200`` QuantLinear backend: reference-compatible Python entry points.

Mirrors the operator API of ryanyue-16/qwen2-int4-systems (paths relative to
that project's root):

* ``b200_w4g64_linear`` has the signature of ``torch_reference_linear`` /
  ``triton_w4g64_linear`` (src/qwen_int4/backends.py:73-84,153-164) and is
  what ``QuantLinear.forward`` (src/qwen_int4/linear.py:56-72) dispatches to
  under ``backend="b200"``. It fails closed before any launch, like
  ``_validate_lpu_functional_inputs`` (src/qwen_int4/backends.py:14-70), and
  unlike the reference's Triton backend it never falls back to the PyTorch
  path: FP32 activations (the model's ``down_proj`` input, model.py:133-136)
  run on the CUDA kernels and return FP32.
* ``linear_canonical_w4g64_b200``, ``dequantize_canonical_w4g64_b200`` and
  ``unpack_canonical_signed_int4_b200`` mirror the Triton operator wrappers
  (src/qwen_int4/triton_kernels.py:206-268,149-203,119-146): same arguments,
  same error classes and message fragments.

All compute goes through ``libqi4_b200.so`` (C ABI, include/qi4_b200.h) on
the caller's current CUDA stream; nothing here computes on the CPU.
"""

from __future__ import annotations

import ctypes

import torch

from . import _lib

SUPPORTED_BACKENDS = ("b200",)
GROUP_SIZE = 64

_DTYPE_CODE = {
    torch.float16: _lib.DTYPE_F16,
    torch.bfloat16: _lib.DTYPE_BF16,
    torch.float32: _lib.DTYPE_F32,
}

_value_checks = False


def set_value_checks(enabled: bool) -> None:
    """Also reject non-finite / non-positive scales and non-finite bias.

    Off by default: the check reads the tensors back to the host (a device
    synchronisation per call), which the reference's Triton path does not do
    either. The shape, dtype, layout and device checks always run.
    """
    global _value_checks
    _value_checks = bool(enabled)


def _packing_value(packing) -> str:
    return str(getattr(packing, "value", packing))


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


# Host cost matters here: the model calls the linear ~200 times per decoded
# token. torch's raw accessors for the current device and stream skip the
# Python wrappers of torch.cuda.current_stream / current_device.
_raw_stream = getattr(torch._C, "_cuda_getCurrentRawStream", None)
_raw_device = getattr(torch._C, "_cuda_getDevice", None)


def _stream(device: torch.device) -> int:
    if _raw_stream is not None:
        return _raw_stream(device.index)
    return torch.cuda.current_stream(device).cuda_stream


def _current_device() -> int:
    return _raw_device() if _raw_device is not None else torch.cuda.current_device()


def _aligned(t: torch.Tensor, n: int = 16) -> torch.Tensor:
    """Return ``t`` or an aligned contiguous copy (the kernels use 16-byte loads)."""
    t = t.contiguous()
    if t.data_ptr() % n:
        t = t.clone()
    return t


_cuda_seen = False

# C++ fast path of b200_w4g64_linear (csrc/torch_binding.cpp): the same checks
# and launch on at::Tensor arguments, calling the C ABI directly. Built with
# the library; without it the call goes through ctypes to the same kernels.
try:
    from . import _qi4_torch as _fast
except ImportError:
    _fast = None


def _require_cuda():
    global _cuda_seen
    if not _cuda_seen:  # once a device was seen it stays (torch.cuda.is_available reads the environment)
        if not torch.cuda.is_available():
            raise RuntimeError("B200 backend requires a CUDA device; there is no CPU fallback")
        _cuda_seen = True
    return _lib.load()


def _validate_linear(x, qweight, scales, zeros, bias, out_features, in_features, group_size, packing):
    if packing != "canonical" and _packing_value(packing) != "canonical":
        raise ValueError("B200 backend supports only canonical INT4 packing")
    if group_size != GROUP_SIZE:
        raise ValueError("B200 backend supports only canonical W4G64 tensors")
    if in_features <= 0 or out_features <= 0 or in_features % GROUP_SIZE:
        raise ValueError("linear dimensions must be positive and divisible by group size 64")
    if x.ndim < 1 or x.shape[-1] != in_features:
        raise ValueError("activation feature dimension does not match QuantLinear")
    if x.dtype not in _DTYPE_CODE:
        raise TypeError("B200 backend activations must use FP16, BF16, or FP32")
    if qweight.dtype != torch.uint8 or zeros.dtype != torch.uint8:
        raise TypeError("canonical packed weights and zero points must use uint8 storage")
    if scales.dtype != torch.float16:
        raise TypeError("canonical group scales must use FP16 storage")
    groups = in_features // GROUP_SIZE
    expected_weight = out_features * in_features // 2
    expected_zero = (out_features * groups + 1) // 2
    if qweight.numel() != expected_weight:
        raise ValueError(f"qweight must contain {expected_weight} bytes, got {qweight.numel()}")
    if scales.shape != (out_features, groups):
        raise ValueError(f"scales must have shape {(out_features, groups)}, got {tuple(scales.shape)}")
    if zeros.numel() != expected_zero:
        raise ValueError(f"zeros must contain {expected_zero} bytes, got {zeros.numel()}")
    if bias is not None:
        if bias.shape != (out_features,):
            raise ValueError(f"bias must have shape {(out_features,)}, got {tuple(bias.shape)}")
        if bias.dtype not in _DTYPE_CODE:
            raise TypeError("bias must use FP16, BF16, or FP32")
    if not (x.is_cuda and qweight.is_cuda and scales.is_cuda and zeros.is_cuda and (bias is None or bias.is_cuda)):
        raise ValueError("B200 backend inputs must be CUDA tensors")
    d = x.get_device()
    if (qweight.get_device() != d or scales.get_device() != d or zeros.get_device() != d
            or (bias is not None and bias.get_device() != d)):
        raise ValueError("all B200 backend inputs must be on the same device")
    if not (qweight.is_contiguous() and scales.is_contiguous() and zeros.is_contiguous()
            and (bias is None or bias.is_contiguous())):
        for name, t in (("qweight", qweight), ("scales", scales), ("zeros", zeros), ("bias", bias)):
            if t is not None and not t.is_contiguous():
                raise ValueError(f"{name} must be contiguous")
    if _value_checks:
        if not torch.isfinite(scales).all() or torch.any(scales <= 0):
            raise ValueError("canonical group scales must be finite and strictly positive")
        if bias is not None and not torch.isfinite(bias).all():
            raise ValueError("bias values must be finite")


def _launch_linear(x2, qweight, scales, zeros, bias, out, n, algo, pdl):
    lib = _lib.load()
    device = x2.device
    if _current_device() != device.index:
        with torch.cuda.device(device):
            return _launch_linear(x2, qweight, scales, zeros, bias, out, n, algo, pdl)
    if qweight.data_ptr() % 16:
        raise ValueError("qweight storage must be 16-byte aligned for the B200 kernels")
    rc = lib.qi4_w4g64_linear_ex(
        x2.data_ptr(), _DTYPE_CODE[x2.dtype], x2.shape[0], x2.shape[1],
        qweight.data_ptr(), scales.data_ptr(), zeros.data_ptr() if zeros is not None else None,
        _ptr(bias), _DTYPE_CODE[bias.dtype] if bias is not None else _lib.DTYPE_NONE,
        out.data_ptr(), n, _stream(device), algo, 1 if pdl else 0)
    _lib.check(rc, "qi4_w4g64_linear")
    return out


def b200_w4g64_linear(
    x: torch.Tensor,
    qweight: torch.Tensor,
    scales: torch.Tensor,
    zeros: torch.Tensor,
    bias: torch.Tensor | None,
    *,
    out_features: int,
    in_features: int,
    group_size: int,
    packing,
    algo: int = _lib.ALGO_AUTO,
    pdl: bool = True,
) -> torch.Tensor:
    """Canonical W4G64 linear on the B200 kernels: ``x @ deq(W).T + bias``.

    Same contract as ``torch_reference_linear``: any leading shape, possibly
    non-contiguous activations; output dtype ``x.dtype``; FP32 accumulation
    and FP32 bias add. ``algo`` forces a kernel (``ALGO_GEMV`` / ``ALGO_TC``)
    and ``pdl`` toggles programmatic dependent launch; both default to the
    library's choice.
    """
    if (_fast is not None and algo == _lib.ALGO_AUTO and pdl and not _value_checks and group_size == GROUP_SIZE
            and (packing == "canonical" or _packing_value(packing) == "canonical")):
        return _fast.linear(x, qweight, scales, zeros, bias, out_features, in_features)
    _validate_linear(x, qweight, scales, zeros, bias, out_features, in_features, group_size, packing)
    _require_cuda()
    x2 = x.reshape(-1, in_features)
    out = torch.empty((x2.shape[0], out_features), dtype=x.dtype, device=x.device)
    if x2.shape[0]:
        _launch_linear(_aligned(x2), qweight, scales, zeros, bias, out, out_features, algo, pdl)
    return out.reshape(*x.shape[:-1], out_features)


def b200_w4g64_linear_multi(x: torch.Tensor, layers) -> list[torch.Tensor]:
    """Several canonical W4G64 linears that share the activations ``x`` (for
    example a decoder layer's q/k/v or gate/up projections), in one launch for
    decode sizes. ``layers`` holds one to three objects with the QuantLinear
    buffers and sizes (``qweight``, ``scales``, ``zeros``, ``bias``,
    ``in_features``, ``out_features``). Returns one output per layer, each as
    ``b200_w4g64_linear`` would (same dtype, shape and tolerance). No reference
    counterpart: the reference runs each QuantLinear separately.
    """
    layers = list(layers)
    if not 1 <= len(layers) <= 3:
        raise ValueError("b200_w4g64_linear_multi takes one to three layers")
    k = layers[0].in_features
    biases = [getattr(l, "bias", None) for l in layers]
    if any(l.in_features != k for l in layers):
        raise ValueError("grouped linears must share in_features")
    if len({b.dtype for b in biases if b is not None}) > 1:
        raise TypeError("grouped linears must share one bias dtype")
    for l, b in zip(layers, biases):
        _validate_linear(x, l.qweight, l.scales, l.zeros, b, l.out_features, k,
                         getattr(l, "group_size", GROUP_SIZE), getattr(l, "packing", "canonical"))
    lib = _require_cuda()
    x2 = _aligned(x.reshape(-1, k))
    outs = [torch.empty((x2.shape[0], l.out_features), dtype=x.dtype, device=x.device) for l in layers]
    if x2.shape[0]:
        device = x2.device
        if _current_device() != device.index:
            with torch.cuda.device(device):
                return b200_w4g64_linear_multi(x, layers)
        if any(l.qweight.data_ptr() % 16 for l in layers):
            raise ValueError("qweight storage must be 16-byte aligned for the B200 kernels")
        n = len(layers)
        arr = lambda vals: (ctypes.c_void_p * n)(*vals)
        bias_dtype = next((_DTYPE_CODE[b.dtype] for b in biases if b is not None), _lib.DTYPE_NONE)
        rc = lib.qi4_w4g64_linear_multi(
            x2.data_ptr(), _DTYPE_CODE[x2.dtype], x2.shape[0], k, n,
            arr([l.qweight.data_ptr() for l in layers]), arr([l.scales.data_ptr() for l in layers]),
            arr([l.zeros.data_ptr() for l in layers]), arr([_ptr(b) for b in biases]), bias_dtype,
            arr([o.data_ptr() for o in outs]), (ctypes.c_int64 * n)(*[l.out_features for l in layers]),
            _stream(device))
        _lib.check(rc, "qi4_w4g64_linear_multi")
    return [o.reshape(*x.shape[:-1], l.out_features) for o, l in zip(outs, layers)]


def b200_w4g64_gate_up_silu(x: torch.Tensor, gate_proj, up_proj) -> torch.Tensor:
    """``F.silu(gate_proj(x).float()) * up_proj(x).float()`` in one call: the
    FP32 tensor the reference MLP passes to ``down_proj``
    (src/qwen_int4/model.py:133-135). ``gate_proj`` / ``up_proj`` carry the
    QuantLinear buffers and sizes (same in/out features, no bias). Each
    projection is rounded to ``x.dtype`` before the SwiGLU, as QuantLinear
    returns it. No reference counterpart as a single call.
    """
    k, n = gate_proj.in_features, gate_proj.out_features
    if up_proj.in_features != k or up_proj.out_features != n:
        raise ValueError("gate_proj and up_proj must have the same shape")
    if getattr(gate_proj, "bias", None) is not None or getattr(up_proj, "bias", None) is not None:
        raise ValueError("the fused gate/up call takes projections without bias")
    for l in (gate_proj, up_proj):
        _validate_linear(x, l.qweight, l.scales, l.zeros, None, n, k,
                         getattr(l, "group_size", GROUP_SIZE), getattr(l, "packing", "canonical"))
    lib = _require_cuda()
    x2 = _aligned(x.reshape(-1, k))
    out = torch.empty((x2.shape[0], n), dtype=torch.float32, device=x.device)
    if x2.shape[0]:
        device = x2.device
        if _current_device() != device.index:
            with torch.cuda.device(device):
                return b200_w4g64_gate_up_silu(x, gate_proj, up_proj)
        if gate_proj.qweight.data_ptr() % 16 or up_proj.qweight.data_ptr() % 16:
            raise ValueError("qweight storage must be 16-byte aligned for the B200 kernels")
        rc = lib.qi4_w4g64_gate_up_silu(
            x2.data_ptr(), _DTYPE_CODE[x2.dtype], x2.shape[0], k,
            gate_proj.qweight.data_ptr(), gate_proj.scales.data_ptr(), gate_proj.zeros.data_ptr(),
            up_proj.qweight.data_ptr(), up_proj.scales.data_ptr(), up_proj.zeros.data_ptr(),
            out.data_ptr(), n, _stream(device))
        _lib.check(rc, "qi4_w4g64_gate_up_silu")
    return out.reshape(*x.shape[:-1], n)


def linear_canonical_w4g64_b200(
    activations: torch.Tensor,
    qweight: torch.Tensor,
    scales: torch.Tensor,
    zeros: torch.Tensor,
    bias: torch.Tensor | None = None,
    *,
    algo: int = _lib.ALGO_AUTO,
) -> torch.Tensor:
    """Rank-2 operator form (mirrors ``linear_canonical_w4g64_triton``).

    ``out_features`` is inferred from ``scales``; validation messages follow
    src/qwen_int4/triton_kernels.py:224-252.
    """
    _require_cuda()
    if activations.ndim != 2 or not activations.is_cuda or not activations.is_contiguous():
        raise ValueError("activations must be a contiguous rank-2 CUDA tensor")
    if activations.dtype not in _DTYPE_CODE:
        raise ValueError("activations must have dtype torch.float16, torch.bfloat16, or torch.float32")
    rows, in_features = activations.shape
    if rows <= 0 or in_features <= 0 or in_features % GROUP_SIZE:
        raise ValueError("activations require a positive W4G64-compatible feature dimension")
    for name, tensor, dtype in (("qweight", qweight, torch.uint8), ("scales", scales, torch.float16),
                                ("zeros", zeros, torch.uint8)):
        if not tensor.is_cuda or not tensor.is_contiguous() or tensor.dtype != dtype:
            raise ValueError(f"{name} must be a contiguous CUDA tensor with dtype {dtype}")
    groups = in_features // GROUP_SIZE
    if scales.numel() % groups:
        raise ValueError("scales do not encode an integral number of output rows")
    out_features = scales.numel() // groups
    if out_features <= 0 or qweight.numel() != out_features * in_features // 2:
        raise ValueError("qweight size does not match the canonical W4G64 layout")
    if zeros.numel() != (out_features * groups + 1) // 2:
        raise ValueError("zeros size does not match the canonical W4G64 layout")
    if bias is not None:
        if not bias.is_cuda or not bias.is_contiguous() or bias.ndim != 1 or bias.numel() != out_features:
            raise ValueError("bias must be a contiguous CUDA vector matching out_features")
        if bias.dtype not in (torch.float16, torch.bfloat16):
            raise ValueError("bias must have dtype torch.float16 or torch.bfloat16")
    out = torch.empty((rows, out_features), dtype=activations.dtype, device=activations.device)
    return _launch_linear(_aligned(activations), qweight, scales, zeros, bias, out, out_features, algo, True)


def dequantize_canonical_w4g64_b200(
    qweight: torch.Tensor,
    scales: torch.Tensor,
    zeros: torch.Tensor,
    *,
    out_features: int,
    in_features: int,
) -> torch.Tensor:
    """FP32 ``[N, K]`` weight, bit-exact with ``dequantize_groupwise``."""
    lib = _require_cuda()
    if not isinstance(out_features, int) or out_features <= 0:
        raise ValueError("out_features must be a positive integer")
    if not isinstance(in_features, int) or in_features <= 0 or in_features % GROUP_SIZE:
        raise ValueError("canonical asymmetric dequantization requires in_features divisible by 64")
    for name, tensor, dtype in (("qweight", qweight, torch.uint8), ("scales", scales, torch.float16),
                                ("zeros", zeros, torch.uint8)):
        if not tensor.is_cuda:
            raise ValueError(f"{name} must be a CUDA tensor")
        if tensor.dtype != dtype:
            raise ValueError(f"{name} must have dtype {dtype}")
        if not tensor.is_contiguous():
            raise ValueError(f"{name} must be contiguous")
    groups = in_features // GROUP_SIZE
    expected_qweight = out_features * in_features // 2
    expected_scales = out_features * groups
    expected_zeros = (expected_scales + 1) // 2
    if qweight.numel() != expected_qweight:
        raise ValueError(f"qweight must contain {expected_qweight} bytes, got {qweight.numel()}")
    if scales.numel() != expected_scales:
        raise ValueError(f"scales must contain {expected_scales} values, got {scales.numel()}")
    if zeros.numel() != expected_zeros:
        raise ValueError(f"zeros must contain {expected_zeros} bytes, got {zeros.numel()}")
    out = torch.empty((out_features, in_features), device=qweight.device, dtype=torch.float32)
    with torch.cuda.device(qweight.device):
        rc = lib.qi4_w4g64_dequant_f32(_aligned(qweight).data_ptr(), scales.data_ptr(), zeros.data_ptr(),
                                       out.data_ptr(), out_features, in_features, _stream(qweight.device))
    _lib.check(rc, "qi4_w4g64_dequant_f32")
    return out


def unpack_canonical_signed_int4_b200(packed: torch.Tensor, *, elements: int | None = None) -> torch.Tensor:
    """Decode canonical packed signed INT4 bytes to int8 (``elements`` may truncate)."""
    lib = _require_cuda()
    if not packed.is_cuda:
        raise ValueError("B200 canonical INT4 unpack requires a CUDA tensor")
    if packed.dtype != torch.uint8:
        raise ValueError("packed canonical INT4 values must have dtype torch.uint8")
    if not packed.is_contiguous():
        raise ValueError("packed canonical INT4 values must be contiguous")
    available = packed.numel() * 2
    count = available if elements is None else elements
    if not isinstance(count, int) or count < 0 or count > available:
        raise ValueError(f"elements must be in [0, {available}], got {count!r}")
    output = torch.empty(count, device=packed.device, dtype=torch.int8)
    if count == 0:
        return output
    with torch.cuda.device(packed.device):
        rc = lib.qi4_w4_unpack(_aligned(packed).data_ptr(), output.data_ptr(), count, _stream(packed.device))
    _lib.check(rc, "qi4_w4_unpack")
    return output
