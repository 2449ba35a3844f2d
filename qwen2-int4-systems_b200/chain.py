"""Persistent decode chain: dependent W4G64 linears in one cooperative launch.

At decode sizes (M <= 8 tokens) each QuantLinear of the reference model
(src/qwen_int4/model.py:71-73 q/k/v, :122 o_proj, :133-135 gate/up/down,
dispatched one by one through src/qwen_int4/linear.py:56-72) moves too few
bytes to hide a kernel launch. ``DecodeChain`` runs a fixed list of stages -
each stage one to three matrices that share their input, the input being an
external tensor or an earlier stage's output - as one persistent kernel
(C ABI ``qi4_chain_*``): one weight stream per SM across all stages, a
device-side counter (bounded wait) between dependent stages.

The chain keeps raw pointers to every input, bias and output tensor it was
built with (this object holds references to them); a run reads whatever the
input tensors hold when it executes on the stream, like a CUDA graph replay.
Weights are copied once into the chain's prepacked tile-major layout; the
module buffers are not modified.
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass, field
from typing import Sequence

import torch

from . import _lib

_DTYPE_CODE = {torch.float16: _lib.DTYPE_F16, torch.bfloat16: _lib.DTYPE_BF16, torch.float32: _lib.DTYPE_F32}


@dataclass
class Weights:
    """One canonical W4G64 matrix (the QuantLinear checkpoint buffers)."""

    qweight: torch.Tensor
    scales: torch.Tensor
    zeros: torch.Tensor | None
    bias: torch.Tensor | None
    out_features: int

    @classmethod
    def of(cls, module, *, symmetric: bool | None = None) -> "Weights":
        """From a QuantLinear-like module (qweight / scales / zeros / bias /
        out_features). ``symmetric=True`` drops the zero points (all zero for
        symmetric RTN); by default they are kept."""
        zeros = None if symmetric else module.zeros
        return cls(module.qweight, module.scales, zeros, module.bias, module.out_features)


@dataclass
class Stage:
    """``outs[i] = x @ W_i^T (+ b_i)``; with ``swiglu`` the two matrices are
    {gate, up} and ``outs[0]`` (FP32) receives ``silu(g) * u``."""

    x: torch.Tensor
    mats: Sequence[Weights]
    outs: Sequence[torch.Tensor]
    swiglu: bool = False
    keep: list = field(default_factory=list)


class DecodeChain:
    def __init__(self, stages: Sequence[Stage], m: int, stream: torch.cuda.Stream | None = None):
        self._lib = _lib.load()
        self.m = int(m)
        self.stages = list(stages)
        arr = (_lib.ChainStage * len(self.stages))()
        device = None
        for i, st in enumerate(self.stages):
            x = st.x
            if not x.is_cuda or not x.is_contiguous():
                raise ValueError(f"stage {i}: x must be a contiguous CUDA tensor")
            device = device or x.device
            if x.dtype not in _DTYPE_CODE:
                raise TypeError(f"stage {i}: activation dtype {x.dtype} is not float16, bfloat16 or float32")
            if x.numel() != self.m * x.shape[-1]:
                raise ValueError(f"stage {i}: x must hold M={self.m} rows")
            d = arr[i]
            d.nmats = len(st.mats)
            d.flags = _lib.CHAIN_SWIGLU if st.swiglu else 0
            d.K = x.shape[-1]
            d.x = x.data_ptr()
            d.x_dtype = _DTYPE_CODE[x.dtype]
            d.out_dtype = _DTYPE_CODE[st.outs[0].dtype]
            biases = [w.bias for w in st.mats if w.bias is not None]
            d.bias_dtype = _DTYPE_CODE[biases[0].dtype] if biases else _lib.DTYPE_NONE
            for j, w in enumerate(st.mats):
                for t in (w.qweight, w.scales, w.zeros, w.bias):
                    if t is not None and (not t.is_cuda or not t.is_contiguous()):
                        raise ValueError(f"stage {i}: weights must be contiguous CUDA tensors")
                d.qweight[j] = w.qweight.data_ptr()
                d.scales_f16[j] = w.scales.data_ptr()
                d.zeros[j] = None if w.zeros is None else w.zeros.data_ptr()
                d.bias[j] = None if w.bias is None else w.bias.data_ptr()
                d.N[j] = w.out_features
            for j, o in enumerate(st.outs):
                if not o.is_cuda or not o.is_contiguous():
                    raise ValueError(f"stage {i}: outputs must be contiguous CUDA tensors")
                d.out[j] = o.data_ptr()
        self._arr = arr
        handle = ctypes.c_void_p()
        stream = stream or torch.cuda.current_stream(device)
        with torch.cuda.device(device):
            rc = self._lib.qi4_chain_create(ctypes.cast(arr, ctypes.c_void_p), len(self.stages), self.m,
                                            stream.cuda_stream, ctypes.byref(handle))
        _lib.check(rc, "qi4_chain_create")
        self._handle = handle
        self.device = device

    def run(self, stream: torch.cuda.Stream | None = None) -> None:
        """Enqueue one pass over every stage on ``stream`` (default: current)."""
        if self._handle is None:
            raise RuntimeError("decode chain is closed")
        stream = stream or torch.cuda.current_stream(self.device)
        rc = self._lib.qi4_chain_run(self._handle, stream.cuda_stream)
        _lib.check(rc, "qi4_chain_run")

    def info(self) -> dict:
        vals = (ctypes.c_int64 * 8)()
        _lib.check(self._lib.qi4_chain_info(self._handle, ctypes.cast(vals, ctypes.c_void_p)), "qi4_chain_info")
        keys = ("ctas", "ring_slots", "smem_bytes", "prepacked_bytes", "alg_bytes", "stages")
        return {k: int(vals[i]) for i, k in enumerate(keys)}

    def close(self) -> None:
        if getattr(self, "_handle", None) is not None:
            self._lib.qi4_chain_destroy(self._handle)
            self._handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def decoder_linear_stages(layers, x: torch.Tensor) -> tuple[list[Stage], dict]:
    """The linear stages of a stack of Qwen2 decoder layers at decode size,
    as the reference composes them (src/qwen_int4/model.py:61-136): per layer
    q/k/v (one stage, shared input), o_proj, gate/up fused with SwiGLU (FP32
    out, the tensor the reference hands to down_proj), down_proj (FP32 in,
    activation dtype out); layer l + 1 takes layer l's down_proj output.

    ``layers``: sequences of modules with ``self_attn.{q,k,v,o}_proj`` and
    ``mlp.{gate,up,down}_proj`` (QuantLinear-like). Attention, the residual
    stream and RMSNorm are not linears and are not part of the chain: o_proj
    reads q_proj's output as the stand-in for the attention output. Returns
    the stages and the buffers they write."""
    m, dtype, dev = x.shape[0], x.dtype, x.device
    stages, bufs = [], {"x": x}
    cur = x
    for li, layer in enumerate(layers):
        a, f = layer.self_attn, layer.mlp
        q = torch.empty(m, a.q_proj.out_features, dtype=dtype, device=dev)
        k = torch.empty(m, a.k_proj.out_features, dtype=dtype, device=dev)
        v = torch.empty(m, a.v_proj.out_features, dtype=dtype, device=dev)
        o = torch.empty(m, a.o_proj.out_features, dtype=dtype, device=dev)
        h = torch.empty(m, f.gate_proj.out_features, dtype=torch.float32, device=dev)
        y = torch.empty(m, f.down_proj.out_features, dtype=dtype, device=dev)
        sym = lambda mod: bool((mod.zeros == 0).all())  # noqa: E731
        W = lambda mod: Weights.of(mod, symmetric=sym(mod))  # noqa: E731
        stages.append(Stage(cur, [W(a.q_proj), W(a.k_proj), W(a.v_proj)], [q, k, v]))
        stages.append(Stage(q, [W(a.o_proj)], [o]))
        stages.append(Stage(o, [W(f.gate_proj), W(f.up_proj)], [h], swiglu=True))
        stages.append(Stage(h, [W(f.down_proj)], [y]))
        bufs[li] = {"q": q, "k": k, "v": v, "o": o, "h": h, "y": y}
        cur = y
    return stages, bufs
