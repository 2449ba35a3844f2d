"""PyTorch-CPU restatement of the reference's ``torch`` backend (the CPU baseline).

TEST / BENCHMARK INFRASTRUCTURE ONLY. ``bench.py`` times this module as the
reference's own CPU implementation of the QuantLinear forward
(``cpu_baseline.kind = "port"``) because the reference package itself does
not travel to the GPU host; tests use it as the FP32 tolerance reference.
The product path never imports it.

It follows ryanyue-16/qwen2-int4-systems ``src/qwen_int4/backends.py:73-98``
(``torch_reference_linear``) and ``src/qwen_int4/quantization.py:221-258``
(``dequantize_groupwise``) step for step, with the same PyTorch CPU kernels
doing the work: decode every packed byte into two signed codes, expand the
per-group zero points and FP32 scales along K, form the full FP32 weight,
then one FP32 matmul, an FP32 bias add and a final cast to ``x.dtype``.
Pinned against the reference's own outputs by ``tests/test_oracle_golden.py``.
"""

from __future__ import annotations

import torch

GROUP_SIZE = 64


def _signed_nibbles(packed: torch.Tensor) -> torch.Tensor:
    """uint8 bytes -> int8 codes, element 2i from the low nibble (two's complement)."""
    byte = packed.reshape(-1).to(torch.int16)
    pair = torch.stack((byte & 0x0F, byte >> 4), dim=-1).reshape(-1)
    return ((pair ^ 0x08) - 8).to(torch.int8)


def dequantize(
    qweight: torch.Tensor,
    scales: torch.Tensor,
    zeros: torch.Tensor | None,
    *,
    out_features: int,
    in_features: int,
    group_size: int = GROUP_SIZE,
) -> torch.Tensor:
    groups = in_features // group_size
    codes = _signed_nibbles(qweight).reshape(out_features, groups, group_size)
    if zeros is None:
        zero = torch.zeros(out_features, groups, dtype=torch.float32)
    else:
        zero = _signed_nibbles(zeros)[: out_features * groups]
        zero = zero.reshape(out_features, groups).to(torch.float32)
    weight = (codes.to(torch.float32) - zero.unsqueeze(-1)) * scales.to(
        torch.float32
    ).unsqueeze(-1)
    return weight.reshape(out_features, in_features)


def linear(
    x: torch.Tensor,
    qweight: torch.Tensor,
    scales: torch.Tensor,
    zeros: torch.Tensor | None,
    bias: torch.Tensor | None,
    *,
    out_features: int,
    in_features: int,
    group_size: int = GROUP_SIZE,
) -> torch.Tensor:
    weight = dequantize(
        qweight, scales, zeros, out_features=out_features,
        in_features=in_features, group_size=group_size,
    )
    out = x.reshape(-1, in_features).to(torch.float32) @ weight.t()
    if bias is not None:
        out = out + bias.to(torch.float32)
    return out.reshape(*x.shape[:-1], out_features).to(x.dtype)
