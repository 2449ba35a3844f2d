"""``QuantLinear`` with the reference's buffers and dispatch, on the ``b200`` backend.

Mirrors ``QuantLinear`` of ryanyue-16/qwen2-int4-systems
(src/qwen_int4/linear.py:17-72): same constructor arguments, the same
registered buffers (``qweight`` uint8 ``[N*K/2, 1]``, ``scales`` fp16
``[N, K/group]``, ``zeros`` uint8 ``[(N*G+1)//2, 1]``, optional bf16
``bias``), so a reference state dict loads into it unchanged; ``set_backend``
rejects unknown names with ``ValueError`` and a backend is only ever chosen
explicitly. The only backend this module can run is ``"b200"``; to use the
reference's own ``QuantLinear`` and model code instead, see
``integration.register_with_reference``.
"""

from __future__ import annotations

import torch
from torch import nn

from .backends import SUPPORTED_BACKENDS, b200_w4g64_linear


class QuantLinear(nn.Module):
    def __init__(
        self,
        in_features: int,
        out_features: int,
        *,
        group_size: int = 64,
        bias: bool = False,
        backend: str = "b200",
        packing: str = "canonical",
    ) -> None:
        super().__init__()
        if in_features % group_size:
            raise ValueError(f"{in_features=} must be divisible by {group_size=}")
        self.in_features = in_features
        self.out_features = out_features
        self.group_size = group_size
        self.num_groups = in_features // group_size
        self.packing = packing
        self.backend = "b200"
        self.register_buffer("qweight", torch.zeros(out_features * in_features // 2, 1, dtype=torch.uint8))
        self.register_buffer("scales", torch.zeros(out_features, self.num_groups, dtype=torch.float16))
        self.register_buffer(
            "zeros", torch.zeros((out_features * self.num_groups + 1) // 2, 1, dtype=torch.uint8))
        if bias:
            self.bias = nn.Parameter(torch.zeros(out_features, dtype=torch.bfloat16), requires_grad=False)
        else:
            self.register_parameter("bias", None)
        self.set_backend(backend)

    def set_backend(self, backend: str) -> None:
        if backend not in SUPPORTED_BACKENDS:
            raise ValueError(f"unknown backend {backend!r}; choose from {SUPPORTED_BACKENDS}")
        self.backend = backend

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        implementation = {"b200": b200_w4g64_linear}[self.backend]
        return implementation(
            x, self.qweight, self.scales, self.zeros, self.bias,
            out_features=self.out_features, in_features=self.in_features,
            group_size=self.group_size, packing=self.packing,
        )
