"""Tied bf16 lm_head with the greedy token fused in (C ABI ``qi4_bf16_gemv_argmax``).

For decode sizes (up to 8 rows): ``logits = x @ weight.T`` in bf16 - the
reference's ``lm_head`` over the tied embedding (src/qwen_int4/model.py:
217-218,243) - and the per-row argmax over those logits, first index on ties,
as the reference's greedy step takes it (src/qwen_int4/generation.py:51).
A caller that needs only the greedy token passes ``return_logits=False`` and
the kernel skips writing the vocabulary-wide logits.
"""

from __future__ import annotations

import torch

from . import _lib
from .backends import _require_cuda, _stream


def b200_lm_head(x: torch.Tensor, weight: torch.Tensor, *, return_logits: bool = True,
                 return_argmax: bool = True):
    """(logits [M, V] bf16 or None, argmax [M] int64 or None) for x [M, D] bf16."""
    lib = _require_cuda()
    if x.dtype != torch.bfloat16 or weight.dtype != torch.bfloat16 or not x.is_cuda or not weight.is_cuda:
        raise TypeError("lm_head GEMV takes bf16 CUDA tensors")
    if not (return_logits or return_argmax):
        raise ValueError("ask for the logits, the argmax, or both")
    x2 = x.reshape(-1, x.shape[-1]).contiguous()
    w = weight.contiguous()
    m, k = x2.shape
    n = w.shape[0]
    if w.shape[1] != k:
        raise ValueError("x and weight disagree on the hidden size")
    logits = torch.empty(m, n, dtype=torch.bfloat16, device=x.device) if return_logits else None
    arg = torch.empty(m, dtype=torch.int64, device=x.device) if return_argmax else None
    rc = lib.qi4_bf16_gemv_argmax(w.data_ptr(), x2.data_ptr(), m, k, n,
                                  None if logits is None else logits.data_ptr(),
                                  None if arg is None else arg.data_ptr(), _stream(x.device))
    _lib.check(rc, "qi4_bf16_gemv_argmax")
    return logits, arg
