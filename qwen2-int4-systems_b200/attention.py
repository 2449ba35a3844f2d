"""Decode attention with in-place KV-cache append, and its drop-in for the reference model.

``b200_gqa_decode_attention`` wraps the C ABI ``qi4_gqa_decode_attention``:
RoPE of the new query/key, append of the new key/value into a preallocated
cache, and grouped-query attention over the cache without expanding the KV
heads - one call per layer and decode step.

``patch_reference_attention`` routes the decode step (one new token per
sequence, a past cache present) of the reference's ``QwenAttention.forward``
(src/qwen_int4/model.py:61-122) through it when the attention's projections
run on the ``b200`` backend. The cache keeps the reference's form - a
``(key, value)`` tuple of ``[B, Hkv, L, D]`` tensors per layer - but those
tensors are views of buffers with spare capacity, so the next step writes its
key/value in place instead of re-copying the whole cache with ``torch.cat``
(model.py:87-88); the ``repeat_interleave`` of the KV heads (model.py:90-91)
disappears. A buffer is extended in place only by the holder of its latest
view: a cache that was forked (two continuations of one prefix) is copied on
write, so every continuation keeps its own keys. Prompts (more than one new
token) and caches without spare capacity go through the reference code, the
latter after one copy into a buffer with capacity.
"""

from __future__ import annotations

import importlib
import sys
import weakref

import torch

from . import _lib
from .backends import _require_cuda, _stream

HEAD_DIM = 128
_CAPACITY_STEP = 256

# Per cache buffer (by its data pointer): the length its latest view covers.
_committed: dict[int, tuple[weakref.ref, int]] = {}


def b200_gqa_decode_attention(q, k_new, v_new, k_cache, v_cache, lengths, *, cos=None, sin=None, positions=None,
                              key_mask=None, scale=None) -> torch.Tensor:
    """out [B, Hq * D] (bf16) for one new token per sequence.

    q [B, Hq, D], k_new / v_new [B, Hkv, D] (bf16, before RoPE when cos/sin
    are given); k_cache / v_cache [B, Hkv, capacity, D] (bf16, last dim
    contiguous); lengths [B] int32 on the device (the past length: the new
    key goes to position lengths[b]); cos / sin [rows, D] bf16 with row
    ``positions[b]`` (or ``b``); key_mask [B, >= L + 1] (non-zero = key
    valid) or None. The caches are written in place; lengths is not changed.
    """
    lib = _require_cuda()
    B, Hq, D = q.shape
    Hkv = k_new.shape[1]
    for t in (q, k_new, v_new, k_cache, v_cache):
        if t.dtype != torch.bfloat16 or not t.is_cuda:
            raise TypeError("decode attention takes bf16 CUDA tensors")
    if k_cache.stride(-1) != 1 or k_cache.stride(-2) != D or v_cache.stride() != k_cache.stride():
        raise ValueError("KV caches must be [B, Hkv, capacity, D] with contiguous rows and equal strides")
    a16 = lambda t: t if t.data_ptr() % 16 == 0 else t.clone()  # noqa: E731  (the kernel copies 16-byte chunks)
    q, k_new, v_new = a16(q.contiguous()), a16(k_new.contiguous()), a16(v_new.contiguous())
    if lengths.dtype != torch.int32 or not lengths.is_cuda:
        raise TypeError("lengths must be an int32 CUDA tensor")
    if cos is not None:
        cos, sin = a16(cos.contiguous()), a16(sin.contiguous())
        if cos.dtype != torch.bfloat16 or sin.dtype != torch.bfloat16 or cos.shape[-1] != D:
            raise TypeError("cos / sin must be bf16 rows of head_dim")
    mask = None
    if key_mask is not None:
        mask = key_mask if key_mask.dtype == torch.uint8 else key_mask.to(torch.uint8)
        mask = mask.contiguous()
    out = torch.empty(B, Hq * D, dtype=torch.bfloat16, device=q.device)
    scale = float(D ** -0.5 if scale is None else scale)
    p = lambda t: None if t is None else t.data_ptr()  # noqa: E731
    rc = lib.qi4_gqa_decode_attention(
        q.data_ptr(), k_new.data_ptr(), v_new.data_ptr(), p(cos), p(sin), p(positions), k_cache.data_ptr(),
        v_cache.data_ptr(), k_cache.stride(0), k_cache.stride(1), k_cache.shape[2], lengths.data_ptr(), p(mask),
        0 if mask is None else mask.stride(0), out.data_ptr(), B, Hq, Hkv, D, scale, _stream(q.device))
    _lib.check(rc, "qi4_gqa_decode_attention")
    return out


def _capacity_view(t: torch.Tensor):
    """(base buffer, capacity) if t is the [B, H, L, D] prefix view of a
    buffer this module created and still the latest view of it, else None."""
    entry = _committed.get(t.untyped_storage().data_ptr())
    if entry is None:
        return None
    base = entry[0]()
    if base is None or t.storage_offset() != 0 or t.stride() != base.stride() or entry[1] != t.shape[2]:
        return None
    return base, base.shape[2]


def _ensure_room(past_k: torch.Tensor, past_v: torch.Tensor):
    """Buffers with room for one more key: the existing ones when the views
    are their latest, else fresh buffers holding a copy of the past."""
    length = past_k.shape[2]
    ck, cv = _capacity_view(past_k), _capacity_view(past_v)
    if ck and cv and ck[1] > length and cv[1] > length:
        return ck[0], cv[0]
    cap = (length + 1 + _CAPACITY_STEP - 1) // _CAPACITY_STEP * _CAPACITY_STEP
    shape = (past_k.shape[0], past_k.shape[1], cap, past_k.shape[3])
    kb = torch.empty(shape, dtype=past_k.dtype, device=past_k.device)
    vb = torch.empty(shape, dtype=past_v.dtype, device=past_v.device)
    kb[:, :, :length].copy_(past_k)
    vb[:, :, :length].copy_(past_v)
    return kb, vb


def _commit(buf: torch.Tensor, length: int) -> torch.Tensor:
    key = buf.untyped_storage().data_ptr()
    entry = _committed.get(key)
    if entry is None or entry[0]() is not buf:
        weakref.finalize(buf, _committed.pop, key, None)
    _committed[key] = (weakref.ref(buf), length)
    return buf[:, :, :length]


def patch_reference_attention(package: str = "qwen_int4", enabled: bool = True) -> None:
    """Route the reference QwenAttention's decode steps through the b200
    decode attention when its projections are on the ``b200`` backend (each
    call sets the switch; the patch itself is installed once)."""
    name = f"{package}.model"
    if not enabled and name not in sys.modules:
        return
    attn_cls = getattr(importlib.import_module(name), "QwenAttention", None)
    if attn_cls is None:
        if enabled:
            raise AttributeError(f"{name} has no QwenAttention to route through the b200 decode attention")
        return
    if not getattr(attn_cls.forward, "_b200_attention", False):
        reference_forward = attn_cls.forward

        def forward(self, hidden_states, cos, sin, attention_mask, past_key_value=None, use_cache=False):
            fast = (type(self)._b200_attention_on and past_key_value is not None and hidden_states.shape[1] == 1
                    and self.q_proj.backend == "b200" and self.k_proj.backend == "b200"
                    and self.v_proj.backend == "b200" and hidden_states.dtype == torch.bfloat16
                    and hidden_states.is_cuda and self.head_dim == HEAD_DIM
                    and self.num_heads // self.num_kv_heads <= 8)
            if not fast:
                return reference_forward(self, hidden_states, cos, sin, attention_mask, past_key_value, use_cache)
            batch = hidden_states.shape[0]
            past_k, past_v = past_key_value
            expected = (batch, self.num_kv_heads, past_k.shape[2], self.head_dim)
            if past_k.shape != expected or past_v.shape != expected:
                raise ValueError("past key/value cache shape does not match this attention layer")
            if past_k.device != hidden_states.device or past_v.device != hidden_states.device:
                raise ValueError("past key/value cache must be on the attention device")
            length = past_k.shape[2]
            if attention_mask is not None and attention_mask.shape != (batch, length + 1):
                raise ValueError("attention_mask must cover cached and current tokens")
            q = self.q_proj(hidden_states).view(batch, self.num_heads, self.head_dim)
            k = self.k_proj(hidden_states).view(batch, self.num_kv_heads, self.head_dim)
            v = self.v_proj(hidden_states).view(batch, self.num_kv_heads, self.head_dim)
            kbuf, vbuf = _ensure_room(past_k, past_v)
            lengths = torch.full((batch,), length, dtype=torch.int32, device=hidden_states.device)
            out = b200_gqa_decode_attention(
                q, k, v, kbuf, vbuf, lengths, cos=cos[:, 0].to(torch.bfloat16), sin=sin[:, 0].to(torch.bfloat16),
                key_mask=attention_mask, scale=self.head_dim ** -0.5)
            next_cache = (_commit(kbuf, length + 1), _commit(vbuf, length + 1)) if use_cache else None
            return self.o_proj(out.view(batch, 1, self.hidden_size)), next_cache

        forward._b200_attention = True
        attn_cls.forward = forward
    attn_cls._b200_attention_on = enabled
