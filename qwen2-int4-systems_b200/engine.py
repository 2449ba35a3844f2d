"""Graph-captured greedy decoding of the reference Qwen2 model on the b200 kernels.

The reference generates one token per step through its Python model code
(src/qwen_int4/generation.py:96-115 ``greedy_generate_cached``, model.py
forward): ~30 tensor ops per decoder layer, each a separate launch with host
overhead, and a KV cache re-concatenated every step. ``DecodeEngine`` takes the
same model (its QuantLinear buffers, norms, rotary table and tied embedding,
read as they are) and runs each decode step as one CUDA graph of this
library's kernels, on static buffers:

  embed -> per layer: residual add + RMSNorm and q/k/v in one launch
           (qi4_w4g64_linear_multi_norm: the GEMV forms its activations from
           the residual stream while staging them; up to 8 sequences, else
           qi4_add_rmsnorm + qi4_w4g64_linear_multi), RoPE + KV append + GQA
           attention (qi4_gqa_decode_attention), o_proj (qi4_w4g64_linear),
           residual add + RMSNorm and gate/up + SwiGLU in one launch
           (qi4_w4g64_gate_up_silu_norm, FP32 out), down_proj
           (qi4_w4g64_linear on FP32 input)
        -> final residual add + RMSNorm -> tied lm_head + greedy argmax
           (qi4_bf16_gemv_argmax for up to 8 sequences; a bf16 matmul and
           qi4_bf16_argmax_rows beyond) -> next tokens, lengths and positions advanced on
           the device.

The prompt runs through the reference model itself (``model(..., use_cache=
True)`` on whatever backend it is set to); its key/value cache is copied into
the engine's preallocated cache. ``generate`` returns what
``greedy_generate_cached`` returns: the prompt followed by the new tokens.
Numerics follow the reference's order of roundings (bf16 residual stream,
FP32 norm statistics, FP32 SwiGLU into down_proj); the kernels' FP32 sums
differ from PyTorch's only in summation order.
"""

from __future__ import annotations

import ctypes

import torch

from . import _lib
from .backends import _require_cuda

BF16, F32, NONE = _lib.DTYPE_BF16, _lib.DTYPE_F32, _lib.DTYPE_NONE


def _ptr(t):
    return None if t is None else t.data_ptr()


class _Linear:
    """Pointers of one QuantLinear (symmetric zero points dropped)."""

    def __init__(self, mod):
        self.mod = mod
        self.n, self.k = mod.out_features, mod.in_features
        self.qweight, self.scales, self.bias = mod.qweight, mod.scales, mod.bias
        self.zeros = None if bool((mod.zeros == 0).all()) else mod.zeros
        if getattr(mod, "group_size", 64) != 64 or str(getattr(mod.packing, "value", mod.packing)) != "canonical":
            raise ValueError("the decode engine runs canonical W4G64 QuantLinear modules")


class DecodeEngine:
    def __init__(self, model, batch: int, max_len: int):
        self.lib = _require_cuda()
        self.model = model
        cfg = model.config
        self.B, self.max_len = int(batch), int(max_len)
        self.D = cfg.hidden_size
        self.Hq, self.Hkv = cfg.num_attention_heads, cfg.num_key_value_heads
        self.hd = getattr(cfg, "head_dim", self.D // self.Hq)
        self.eps = float(cfg.rms_norm_eps)
        emb = model.model.embed_tokens.weight
        self.device = emb.device
        dev = self.device
        bf = dict(dtype=torch.bfloat16, device=dev)
        self.layers = []
        for layer in model.model.layers:
            a, f = layer.self_attn, layer.mlp
            self.layers.append(dict(
                qkv=[_Linear(a.q_proj), _Linear(a.k_proj), _Linear(a.v_proj)], o=_Linear(a.o_proj),
                gate=_Linear(f.gate_proj), up=_Linear(f.up_proj), down=_Linear(f.down_proj),
                w_in=layer.input_layernorm.weight, w_post=layer.post_attention_layernorm.weight))
        self.w_final = model.model.norm.weight
        self.embed = emb
        self.lm_weight = model.lm_head.weight
        inter = self.layers[0]["gate"].n
        B = self.B
        # Static buffers of a step.
        self.tokens = torch.zeros(B, dtype=torch.int64, device=dev)
        # The bf16 residual stream: with the norm folded into the next launch
        # (up to 8 sequences: every CTA of that launch recomputes the rows'
        # statistics, which at 16 sequences costs more than a norm launch)
        # each boundary reads one buffer and writes the other; otherwise the
        # norm kernel updates hbuf[0] in place.
        self.hbuf = [torch.empty(B, self.D, **bf), torch.empty(B, self.D, **bf)]
        self.fuse_norm = B <= 8
        self.x = torch.empty(B, self.D, **bf)
        self.q = torch.empty(B, self.Hq * self.hd, **bf)
        self.k = torch.empty(B, self.Hkv * self.hd, **bf)
        self.v = torch.empty(B, self.Hkv * self.hd, **bf)
        self.attn = torch.empty(B, self.Hq * self.hd, **bf)
        self.o = torch.empty(B, self.D, **bf)
        self.hm = torch.empty(B, inter, dtype=torch.float32, device=dev)
        self.y = torch.empty(B, self.D, dtype=torch.float32, device=dev)
        self.next = torch.zeros(B, dtype=torch.int64, device=dev)
        # Beyond the GEMV's 8 tokens the tied lm_head is a bf16 matmul into
        # these logits, then qi4_bf16_argmax_rows.
        self.logits = (torch.empty(B, self.lm_weight.shape[0], dtype=torch.bfloat16, device=dev)
                       if B > 8 else None)
        self.lengths = torch.zeros(B, dtype=torch.int32, device=dev)
        self.positions = torch.zeros(B, dtype=torch.int32, device=dev)
        self.key_mask = torch.zeros(B, max_len, dtype=torch.uint8, device=dev)
        shape = (len(self.layers), B, self.Hkv, max_len, self.hd)
        self.kcache = torch.zeros(shape, **bf)
        self.vcache = torch.zeros(shape, **bf)
        # RoPE table of the reference's own rotary embedding, by position.
        with torch.inference_mode():
            pos = torch.arange(max_len, device=dev).view(1, -1)
            cos, sin = model.model.rotary_emb(pos, torch.bfloat16)
        self.cos, self.sin = cos[0].contiguous(), sin[0].contiguous()
        # Caller-owned workspaces: the captured step holds only kernel nodes,
        # so programmatic dependent launch links every kernel to the next.
        ws = self.lib.qi4_gqa_decode_attention_workspace(B, self.Hq, self.Hkv, max_len)
        self.attn_ws = torch.empty(max(ws, 16), dtype=torch.uint8, device=dev)
        self.lm_keys = torch.zeros(8, dtype=torch.int64, device=dev)
        self.graph = None
        self.stream = torch.cuda.Stream(device=dev)

    # -- one decode step (C ABI calls on the current stream) ---------------
    def _linear(self, lin: _Linear, x, x_dtype, out):
        rc = self.lib.qi4_w4g64_linear(x.data_ptr(), x_dtype, self.B, lin.k, lin.qweight.data_ptr(),
                                       lin.scales.data_ptr(), _ptr(lin.zeros), _ptr(lin.bias),
                                       BF16 if lin.bias is not None else NONE, out.data_ptr(), lin.n, self._s)
        _lib.check(rc, "qi4_w4g64_linear")

    def _norm(self, h, delta, delta_dtype, w):
        rc = self.lib.qi4_add_rmsnorm(h.data_ptr(), _ptr(delta), delta_dtype, w.data_ptr(), self.x.data_ptr(),
                                      self.B, self.D, self.eps, self._s)
        _lib.check(rc, "qi4_add_rmsnorm")

    def _prologue(self, delta, delta_dtype, w):
        """The boundary folded into the next launch: hbuf[cur] + delta -> hbuf[cur ^ 1]."""
        src, dst = self.hbuf[self._cur], self.hbuf[self._cur ^ 1]
        self._cur ^= 1
        return _lib.RmsNormPrologue(src.data_ptr(), _ptr(delta), delta_dtype, self.eps, w.data_ptr(), dst.data_ptr())

    def _step(self):
        B, L = self.B, self.lib
        self._s = torch.cuda.current_stream().cuda_stream
        # The new token is a valid key at position lengths[b].
        self.key_mask.scatter_(1, self.lengths.view(B, 1).long(), 1)
        self._cur = 0
        torch.index_select(self.embed, 0, self.tokens, out=self.hbuf[0])
        delta, ddt = None, NONE
        for li, lay in enumerate(self.layers):
            qkv = lay["qkv"]
            arr = lambda vals: (ctypes.c_void_p * 3)(*vals)  # noqa: E731
            mats = (3, arr([m.qweight.data_ptr() for m in qkv]), arr([m.scales.data_ptr() for m in qkv]),
                    arr([_ptr(m.zeros) for m in qkv]), arr([_ptr(m.bias) for m in qkv]), BF16,
                    arr([self.q.data_ptr(), self.k.data_ptr(), self.v.data_ptr()]),
                    (ctypes.c_int64 * 3)(*[m.n for m in qkv]), self._s)
            if self.fuse_norm:
                pro = self._prologue(delta, ddt, lay["w_in"])
                rc = L.qi4_w4g64_linear_multi_norm(ctypes.byref(pro), B, self.D, *mats)
            else:
                self._norm(self.hbuf[0], delta, ddt, lay["w_in"])
                rc = L.qi4_w4g64_linear_multi(self.x.data_ptr(), BF16, B, self.D, *mats)
            _lib.check(rc, "qi4_w4g64_linear_multi")
            kc, vc = self.kcache[li], self.vcache[li]
            # Early cache reads: within a step nothing writes the caches or
            # lengths before the attention of a layer but that attention.
            rc = L.qi4_gqa_decode_attention_ex(
                self.q.data_ptr(), self.k.data_ptr(), self.v.data_ptr(), self.cos.data_ptr(), self.sin.data_ptr(),
                self.positions.data_ptr(), kc.data_ptr(), vc.data_ptr(), kc.stride(0), kc.stride(1), self.max_len,
                self.lengths.data_ptr(), self.key_mask.data_ptr(), self.key_mask.stride(0), self.attn.data_ptr(), B,
                self.Hq, self.Hkv, self.hd, float(self.hd ** -0.5), _lib.ATTN_EARLY_CACHE_READ,
                self.attn_ws.data_ptr(), self.attn_ws.numel(), self._s)
            _lib.check(rc, "qi4_gqa_decode_attention")
            self._linear(lay["o"], self.attn, BF16, self.o)
            g, u = lay["gate"], lay["up"]
            mats = (g.qweight.data_ptr(), g.scales.data_ptr(), _ptr(g.zeros), u.qweight.data_ptr(),
                    u.scales.data_ptr(), _ptr(u.zeros), self.hm.data_ptr(), g.n, self._s)
            if self.fuse_norm:
                pro = self._prologue(self.o, BF16, lay["w_post"])
                rc = L.qi4_w4g64_gate_up_silu_norm(ctypes.byref(pro), B, self.D, *mats)
            else:
                self._norm(self.hbuf[0], self.o, BF16, lay["w_post"])
                rc = L.qi4_w4g64_gate_up_silu(self.x.data_ptr(), BF16, B, self.D, *mats)
            _lib.check(rc, "qi4_w4g64_gate_up_silu")
            self._linear(lay["down"], self.hm, F32, self.y)
            delta, ddt = self.y, F32
        self._norm(self.hbuf[self._cur], delta, ddt, self.w_final)
        if B <= 8:
            rc = L.qi4_bf16_gemv_argmax_ws(self.lm_weight.data_ptr(), self.x.data_ptr(), B, self.D,
                                           self.lm_weight.shape[0], None, self.next.data_ptr(),
                                           self.lm_keys.data_ptr(), self._s)
            _lib.check(rc, "qi4_bf16_gemv_argmax")
        else:
            torch.mm(self.x, self.lm_weight.t(), out=self.logits)
            rc = L.qi4_bf16_argmax_rows(self.logits.data_ptr(), B, self.logits.shape[1], self.logits.shape[1],
                                        self.next.data_ptr(), self._s)
            _lib.check(rc, "qi4_bf16_argmax_rows")
        self.lengths.add_(1)
        self.positions.add_(1)
        self.tokens.copy_(self.next)

    def _capture(self):
        # The capture stream first waits for the caller's stream: the prefill's
        # cache copies, lengths, positions and tokens must have landed before
        # the warm-up step reads them and before they are saved for restoring.
        self.stream.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(self.stream):
            # Warm-up outside capture, on a state that is restored afterwards.
            saved = (self.lengths.clone(), self.positions.clone(), self.key_mask.clone(), self.tokens.clone())
            self._step()
            torch.cuda.current_stream().synchronize()
            for t, s in zip((self.lengths, self.positions, self.key_mask, self.tokens), saved):
                t.copy_(s)
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=self.stream):
                self._step()
        torch.cuda.current_stream().wait_stream(self.stream)
        self.graph = g

    # -- public API ---------------------------------------------------------
    @torch.inference_mode()
    def prefill(self, input_ids: torch.Tensor, attention_mask: torch.Tensor | None = None) -> torch.Tensor:
        """Run the prompt through the reference model; load its KV cache.
        Returns the first greedy token per sequence."""
        B, P = input_ids.shape
        if B != self.B:
            raise ValueError(f"the engine was built for batch {self.B}")
        if P + 1 > self.max_len:
            raise ValueError("prompt longer than the engine's max_len")
        mask = torch.ones_like(input_ids, dtype=torch.bool) if attention_mask is None else attention_mask.bool()
        logits, cache = self.model(input_ids, attention_mask=mask, use_cache=True)
        for li, (k, v) in enumerate(cache):
            self.kcache[li, :, :, :P].copy_(k)
            self.vcache[li, :, :, :P].copy_(v)
        self.key_mask.zero_()
        self.key_mask[:, :P].copy_(mask)
        self.lengths.fill_(P)
        self.positions.copy_(mask.sum(dim=-1).to(torch.int32))
        first = logits[:, -1].argmax(dim=-1)
        self.tokens.copy_(first)
        return first

    @torch.inference_mode()
    def decode(self, steps: int) -> torch.Tensor:
        """Run `steps` graph-captured decode steps from the current state;
        returns the tokens fed to the steps ([B, steps]): the first is the
        prefill's greedy token."""
        if self.graph is None:
            self._capture()
        if int(self.lengths.max()) + steps > self.max_len:
            raise ValueError("decode would overrun the engine's KV cache")
        out = torch.empty(self.B, steps, dtype=torch.int64, device=self.device)
        for i in range(steps):
            out[:, i].copy_(self.tokens)
            self.graph.replay()
        return out

    @torch.inference_mode()
    def generate(self, input_ids: torch.Tensor, max_new_tokens: int,
                 attention_mask: torch.Tensor | None = None) -> torch.Tensor:
        """Greedy continuation with the semantics of the reference's
        ``greedy_generate_cached``: prompt followed by max_new_tokens tokens."""
        if max_new_tokens <= 0:
            return input_ids.clone()
        self.prefill(input_ids, attention_mask)
        new = self.decode(max_new_tokens)
        return torch.cat((input_ids, new), dim=1)

    def close(self):
        self.graph = None
