"""Register the ``b200`` backend with the reference package at run time.

The reference project ryanyue-16/qwen2-int4-systems selects a QuantLinear
backend by name (src/qwen_int4/backends.py:11 ``SUPPORTED_BACKENDS``,
src/qwen_int4/linear.py:51-72 ``set_backend`` / ``forward``,
src/qwen_int4/cli.py:59 ``--backend`` choices). ``register_with_reference``
adds ``"b200"`` to those tables in an already-imported ``qwen_int4`` package,
so the unmodified model (src/qwen_int4/model.py) runs on the B200 kernels
after ``model.set_backend("b200")``. The static patch a maintainer would
commit instead is a three-line change to those tables.

``fuse_mlp=True`` also routes ``QwenMLP.forward`` (src/qwen_int4/model.py:
133-136) through the fused gate/up SwiGLU call when both projections are on
the ``b200`` backend: one launch computes ``silu(gate(x)) * up(x)`` (each
projection rounded to ``x.dtype`` first, as QuantLinear returns it) in FP32,
which ``down_proj`` consumes exactly as the reference MLP passes it.

``fast_attention=True`` routes the reference attention's decode steps through
the b200 decode attention (RoPE + in-place KV append + GQA attention in one
call; see the ``attention`` module), keeping the reference's cache tuples.
"""

from __future__ import annotations

import importlib
import sys

from .backends import b200_w4g64_gate_up_silu, b200_w4g64_linear

BACKEND = "b200"


def register_with_reference(package: str = "qwen_int4", *, fuse_mlp: bool = False,
                            fast_attention: bool = False) -> None:
    """Make ``backend="b200"`` valid in the reference's QuantLinear. Idempotent.

    ``fuse_mlp`` selects whether the reference MLP uses the fused gate/up
    SwiGLU call on that backend; ``fast_attention`` whether the reference
    attention's decode steps use the b200 decode attention with in-place KV
    cache append (attention.patch_reference_attention). Each call sets both
    switches (default off).
    """
    _register_linear(package)
    _set_mlp_fusion(package, fuse_mlp)
    from .attention import patch_reference_attention

    patch_reference_attention(package, fast_attention)


def _register_linear(package: str) -> None:
    backends = importlib.import_module(f"{package}.backends")
    linear = importlib.import_module(f"{package}.linear")
    if BACKEND not in backends.SUPPORTED_BACKENDS:
        backends.SUPPORTED_BACKENDS = tuple(backends.SUPPORTED_BACKENDS) + (BACKEND,)
    # linear.py imported the tuple by name, so its binding is updated too.
    linear.SUPPORTED_BACKENDS = backends.SUPPORTED_BACKENDS
    backends.b200_w4g64_linear = b200_w4g64_linear
    quant_linear = linear.QuantLinear
    if getattr(quant_linear.forward, "_b200_dispatch", False):
        return
    reference_forward = quant_linear.forward

    def forward(self, x):
        if self.backend == BACKEND:
            return b200_w4g64_linear(
                x, self.qweight, self.scales, self.zeros, self.bias,
                out_features=self.out_features, in_features=self.in_features,
                group_size=self.group_size, packing=self.packing,
            )
        return reference_forward(self, x)

    forward._b200_dispatch = True
    quant_linear.forward = forward


def _set_mlp_fusion(package: str, enabled: bool) -> None:
    name = f"{package}.model"
    if not enabled and name not in sys.modules:
        return
    mlp = importlib.import_module(name).QwenMLP
    if not getattr(mlp.forward, "_b200_fused", False):
        if not enabled:
            return
        reference_forward = mlp.forward

        def forward(self, x):
            gate, up = self.gate_proj, self.up_proj
            if type(self)._b200_fuse_mlp and gate.backend == BACKEND and up.backend == BACKEND:
                return self.down_proj(b200_w4g64_gate_up_silu(x, gate, up)).to(x.dtype)
            return reference_forward(self, x)

        forward._b200_fused = True
        mlp.forward = forward
    mlp._b200_fuse_mlp = enabled
