"""Run the reference's own Qwen2 model on the ``b200`` backend.

The model code is the reference project's, unchanged: ``QwenInt4ForCausalLM``
(src/qwen_int4/model.py:202), its KV cache and ``greedy_generate_cached``
(src/qwen_int4/generation.py:96). This module only

* finds the reference package (an installed ``qwen_int4``, or one installed
  with pip into ``<repo>/baseline/_ref``),
* registers the ``b200`` backend with it (``integration.register_with_reference``),
* builds a random-init, W4G64-RTN-quantised Qwen2-1.5B on a device (the
  batch-1 and batch-64 decode workloads; no checkpoint or network is needed).

Quantisation follows ``quantize_symmetric_rtn`` (src/qwen_int4/quantization.py:
87-111: per-row, per-64-group ``scale = amax / 7``, ``round(w / scale)`` clamped
to [-7, 7], canonical packing), computed with torch ops on the target device.
"""

from __future__ import annotations

import importlib
import sys
from pathlib import Path
from types import SimpleNamespace

import torch

from .integration import register_with_reference

REPO = Path(__file__).resolve().parent.parent

# Qwen2-1.5B architecture (the reference's configs/qwen2-1.5b/config.json).
QWEN2_1_5B = dict(
    hidden_size=1536, intermediate_size=8960, num_hidden_layers=28, num_attention_heads=12,
    num_key_value_heads=2, head_dim=128, vocab_size=151936, rms_norm_eps=1e-6,
    rope_theta=1_000_000.0, max_position_embeddings=32768, tie_word_embeddings=True,
)


def reference_package():
    """Import the reference ``qwen_int4`` package, or raise ImportError."""
    try:
        return importlib.import_module("qwen_int4")
    except ImportError:
        candidate = REPO / "baseline" / "_ref"
        if (candidate / "qwen_int4").is_dir() and str(candidate) not in sys.path:
            sys.path.insert(0, str(candidate))
        return importlib.import_module("qwen_int4")


def qwen2_config(**overrides) -> SimpleNamespace:
    cfg = dict(QWEN2_1_5B)
    cfg.update(overrides)
    return SimpleNamespace(**cfg)


def quantize_symmetric_rtn_torch(weight: torch.Tensor, group_size: int = 64):
    """W4 symmetric RTN on any device: (packed uint8 [N*K/2, 1], fp16 scales [N, K/group])."""
    n, k = weight.shape
    g = weight.to(torch.float32).reshape(n, k // group_size, group_size)
    scale = g.abs().amax(dim=-1) / 7.0
    scale = torch.where(scale == 0, torch.ones_like(scale), scale)
    codes = torch.round(g / scale.unsqueeze(-1)).clamp_(-7, 7).to(torch.int16).reshape(n, k)
    packed = ((codes[:, 0::2] & 0xF) | ((codes[:, 1::2] & 0xF) << 4)).to(torch.uint8)
    return packed.reshape(-1, 1).contiguous(), scale.to(torch.float16).contiguous()


def quantize_asymmetric_rtn_torch(weight: torch.Tensor, group_size: int = 64):
    """W4 asymmetric RTN on any device, as the reference's
    ``quantize_asymmetric_rtn`` (src/qwen_int4/quantization.py:114-162): per
    group, scale = max(hi - lo, 1e-5) / 15 with lo <= 0 <= hi, zero =
    clip(round(-lo / scale), 0, 15), code = clip(round(w / scale) + zero, 0,
    15); codes and zeros are stored shifted by -8 as signed INT4 (an odd zero
    count is padded with one zero nibble). Returns (packed uint8 [N*K/2, 1],
    fp16 scales [N, K/group], packed zeros uint8 [(N*G+1)//2, 1])."""
    n, k = weight.shape
    g = weight.to(torch.float32).reshape(n, k // group_size, group_size)
    lo = torch.clamp(g.amin(dim=-1), max=0.0)
    hi = torch.clamp(g.amax(dim=-1), min=0.0)
    scale = torch.clamp(hi - lo, min=1e-5) / 15.0
    uzero = torch.clamp(torch.round(-lo / scale), 0, 15)
    ucode = torch.clamp(torch.round(g / scale.unsqueeze(-1)) + uzero.unsqueeze(-1), 0, 15)
    codes = (ucode.to(torch.int16) - 8).reshape(n, k)
    zeros = (uzero.to(torch.int16) - 8).reshape(-1)
    if zeros.numel() % 2:
        zeros = torch.cat([zeros, zeros.new_zeros(1)])
    pack = lambda v: ((v[0::2] & 0xF) | ((v[1::2] & 0xF) << 4)).to(torch.uint8)
    packed = ((codes[:, 0::2] & 0xF) | ((codes[:, 1::2] & 0xF) << 4)).to(torch.uint8)
    return (packed.reshape(-1, 1).contiguous(), scale.to(torch.float16).contiguous(),
            pack(zeros).reshape(-1, 1).contiguous())


@torch.no_grad()
def build_random_qwen2(config=None, *, device="cuda", seed: int = 0, backend: str = "b200",
                       fuse_mlp: bool = False, fast_attention: bool = False):
    """Reference ``QwenInt4ForCausalLM`` with random W4G64 RTN weights on ``device``.

    Every QuantLinear gets ``quantize_symmetric_rtn(bf16(randn * 0.02))``,
    q/k/v biases ~N(0, 0.02), embeddings ~N(0, 0.02) (tied lm_head), norms 1.
    ``fuse_mlp`` and ``fast_attention`` are passed to ``register_with_reference``.
    """
    ref = reference_package()
    register_with_reference(ref.__name__, fuse_mlp=fuse_mlp, fast_attention=fast_attention)
    from qwen_int4.linear import QuantLinear
    from qwen_int4.model import QwenInt4ForCausalLM
    from qwen_int4.quantization import PackingFormat

    config = config or qwen2_config()
    gen = torch.Generator(device=device).manual_seed(seed)
    with torch.device(device):  # allocate the module's buffers directly on the device
        model = QwenInt4ForCausalLM(config, backend="torch", packing=PackingFormat.CANONICAL, group_size=64)
    model.model.embed_tokens.weight.copy_(
        (torch.randn(model.model.embed_tokens.weight.shape, device=device, generator=gen) * 0.02)
        .to(torch.bfloat16))
    for module in model.modules():
        if isinstance(module, QuantLinear):
            w = (torch.randn(module.out_features, module.in_features, device=device, generator=gen) * 0.02)
            qw, sc = quantize_symmetric_rtn_torch(w.to(torch.bfloat16).float())
            module.qweight.copy_(qw)
            module.scales.copy_(sc)
            module.zeros.zero_()
            if module.bias is not None:
                module.bias.copy_((torch.randn(module.out_features, device=device, generator=gen) * 0.02)
                                  .to(torch.bfloat16))
    model.set_backend(backend)
    return model.eval()
