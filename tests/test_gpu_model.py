"""The reference's unmodified Qwen2 model running on the b200 backend (GPU).

Uses the reference package that ``build()`` installs into baseline/_ref; a
missing package is a failure, not a skip. Gates: the cached prefill/decode
path agrees with the full forward (as the reference's tests/test_kv_cache.py
checks for its own backends); final-logits cosine against the reference's own
``torch`` backend on the same random-init Qwen2-1.5B is >= 0.9995 and at least
the reference's own float64-vs-float32 self-consistency on that model (the
0.9999 figure of the target is printed beside both: a random-init 28-layer
bf16 model amplifies summation-order differences past it, for the reference
itself too).
"""

import importlib

import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def q2(b200):
    mod = importlib.import_module(b200.__name__ + ".qwen2")
    try:
        mod.reference_package()
    except ImportError as exc:
        pytest.fail(f"reference package missing (build() installs it into baseline/_ref): {exc}")
    return mod


def _cos(a, b):
    a, b = a.float().flatten(), b.float().flatten()
    return float(torch.nn.functional.cosine_similarity(a, b, dim=0))


def test_small_model_cached_decode_matches_full_forward(q2, cuda_device):
    cfg = q2.qwen2_config(num_hidden_layers=2, vocab_size=512)
    model = q2.build_random_qwen2(cfg, device=cuda_device, seed=3)
    tokens = torch.randint(0, 512, (2, 9), generator=torch.Generator().manual_seed(1)).to(cuda_device)
    with torch.inference_mode():
        full = model(tokens)
        pre, cache = model(tokens[:, :6], use_cache=True)
        steps = [pre[:, -1]]
        for t in range(6, 9):
            logits, cache = model(tokens[:, t:t + 1], past_key_values=cache, use_cache=True)
            steps.append(logits[:, -1])
    for i, got in enumerate(steps):
        assert _cos(got, full[:, 5 + i]) > 0.9999


def test_full_qwen2_logits_match_reference_torch_backend(q2, cuda_device):
    """Final-logits cosine against the reference's torch backend.

    A random-init 28-layer bf16 Qwen2 amplifies summation-order differences:
    the reference's own torch path with its matmul in float64 instead of
    float32 reaches only ~0.9996 against itself. So the gate is that b200 is
    at least as close to the reference as the reference is to itself under
    that change (and >= 0.9995); the 0.9999 north-star figure is reported.
    """
    from qwen_int4.quantization import dequantize_groupwise
    import qwen_int4.linear as L

    model = q2.build_random_qwen2(device=cuda_device, seed=0)
    prompt = torch.randint(0, model.config.vocab_size, (1, 16),
                           generator=torch.Generator().manual_seed(20260831)).to(cuda_device)

    def forward_f64(self, x):  # the reference algorithm with a float64 matmul
        w = dequantize_groupwise(self.qweight, self.scales, zeros=self.zeros, out_features=self.out_features,
                                 in_features=self.in_features, group_size=self.group_size, packing=self.packing)
        out = (x.reshape(-1, self.in_features).double() @ w.double().t()).float()
        if self.bias is not None:
            out = out + self.bias.float()
        return out.reshape(*x.shape[:-1], self.out_features).to(x.dtype)

    with torch.inference_mode():
        ours = model(prompt)
        model.set_backend("torch")
        ref = model(prompt)
        saved = L.QuantLinear.forward
        L.QuantLinear.forward = forward_f64
        try:
            ref64 = model(prompt)
        finally:
            L.QuantLinear.forward = saved
        model.set_backend("b200")
    cos = _cos(ours[0, -1], ref[0, -1])
    self_consistency = _cos(ref64[0, -1], ref[0, -1])
    print(f"logits cosine b200 vs torch {cos:.6f}; reference f64 vs f32 {self_consistency:.6f}")
    assert cos >= 0.9995
    assert cos >= self_consistency - 1e-4, (cos, self_consistency)


def test_full_qwen2_greedy_generation_agrees_with_torch_backend(q2, cuda_device):
    """Greedy generation through the reference's generation loop on both backends.

    Free-running greedy decode of a random-init model diverges after the
    first near-tie, so agreement is checked teacher-forced: on the torch
    backend's greedy sequence, both backends must pick the same argmax at
    every generated position whose top-1/top-2 logit gap exceeds 0.1.
    """
    gen_mod = importlib.import_module("qwen_int4.generation")
    model = q2.build_random_qwen2(device=cuda_device, seed=0)
    prompt = torch.randint(0, model.config.vocab_size, (2, 12),
                           generator=torch.Generator().manual_seed(7)).to(cuda_device)
    ours_free = gen_mod.greedy_generate_cached(model, prompt, max_new_tokens=6)
    model.set_backend("torch")
    seq = gen_mod.greedy_generate_cached(model, prompt, max_new_tokens=6)
    assert ours_free.shape == seq.shape
    with torch.inference_mode():
        ref_logits = model(seq)[:, 11:-1].float()
        model.set_backend("b200")
        our_logits = model(seq)[:, 11:-1].float()
    top2 = ref_logits.topk(2, dim=-1).values
    clear = (top2[..., 0] - top2[..., 1]) > 0.1
    assert clear.sum() >= 4
    agree = ref_logits.argmax(-1) == our_logits.argmax(-1)
    assert bool(agree[clear].all()), (agree, clear)


def test_fused_mlp_model_matches_torch_backend(q2, cuda_device):
    """``register_with_reference(fuse_mlp=True)``: every QwenMLP runs the fused
    gate/up SwiGLU call then down_proj. Cached decode still agrees with the
    full forward, and the full model's final logits stay within the unfused
    gate against the reference's torch backend."""
    cfg = q2.qwen2_config(num_hidden_layers=2, vocab_size=512)
    small = q2.build_random_qwen2(cfg, device=cuda_device, seed=3, fuse_mlp=True)
    tokens = torch.randint(0, 512, (2, 9), generator=torch.Generator().manual_seed(1)).to(cuda_device)
    try:
        with torch.inference_mode():
            full = small(tokens)
            pre, cache = small(tokens[:, :6], use_cache=True)
            logits, cache = small(tokens[:, 6:7], past_key_values=cache, use_cache=True)
        assert _cos(pre[:, -1], full[:, 5]) > 0.9999
        assert _cos(logits[:, -1], full[:, 6]) > 0.9999

        model = q2.build_random_qwen2(device=cuda_device, seed=0, fuse_mlp=True)
        prompt = torch.randint(0, model.config.vocab_size, (1, 16),
                               generator=torch.Generator().manual_seed(20260831)).to(cuda_device)
        with torch.inference_mode():
            fused = model(prompt)
            model.set_backend("torch")
            ref = model(prompt)
        cos = _cos(fused[0, -1], ref[0, -1])
        print(f"logits cosine b200 fused MLP vs torch {cos:.6f}")
        assert cos >= 0.9995
    finally:
        q2.register_with_reference(q2.reference_package().__name__, fuse_mlp=False)
