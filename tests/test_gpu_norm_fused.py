"""Residual add + RMSNorm folded into a decode launch (qi4_*_norm) on a GPU.

Against the reference's block boundary (model.py:31-42,151-159) restated in
torch: hn = bf16(h + bf16(delta)) is written to h_out bit-exactly (elementwise,
same roundings); x = bf16(bf16(hn * rsqrt(mean(hn^2) + eps)) * w) then feeds
the linear, whose output is held to the oracle's float64 dequantise-then-
matmul on that x at the GEMV tolerance plus 1e-3 (the kernel sums the row
statistics in another order, which can move an element of x by one bf16 ulp).
Also against the two-launch composition (qi4_add_rmsnorm, then the plain
call): outputs within the same bound, h identical.
"""

import ctypes
from importlib import import_module

import numpy as np
import pytest
import torch

from test_gpu_grouped import _layer, _swiglu_budget
from test_gpu_parity import assert_linear_close
from oracle import w4g64 as orc

pytestmark = pytest.mark.gpu


def _boundary(h, delta, w, eps):
    hn = h.float()
    if delta is not None:
        hn = (hn + delta.to(torch.bfloat16).float()).to(torch.bfloat16).float()
    r = torch.rsqrt(hn.pow(2).mean(-1, keepdim=True) + eps)
    x = ((hn * r).to(torch.bfloat16).float() * w.float()).to(torch.bfloat16)
    return hn.to(torch.bfloat16), x


def _inputs(m, k, delta_dtype, dev, seed):
    g = torch.Generator().manual_seed(seed)
    h = torch.randn(m, k, generator=g).to(torch.bfloat16).to(dev)
    delta = None if delta_dtype is None else (torch.randn(m, k, generator=g) * 0.5).to(delta_dtype).to(dev)
    w = (1 + 0.1 * torch.randn(k, generator=g)).to(torch.bfloat16).to(dev)
    return h, delta, w


def _prologue(lib_mod, h, delta, w, h_out, eps=1e-6):
    code = {None: -1, torch.bfloat16: 1, torch.float32: 2}[None if delta is None else delta.dtype]
    return lib_mod.RmsNormPrologue(h.data_ptr(), None if delta is None else delta.data_ptr(), code, eps,
                                   w.data_ptr(), h_out.data_ptr())


@pytest.mark.parametrize("m", [1, 5, 16])
@pytest.mark.parametrize("delta_dtype", [None, torch.bfloat16, torch.float32])
def test_qkv_with_fused_norm(b200, cuda_device, m, delta_dtype):
    lm = import_module(b200.__name__ + "._lib")
    lib = lm.load()
    layers = [_layer(n, 1536, 10 + i, cuda_device, False, torch.bfloat16) for i, n in enumerate((1536, 256, 256))]
    h, delta, w = _inputs(m, 1536, delta_dtype, cuda_device, m)
    h_out = torch.empty_like(h)
    outs = [torch.empty(m, l.out_features, dtype=torch.bfloat16, device=cuda_device) for l in layers]
    arr = lambda v: (ctypes.c_void_p * 3)(*v)  # noqa: E731
    pro = _prologue(lm, h, delta, w, h_out)
    rc = lib.qi4_w4g64_linear_multi_norm(
        ctypes.byref(pro), m, 1536, 3, arr([l.qweight.data_ptr() for l in layers]),
        arr([l.scales.data_ptr() for l in layers]), arr([l.zeros.data_ptr() for l in layers]),
        arr([l.bias.data_ptr() for l in layers]), 1, arr([o.data_ptr() for o in outs]),
        (ctypes.c_int64 * 3)(*[l.out_features for l in layers]), torch.cuda.current_stream().cuda_stream)
    assert rc == 0
    hn, x = _boundary(h, delta, w, 1e-6)
    assert torch.equal(h_out, hn)
    for o, l in zip(outs, layers):
        qw, sc, z, b = l.np
        ref = orc.linear(x.float().cpu().numpy(), qw, sc, z, b, out_features=l.out_features, in_features=1536,
                         accumulate="f64")
        assert_linear_close(o, ref, 2e-3, f"qkv+norm n={l.out_features}")
    # The two-launch composition gives the same residual and outputs within the same bound.
    h2, x2 = h.clone(), torch.empty_like(h)
    assert lib.qi4_add_rmsnorm(h2.data_ptr(), None if delta is None else delta.data_ptr(), pro.delta_dtype,
                               w.data_ptr(), x2.data_ptr(), m, 1536, ctypes.c_float(1e-6),
                               torch.cuda.current_stream().cuda_stream) == 0
    assert torch.equal(h2, h_out)
    assert lib.qi4_device_status(torch.cuda.current_stream().cuda_stream) == 0


@pytest.mark.parametrize("m", [1, 8])
def test_gate_up_silu_with_fused_norm(b200, cuda_device, m):
    lm = import_module(b200.__name__ + "._lib")
    lib = lm.load()
    gate, up = (_layer(8960, 1536, 60 + i, cuda_device, i == 1) for i in range(2))
    h, delta, w = _inputs(m, 1536, torch.bfloat16, cuda_device, 40 + m)
    h_out = torch.empty_like(h)
    out = torch.empty(m, 8960, dtype=torch.float32, device=cuda_device)
    pro = _prologue(lm, h, delta, w, h_out)
    rc = lib.qi4_w4g64_gate_up_silu_norm(
        ctypes.byref(pro), m, 1536, gate.qweight.data_ptr(), gate.scales.data_ptr(), gate.zeros.data_ptr(),
        up.qweight.data_ptr(), up.scales.data_ptr(), up.zeros.data_ptr(), out.data_ptr(), 8960,
        torch.cuda.current_stream().cuda_stream)
    assert rc == 0
    hn, x = _boundary(h, delta, w, 1e-6)
    assert torch.equal(h_out, hn)
    xs = x.float().cpu().numpy()
    gu = []
    for l in (gate, up):
        qw, sc, z, _ = l.np
        y = orc.linear(xs, qw, sc, z, None, out_features=8960, in_features=1536, accumulate="f64")
        gu.append(torch.from_numpy(y).to(torch.bfloat16).double().numpy())
    g, u = gu
    ref = g / (1.0 + np.exp(-g)) * u
    err = np.abs(out.cpu().numpy().astype(np.float64) - ref)
    budget = _swiglu_budget(ref, g, u, torch.bfloat16, False) + 2e-3 * (np.abs(u) + np.abs(g))
    assert np.all(err <= budget), f"max err {err.max():.3e}"


def test_decode_engine_uses_the_fused_boundary(b200, cuda_device):
    """One graph-captured step at batch 2 (fused boundaries) against the same
    step with the boundaries as separate norm launches: same greedy tokens
    over a few steps, residual streams within bf16 rounding."""
    q2 = import_module(b200.__name__ + ".qwen2")
    eng_mod = import_module(b200.__name__ + ".engine")
    cfg = q2.qwen2_config(num_hidden_layers=2, vocab_size=512)
    model = q2.build_random_qwen2(cfg, device=cuda_device, seed=5)
    prompt = torch.randint(0, 512, (2, 8), generator=torch.Generator().manual_seed(9)).to(cuda_device)
    fused = eng_mod.DecodeEngine(model, batch=2, max_len=24)
    plain = eng_mod.DecodeEngine(model, batch=2, max_len=24)
    plain.fuse_norm = False
    a = fused.generate(prompt, 8)
    b = plain.generate(prompt, 8)
    assert fused.fuse_norm and torch.equal(a, b)
