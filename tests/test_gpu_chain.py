"""Persistent decode chain (qi4_chain_*) on a GPU.

Every stage output is checked against the oracle's dequantise-then-matmul at
the tolerance of the decode GEMV (1e-3 + 1 ulp of the output dtype), the
SwiGLU stage against the reference MLP's composition with the same budget as
the fused gate/up tests. A Qwen2-1.5B two-layer chain is checked stage by
stage against the per-launch kernels on the chain's own intermediate inputs,
and repeated runs must be bit-identical (deterministic reduction, counters
reset between launches).
"""

import importlib
from types import SimpleNamespace

import numpy as np
import pytest
import torch

from oracle import w4g64 as orc
from test_gpu_grouped import _layer, _swiglu_budget, _swiglu_ref
from test_gpu_parity import assert_linear_close

pytestmark = pytest.mark.gpu


def _chain_mod(b200):
    return importlib.import_module(b200.__name__ + ".chain")


def _weights(mod, layer, symmetric):
    return mod.Weights(layer.qweight, layer.scales, None if symmetric else layer.zeros, layer.bias,
                       layer.out_features)


def _oracle(x, layer):
    qw, sc, z, b = layer.np
    return orc.linear(x.float().cpu().numpy().reshape(-1, layer.in_features), qw, sc, z, b,
                      out_features=layer.out_features, in_features=layer.in_features, accumulate="f64")


def _status(b200):
    lib = importlib.import_module(b200.__name__ + "._lib").load()
    return lib.qi4_device_status(torch.cuda.current_stream().cuda_stream)


@pytest.mark.parametrize("m", [1, 3, 8])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
def test_single_stage_three_matrices_match_oracle(b200, cuda_device, m, dtype):
    mod = _chain_mod(b200)
    asym = dtype == torch.float16
    layers = [_layer(n, 1536, 30 + i, cuda_device, asym, torch.bfloat16) for i, n in enumerate((1536, 256, 256))]
    x = torch.randn(m, 1536, generator=torch.Generator().manual_seed(m)).to(dtype).to(cuda_device)
    outs = [torch.empty(m, l.out_features, dtype=dtype, device=cuda_device) for l in layers]
    chain = mod.DecodeChain([mod.Stage(x, [_weights(mod, l, not asym) for l in layers], outs)], m)
    chain.run()
    torch.cuda.synchronize()
    for o, l in zip(outs, layers):
        assert_linear_close(o, _oracle(x, l), 1e-3, f"chain n={l.out_features}")
    assert _status(b200) == 0


@pytest.mark.parametrize("n,k", [(100, 192), (8, 64), (1000, 8960), (17, 1280)])
def test_ragged_rows_and_long_k(b200, cuda_device, n, k):
    """Row counts that are not whole 16-row blocks, one-group rows, and rows
    shared by several CTAs (K = 8960 at N = 1000)."""
    mod = _chain_mod(b200)
    layer = _layer(n, k, 40, cuda_device, True, torch.float32)
    for m in (1, 2):
        x = torch.randn(m, k, generator=torch.Generator().manual_seed(k + m)).to(torch.bfloat16).to(cuda_device)
        out = torch.empty(m, n, dtype=torch.bfloat16, device=cuda_device)
        chain = mod.DecodeChain([mod.Stage(x, [_weights(mod, layer, False)], [out])], m)
        chain.run()
        torch.cuda.synchronize()
        assert_linear_close(out, _oracle(x, layer), 1e-3, f"chain n={n} k={k} m={m}")
    assert _status(b200) == 0


@pytest.mark.parametrize("m", [1, 4])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_swiglu_stage_matches_reference_composition(b200, cuda_device, m, dtype):
    mod = _chain_mod(b200)
    gate, up = (_layer(8960, 1536, 60 + i, cuda_device, i == 1) for i in range(2))
    x = torch.randn(m, 1536, generator=torch.Generator().manual_seed(m)).to(dtype).to(cuda_device)
    out = torch.empty(m, 8960, dtype=torch.float32, device=cuda_device)
    chain = mod.DecodeChain([mod.Stage(x, [_weights(mod, gate, False), _weights(mod, up, False)], [out],
                                       swiglu=True)], m)
    chain.run()
    torch.cuda.synchronize()
    ref, g, u = _swiglu_ref(x, gate, up)
    err = np.abs(out.cpu().numpy().astype(np.float64) - ref)
    assert np.all(err <= _swiglu_budget(ref, g, u, dtype, False)), f"max err {err.max():.3e}"
    assert _status(b200) == 0


def _qwen_layer(seed, dev):
    mk = lambda n, k, s, bias: _layer(n, k, seed * 10 + s, dev, False, torch.bfloat16 if bias else None)  # noqa
    attn = SimpleNamespace(q_proj=mk(1536, 1536, 0, True), k_proj=mk(256, 1536, 1, True),
                           v_proj=mk(256, 1536, 2, True), o_proj=mk(1536, 1536, 3, False))
    mlp = SimpleNamespace(gate_proj=mk(8960, 1536, 4, False), up_proj=mk(8960, 1536, 5, False),
                          down_proj=mk(1536, 8960, 6, False))
    return SimpleNamespace(self_attn=attn, mlp=mlp)


def test_two_qwen2_layers_stagewise_against_per_launch_kernels(b200, cuda_device):
    """The chain of two Qwen2-1.5B decoder layers (8 stages): each stage's
    output equals the per-launch kernels' output on the chain's own input for
    that stage (GEMV tolerance), and the down_proj output also the oracle's;
    three runs in a row give bit-identical results."""
    mod = _chain_mod(b200)
    layers = [_qwen_layer(s, cuda_device) for s in (1, 2)]
    x = torch.randn(1, 1536, generator=torch.Generator().manual_seed(9)).to(torch.bfloat16).to(cuda_device)
    stages, bufs = mod.decoder_linear_stages(layers, x)
    chain = mod.DecodeChain(stages, 1)
    chain.run()
    torch.cuda.synchronize()
    first = {li: {k: v.clone() for k, v in bufs[li].items()} for li in (0, 1)}
    for _ in range(2):
        chain.run()
    torch.cuda.synchronize()
    for li in (0, 1):
        for key, t in bufs[li].items():
            assert torch.equal(t, first[li][key]), f"layer {li} {key} differs between runs"
    cur = x
    for li, layer in enumerate(layers):
        b = bufs[li]
        a, f = layer.self_attn, layer.mlp
        for name, lin in (("q", a.q_proj), ("k", a.k_proj), ("v", a.v_proj)):
            want = b200.b200_w4g64_linear(cur, lin.qweight, lin.scales, lin.zeros, lin.bias,
                                          out_features=lin.out_features, in_features=1536, group_size=64,
                                          packing="canonical")
            assert_linear_close(b[name], want.float().cpu().numpy(), 1e-3, f"layer {li} {name}")
        want = b200.b200_w4g64_linear(b["q"], a.o_proj.qweight, a.o_proj.scales, a.o_proj.zeros, None,
                                      out_features=1536, in_features=1536, group_size=64, packing="canonical")
        assert_linear_close(b["o"], want.float().cpu().numpy(), 1e-3, f"layer {li} o")
        ref, g, u = _swiglu_ref(b["o"], f.gate_proj, f.up_proj)
        err = np.abs(b["h"].cpu().numpy().astype(np.float64) - ref)
        assert np.all(err <= _swiglu_budget(ref, g, u, torch.bfloat16, False)), f"layer {li} h {err.max():.3e}"
        assert_linear_close(b["y"], _oracle(b["h"], f.down_proj), 1e-3, f"layer {li} down")
        cur = b["y"]
    info = chain.info()
    assert info["stages"] == 8 and info["ctas"] == torch.cuda.get_device_properties(0).multi_processor_count
    assert _status(b200) == 0


def test_chain_rejects_bad_stages(b200, cuda_device):
    mod = _chain_mod(b200)
    layer = _layer(64, 128, 1, cuda_device, False)
    x = torch.randn(9, 128, device=cuda_device).to(torch.bfloat16)
    out = torch.empty(9, 64, dtype=torch.bfloat16, device=cuda_device)
    with pytest.raises(ValueError, match="M <= 8|SHAPE"):
        mod.DecodeChain([mod.Stage(x, [_weights(mod, layer, True)], [out])], 9)
    x1 = torch.randn(1, 96, device=cuda_device).to(torch.bfloat16)
    with pytest.raises(ValueError, match="multiple of 64"):
        mod.DecodeChain([mod.Stage(x1, [_weights(mod, layer, True)], [out[:1]])], 1)
