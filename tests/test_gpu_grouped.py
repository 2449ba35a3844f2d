"""Grouped linears sharing one activation block (qi4_w4g64_linear_multi) on a GPU.

Decode sizes (M <= 16) run as one GEMV launch over all matrices; prefill sizes
as one tensor-core launch per matrix. Every output is checked against the
oracle's dequantise-then-matmul at the tolerance of the single-linear path
(1e-3 + 1 ulp for the GEMV, 2e-2 + 1 ulp for the tensor core).
"""

from types import SimpleNamespace

import numpy as np
import pytest
import torch

from oracle import w4g64 as orc
from test_gpu_parity import assert_linear_close, to_dev

pytestmark = pytest.mark.gpu


def _layer(n, k, seed, dev, asym, bias_dtype=None):
    rng = np.random.default_rng(seed)
    w = rng.standard_normal((n, k), dtype=np.float32) * 0.02
    if asym:
        qw, sc, z = orc.quantize_asymmetric_rtn(w)
    else:
        qw, sc = orc.quantize_symmetric_rtn(w)
        z = np.zeros(((n * (k // 64) + 1) // 2, 1), dtype=np.uint8)
    bias = None
    if bias_dtype is not None:
        bias = torch.from_numpy(rng.standard_normal(n, dtype=np.float32) * 0.05).to(bias_dtype)
    return SimpleNamespace(qweight=to_dev(qw, dev), scales=to_dev(sc, dev), zeros=to_dev(z, dev),
                           bias=None if bias is None else bias.to(dev), in_features=k, out_features=n,
                           np=(qw, sc, z, None if bias is None else bias.float().numpy()))


def _check(outs, layers, x, atol):
    for o, l in zip(outs, layers):
        qw, sc, z, b = l.np
        ref = orc.linear(x.float().cpu().numpy().reshape(-1, l.in_features), qw, sc, z, b,
                         out_features=l.out_features, in_features=l.in_features, accumulate="f64")
        assert o.shape == (*x.shape[:-1], l.out_features) and o.dtype == x.dtype
        assert_linear_close(o.reshape(-1, l.out_features), ref, atol, f"grouped n={l.out_features}")


@pytest.mark.parametrize("m", [1, 3, 16])
def test_qkv_shapes_with_bias_in_one_launch(b200, cuda_device, m):
    layers = [_layer(n, 1536, 10 + i, cuda_device, False, torch.bfloat16) for i, n in enumerate((1536, 256, 256))]
    x = torch.randn(m, 1536, generator=torch.Generator().manual_seed(m)).to(torch.bfloat16).to(cuda_device)
    _check(b200.b200_w4g64_linear_multi(x, layers), layers, x, 1e-3)


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16, torch.float32])
def test_gate_up_asymmetric_all_dtypes(b200, cuda_device, dtype):
    layers = [_layer(8960, 1536, 20 + i, cuda_device, True) for i in range(2)]
    x = torch.randn(2, 1536, generator=torch.Generator().manual_seed(5)).to(dtype).to(cuda_device)
    _check(b200.b200_w4g64_linear_multi(x, layers), layers, x, 1e-3)


@pytest.mark.parametrize("ns", [(7, 100, 300), (16, 17), (1000,)])
def test_ragged_row_counts_across_matrices(b200, cuda_device, ns):
    """Tile boundaries between matrices: row counts that are not multiples of the tile."""
    layers = [_layer(n, 192, 30 + i, cuda_device, True, torch.float32) for i, n in enumerate(ns)]
    x = torch.randn(1, 2, 192, generator=torch.Generator().manual_seed(7)).to(torch.bfloat16).to(cuda_device)
    _check(b200.b200_w4g64_linear_multi(x, layers), layers, x, 1e-3)


def test_long_rows_with_k_split_and_prefill_sizes(b200, cuda_device):
    layers = [_layer(n, 8960, 40 + i, cuda_device, True) for i, n in enumerate((1536, 512))]
    for m, atol in ((8, 1e-3), (64, 2e-2)):
        x = torch.randn(m, 8960, generator=torch.Generator().manual_seed(m)).to(torch.bfloat16).to(cuda_device)
        _check(b200.b200_w4g64_linear_multi(x, layers), layers, x, atol)


def test_grouped_equals_single_calls_for_the_same_plan(b200, cuda_device):
    """q/k/v through one launch and through three: same tiles, same sums."""
    from importlib import import_module

    lib = import_module(b200.__name__ + "._lib").load()
    layers = [_layer(n, 1536, 50 + i, cuda_device, False, torch.bfloat16) for i, n in enumerate((1536, 256, 256))]
    x = torch.randn(1, 1536, generator=torch.Generator().manual_seed(9)).to(torch.bfloat16).to(cuda_device)
    assert lib.qi4_gemv_mma_plan_override(16, 1, 8) == 0
    try:
        grouped = b200.b200_w4g64_linear_multi(x, layers)
        single = [b200.b200_w4g64_linear(x, l.qweight, l.scales, l.zeros, l.bias, out_features=l.out_features,
                                         in_features=1536, group_size=64, packing="canonical", algo=1)
                  for l in layers]
    finally:
        lib.qi4_gemv_mma_plan_override(0, 0, 0)
    for g, s in zip(grouped, single):
        assert torch.equal(g, s)
    assert lib.qi4_device_status(torch.cuda.current_stream().cuda_stream) == 0


def _swiglu_ref(x, gate, up):
    """silu(round(gate(x))) * round(up(x)) in float64 from the oracle, the
    rounding to x's dtype standing in for QuantLinear's output dtype."""
    xs = x.float().cpu().numpy().reshape(-1, gate.in_features)
    outs = []
    for l in (gate, up):
        qw, sc, z, _ = l.np
        y = orc.linear(xs, qw, sc, z, None, out_features=l.out_features, in_features=l.in_features,
                       accumulate="f64")
        outs.append(torch.from_numpy(y).to(x.dtype).double().numpy())
    g, u = outs
    return g / (1.0 + np.exp(-g)) * u, g, u


def _swiglu_budget(ref, g, u, dtype, tensor_cores):
    # One rounding of g or u to x's dtype may land on the neighbouring value
    # (the kernel's and the float64 oracle's sums differ far below that step):
    # d(silu(g) u) <= 1.1 |u| dg + |g| du, dg and du one step each.
    step = {torch.bfloat16: 2.0 ** -7, torch.float16: 2.0 ** -10, torch.float32: 1e-5}[dtype]
    budget = 1e-3 + step * (np.abs(ref) + 2.1 * np.abs(g * u))
    if tensor_cores:
        # g and u carry the GEMM tolerance (2e-2 absolute: the weight rounded once).
        budget = budget + 2e-2 * (1.1 * np.abs(u) + np.abs(g) + 2e-2)
    return budget


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("m", [1, 5, 16, 40])
def test_fused_gate_up_silu_matches_the_reference_composition(b200, cuda_device, dtype, m):
    from importlib import import_module

    gate, up = (_layer(8960 if m < 40 else 1000, 1536, 60 + i, cuda_device, i == 1) for i in range(2))
    x = torch.randn(m, 1536, generator=torch.Generator().manual_seed(m)).to(dtype).to(cuda_device)
    got = b200.b200_w4g64_gate_up_silu(x, gate, up)
    assert got.dtype == torch.float32 and got.shape == (m, gate.out_features)
    ref, g, u = _swiglu_ref(x, gate, up)
    err = np.abs(got.cpu().numpy().astype(np.float64) - ref)
    assert np.all(err <= _swiglu_budget(ref, g, u, dtype, m > 16)), f"max err {err.max():.3e}"
    lib = import_module(b200.__name__ + "._lib").load()
    assert lib.qi4_device_status(torch.cuda.current_stream().cuda_stream) == 0


def test_fused_gate_up_silu_ragged_rows_and_k(b200, cuda_device):
    gate, up = (_layer(100, 192, 70 + i, cuda_device, True) for i in range(2))
    x = torch.randn(2, 3, 192, generator=torch.Generator().manual_seed(3)).to(torch.bfloat16).to(cuda_device)
    got = b200.b200_w4g64_gate_up_silu(x, gate, up)
    ref, g, u = _swiglu_ref(x, gate, up)
    assert got.shape == (2, 3, 100)
    err = np.abs(got.reshape(-1, 100).cpu().numpy().astype(np.float64) - ref)
    assert np.all(err <= _swiglu_budget(ref, g, u, torch.bfloat16, False)), f"max err {err.max():.3e}"
