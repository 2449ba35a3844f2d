"""GPU parity of the tcgen05 dequant-GEMM (prefill path) against the oracle.

Tolerance: |out - ref| <= 2e-2 + 1 ulp of the output
dtype, ref = FP32 dequantise-then-matmul of the same bf16/fp16 activations
(summed in float64 here). The tensor core sees the dequantised weight rounded
once to bf16 (fp16 for fp16 activations), which is the only difference.
"""

import numpy as np
import pytest
import torch

from oracle import w4g64 as orc

import _golden as G
from test_gpu_parity import assert_linear_close, to_dev

pytestmark = pytest.mark.gpu

TC = 2
QWEN_SHAPES = {"q": (1536, 1536), "k": (1536, 256), "o": (1536, 1536), "gate": (1536, 8960),
               "down": (8960, 1536)}
_W = {}


def _weights(k, n, kind, seed):
    key = (k, n, kind, seed)
    if key not in _W:
        rng = np.random.default_rng(seed)
        w = (rng.standard_normal((n, k), dtype=np.float32) * 0.02)
        if kind == "sym":
            qw, sc = orc.quantize_symmetric_rtn(w)
            z = np.zeros(((n * (k // 64) + 1) // 2, 1), dtype=np.uint8)
        else:
            qw, sc, z = orc.quantize_asymmetric_rtn(w)
        _W[key] = (qw, sc, z)
    return _W[key]


def _run(b200, dev, x, qw, sc, z, bias, n, k, algo=TC):
    return b200.b200_w4g64_linear(
        x.to(dev), to_dev(qw, dev), to_dev(sc, dev), to_dev(z, dev), None if bias is None else bias.to(dev),
        out_features=n, in_features=k, group_size=64, packing="canonical", algo=algo)


def _ref(x, qw, sc, z, bias, n, k):
    acc = "f64" if x.shape[0] * n * k <= 2e9 else "f32"
    return orc.linear(x.float().numpy(), qw, sc, z, None if bias is None else bias.float().numpy(),
                      out_features=n, in_features=k, accumulate=acc)


@pytest.mark.parametrize("m", [17, 64, 128, 300, 512])
@pytest.mark.parametrize("name", list(QWEN_SHAPES))
def test_tc_qwen_shapes_bf16(b200, cuda_device, name, m):
    k, n = QWEN_SHAPES[name]
    qw, sc, z = _weights(k, n, "sym", 31)
    g = torch.Generator().manual_seed(7 + m)
    x = torch.randn(m, k, generator=g).to(torch.bfloat16)
    bias = (torch.randn(n, generator=g) * 0.02).to(torch.bfloat16) if name in ("q", "k") else None
    got = _run(b200, cuda_device, x, qw, sc, z, bias, n, k)
    assert_linear_close(got, _ref(x, qw, sc, z, bias, n, k), 2e-2, f"tc {name} m={m}")


@pytest.mark.parametrize("m", [128, 2048])
def test_tc_awq_down_proj_config2(b200, cuda_device, m):
    qw, sc, z = G.cfg2_weights()
    chan = torch.from_numpy(G.arrays()["cfg2_chan"])
    x = (torch.randn(m, 8960, generator=torch.Generator().manual_seed(500 + m)) / chan).to(torch.bfloat16)
    got = _run(b200, cuda_device, x, qw, sc, z, None, 1536, 8960)
    assert_linear_close(got, _ref(x, qw, sc, z, None, 1536, 8960), 2e-2, f"tc awq down m={m}")


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize(("m", "n", "k"), [(1, 128, 64), (100, 1000, 192), (257, 136, 320), (2048, 8960, 1536)])
def test_tc_ragged_shapes(b200, cuda_device, dtype, m, n, k):
    qw, sc, z = _weights(k, n, "asym", 41)
    g = torch.Generator().manual_seed(m * 7 + n)
    x = torch.randn(m, k, generator=g).to(dtype)
    bias = (torch.randn(n, generator=g) * 0.05).to(dtype)
    got = _run(b200, cuda_device, x, qw, sc, z, bias, n, k)
    assert got.dtype == dtype
    assert_linear_close(got, _ref(x, qw, sc, z, bias, n, k), 2e-2, f"tc ragged {m}x{n}x{k} {dtype}")


@pytest.mark.parametrize("key", G.LINEAR_CASES)
def test_tc_on_reference_golden_cases(b200, cuda_device, key):
    c = G.linear_case(key)
    x = c["x"]
    got = b200.b200_w4g64_linear(
        x.to(cuda_device), to_dev(c["qweight"], cuda_device), to_dev(c["scales"], cuda_device),
        to_dev(c["zeros"], cuda_device), None if c["bias"] is None else c["bias"].to(cuda_device),
        out_features=c["n"], in_features=c["k"], group_size=64, packing="canonical", algo=TC)
    exp = c["expected"]
    rtol, atol = (0.02, 0.25) if exp.dtype == torch.bfloat16 else (0.01, 0.0625)
    torch.testing.assert_close(got.cpu(), exp, rtol=rtol, atol=atol)


def test_auto_dispatch_uses_tc_for_large_m_and_status_is_clean(b200, cuda_device):
    from importlib import import_module

    lib = import_module(b200.__name__ + "._lib").load()
    k, n = 1536, 256
    qw, sc, z = _weights(k, n, "sym", 3)
    x = torch.randn(96, k, generator=torch.Generator().manual_seed(3)).to(torch.bfloat16)
    auto = _run(b200, cuda_device, x, qw, sc, z, None, n, k, algo=0)
    tc = _run(b200, cuda_device, x, qw, sc, z, None, n, k, algo=TC)
    assert torch.equal(auto, tc)
    assert lib.qi4_device_status(torch.cuda.current_stream().cuda_stream) == 0


@pytest.mark.parametrize(("m", "n", "k"), [(17, 256, 1536), (200, 1000, 192), (512, 1536, 8960)])
def test_tc_fp32_activations_down_proj_path(b200, cuda_device, m, n, k):
    """FP32 activations (the model's down_proj input) on the tensor-core path.

    x is split into bf16 hi + lo (16 significant bits) and both halves go
    through the MMA; the output is FP32 like the reference's for FP32 input.
    """
    qw, sc, z = _weights(k, n, "asym", 61)
    x = torch.randn(m, k, generator=torch.Generator().manual_seed(m + k)) * 0.5
    got = _run(b200, cuda_device, x, qw, sc, z, None, n, k)
    assert got.dtype == torch.float32
    assert_linear_close(got, _ref(x, qw, sc, z, None, n, k), 2e-2, f"tc fp32 {m}x{n}x{k}")


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize(("bn", "ks"), [(32, 2), (64, 2), (64, 3), (64, 5), (64, 8), (128, 4), (128, 7)])
def test_tc_k_split_clusters(b200, cuda_device, bn, ks, dtype):
    """Every tile width and cluster size of the K split (forced through the
    plan override): the cluster's partial tiles summed over distributed
    shared memory, rows shared out in multiples of 4, bias added once; a
    ragged N and a K whose boxes do not divide evenly over the cluster."""
    from importlib import import_module

    lib = import_module(b200.__name__ + "._lib").load()
    m, n, k = 70, 1000, 8960 - 64 * 5
    qw, sc, z = _weights(k, n, "asym", 71)
    g = torch.Generator().manual_seed(bn * 10 + ks)
    x = torch.randn(m, k, generator=g).to(dtype)
    bias = (torch.randn(n, generator=g) * 0.05).to(torch.bfloat16) if dtype == torch.bfloat16 else None
    assert lib.qi4_gemm_tc_plan_override(bn, ks) == 0
    try:
        got = _run(b200, cuda_device, x, qw, sc, z, bias, n, k)
        torch.cuda.synchronize()
    finally:
        lib.qi4_gemm_tc_plan_override(0, 0)
    assert lib.qi4_device_status(torch.cuda.current_stream().cuda_stream) == 0
    assert_linear_close(got, _ref(x, qw, sc, z, bias, n, k), 2e-2, f"tc k-split bn={bn} ks={ks} {dtype}")
