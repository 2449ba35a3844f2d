"""The allocation-free FP32 entry point (qi4_w4g64_linear_f32_noalloc), on a GPU.

It serves callers that cannot allocate device memory while serving a request
(fixed device-memory budgets, FFI hosts without a CUDA allocator); its
scratch is a fixed array in the library instead of a call-time allocation.
Checked here through the C ABI against the allocating entry point
(qi4_w4g64_linear_ex with the tensor-core kernel) and against the oracle, on
two calls in a row with different inputs and on an input that fills the
array exactly, within the tolerance of the other tensor-core tests (2e-2 + 1
ulp of FP32).

This file is named so that pytest collects it last.
"""

import importlib

import numpy as np
import pytest
import torch

from oracle import w4g64 as orc

pytestmark = pytest.mark.gpu

TC = 2
F32, BF16, NONE = 2, 1, -1


def _lib(b200):
    mod = importlib.import_module(b200.__name__ + "._lib")
    return mod, mod.load()


def _inputs(m, n, k, seed, dev):
    rng = np.random.default_rng(seed)
    qw, sc, z = orc.quantize_asymmetric_rtn(rng.standard_normal((n, k), dtype=np.float32) * 0.02)
    x = torch.from_numpy(rng.standard_normal((m, k), dtype=np.float32)).to(dev)
    bias = torch.from_numpy(rng.standard_normal(n, dtype=np.float32) * 0.1).to(torch.bfloat16).to(dev)
    return x, torch.from_numpy(qw).to(dev), torch.from_numpy(sc).to(dev), torch.from_numpy(z).to(dev), bias


def _call_both(lib, mod, x, qw, sc, z, bias, m, n, k, dev):
    stream = torch.cuda.current_stream().cuda_stream
    ours = torch.empty(m, n, device=dev, dtype=torch.float32)
    ref = torch.empty(m, n, device=dev, dtype=torch.float32)
    rc = lib.qi4_w4g64_linear_f32_noalloc(x.data_ptr(), m, k, qw.data_ptr(), sc.data_ptr(), z.data_ptr(),
                                          bias.data_ptr(), BF16, ours.data_ptr(), n, stream)
    mod.check(rc, "qi4_w4g64_linear_f32_noalloc")
    rc = lib.qi4_w4g64_linear_ex(x.data_ptr(), F32, m, k, qw.data_ptr(), sc.data_ptr(), z.data_ptr(),
                                 bias.data_ptr(), BF16, ref.data_ptr(), n, stream, TC, 0)
    mod.check(rc, "qi4_w4g64_linear_ex")
    torch.cuda.synchronize()
    return ours.cpu().numpy(), ref.cpu().numpy()


def _ulp32(v):
    return np.exp2(np.floor(np.log2(np.maximum(np.abs(v), 2.0 ** -14))) - 23)


def _oracle_budget_ok(got, x, qw, sc, z, bias, n, k):
    """Against the oracle (FP32 dequantise-then-matmul, f64 sums): the
    tensor-core tolerance of the other GPU tests, 2e-2 + 1 ulp of FP32."""
    ref = orc.linear(x.cpu().numpy(), qw.cpu().numpy(), sc.cpu().numpy(), z.cpu().numpy(),
                     bias.float().cpu().numpy(), out_features=n, in_features=k, accumulate="f64")
    err = np.abs(got - ref)
    return bool(np.all(err <= 2e-2 + _ulp32(ref))), float(err.max())


def test_noalloc_matches_allocating_entry_point_on_two_calls(b200, cuda_device):
    mod, lib = _lib(b200)
    n, k = 1536, 8960
    for call, (m, seed) in enumerate(((512, 1), (200, 2))):
        x, qw, sc, z, bias = _inputs(m, n, k, seed, cuda_device)
        a, b = _call_both(lib, mod, x, qw, sc, z, bias, m, n, k, cuda_device)
        assert np.all(np.abs(a - b) <= 2e-2 + _ulp32(b)), f"call {call}: max diff {np.abs(a - b).max()}"
        ok, worst = _oracle_budget_ok(a, x, qw, sc, z, bias, n, k)
        assert ok, f"call {call}: max error against the oracle {worst}"
    assert lib.qi4_device_status(torch.cuda.current_stream().cuda_stream) == 0


def test_noalloc_input_that_exactly_fills_the_scratch(b200, cuda_device):
    """M * K = 8 Mi elements fills the 32 MiB array exactly (hi copy in the
    first half, lo copy in the second): the last rows of x must land in the
    last bytes of the lo half and be read back from there."""
    mod, lib = _lib(b200)
    m, n, k = 1024, 128, 8192
    assert m * k == 8388608
    x, qw, sc, z, bias = _inputs(m, n, k, 3, cuda_device)
    a, b = _call_both(lib, mod, x, qw, sc, z, bias, m, n, k, cuda_device)
    assert np.all(np.abs(a - b) <= 2e-2 + _ulp32(b)), f"max diff {np.abs(a - b).max()}"
    ok, worst = _oracle_budget_ok(a, x, qw, sc, z, bias, n, k)
    assert ok, f"max error against the oracle {worst}"


@pytest.mark.parametrize("m,k", [(1025, 8192), (4096, 8960)])
def test_noalloc_rejects_inputs_beyond_its_scratch(b200, cuda_device, m, k):
    mod, lib = _lib(b200)
    n = 64  # M*K > 8 Mi elements: refused before any launch
    x = torch.empty(1, dtype=torch.float32, device=cuda_device)
    qw = torch.empty(16, dtype=torch.uint8, device=cuda_device)
    sc = torch.empty(1, dtype=torch.float16, device=cuda_device)
    out = torch.empty(1, dtype=torch.float32, device=cuda_device)
    rc = lib.qi4_w4g64_linear_f32_noalloc(x.data_ptr(), m, k, qw.data_ptr(), sc.data_ptr(), None, None, NONE,
                                          out.data_ptr(), n, torch.cuda.current_stream().cuda_stream)
    assert rc == -3
    assert "fixed scratch" in mod.last_error()
