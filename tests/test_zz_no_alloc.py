"""The allocation-free FP32 entry point (qi4_w4g64_linear_f32_noalloc), on a GPU.

It serves callers that cannot allocate device memory while serving a request
(fixed device-memory budgets, FFI hosts without a CUDA allocator); its
scratch is a fixed array in the library instead of a call-time allocation.
Checked here through the C ABI against the allocating entry point
(qi4_w4g64_linear_ex with the tensor-core kernel), on two calls in a row with
different inputs, within the tolerance of the other tensor-core tests
(2e-2 + 1 ulp of FP32 against each other; both compute the same sums).

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


def test_noalloc_matches_allocating_entry_point_on_two_calls(b200, cuda_device):
    mod, lib = _lib(b200)
    stream = torch.cuda.current_stream().cuda_stream
    n, k = 1536, 8960
    for call, (m, seed) in enumerate(((512, 1), (200, 2))):
        x, qw, sc, z, bias = _inputs(m, n, k, seed, cuda_device)
        ours = torch.empty(m, n, device=cuda_device, dtype=torch.float32)
        ref = torch.empty(m, n, device=cuda_device, dtype=torch.float32)
        rc = lib.qi4_w4g64_linear_f32_noalloc(x.data_ptr(), m, k, qw.data_ptr(), sc.data_ptr(), z.data_ptr(),
                                              bias.data_ptr(), BF16, ours.data_ptr(), n, stream)
        mod.check(rc, "qi4_w4g64_linear_f32_noalloc")
        rc = lib.qi4_w4g64_linear_ex(x.data_ptr(), F32, m, k, qw.data_ptr(), sc.data_ptr(), z.data_ptr(),
                                     bias.data_ptr(), BF16, ref.data_ptr(), n, stream, TC, 0)
        mod.check(rc, "qi4_w4g64_linear_ex")
        torch.cuda.synchronize()
        a, b = ours.cpu().numpy(), ref.cpu().numpy()
        ulp = np.exp2(np.floor(np.log2(np.maximum(np.abs(b), 2.0 ** -14))) - 23)
        assert np.all(np.abs(a - b) <= 2e-2 + ulp), f"call {call}: max diff {np.abs(a - b).max()}"
    assert lib.qi4_device_status(stream) == 0


def test_noalloc_rejects_inputs_beyond_its_scratch(b200, cuda_device):
    mod, lib = _lib(b200)
    m, n, k = 4096, 64, 8960  # M*K = 36.7 Mi elements > 8 Mi: refused before any launch
    x = torch.empty(1, dtype=torch.float32, device=cuda_device)
    qw = torch.empty(16, dtype=torch.uint8, device=cuda_device)
    sc = torch.empty(1, dtype=torch.float16, device=cuda_device)
    out = torch.empty(1, dtype=torch.float32, device=cuda_device)
    rc = lib.qi4_w4g64_linear_f32_noalloc(x.data_ptr(), m, k, qw.data_ptr(), sc.data_ptr(), None, None, NONE,
                                          out.data_ptr(), n, torch.cuda.current_stream().cuda_stream)
    assert rc == -3
    assert "fixed scratch" in mod.last_error()
