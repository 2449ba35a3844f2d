"""The C++ fast path of b200_w4g64_linear against the ctypes path (GPU).

Both end in the same C ABI call, so their outputs must be bit-identical for
every activation dtype, bias dtype, leading shape and memory layout the
reference's QuantLinear hands over (src/qwen_int4/linear.py:62-72,
backends.py:73-98).
"""

import importlib

import pytest
import torch

from oracle import w4g64 as orc

pytestmark = pytest.mark.gpu


def _weights(device, n, k, seed):
    g = torch.Generator().manual_seed(seed)
    w = (torch.randn(n, k, generator=g) * 0.02).numpy()
    qw, sc, z = orc.quantize_asymmetric_rtn(w)
    return tuple(torch.from_numpy(a).to(device) for a in (qw, sc, z))


def _both(b200, x, qw, sc, z, bias, n, k):
    backends = importlib.import_module(b200.__name__ + ".backends")
    assert backends._fast is not None, "the _qi4_torch fast path was not built"
    kw = {"out_features": n, "in_features": k, "group_size": 64, "packing": "canonical"}
    fast = b200.b200_w4g64_linear(x, qw, sc, z, bias, **kw)
    saved = backends._fast
    backends._fast = None
    try:
        slow = b200.b200_w4g64_linear(x, qw, sc, z, bias, **kw)
    finally:
        backends._fast = saved
    torch.cuda.synchronize()
    return fast, slow


@pytest.mark.parametrize("x_dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("m", [1, 5, 40])
@pytest.mark.parametrize("bias_dtype", [None, torch.bfloat16, torch.float16])
def test_fast_path_matches_ctypes_path(b200, cuda_device, x_dtype, m, bias_dtype):
    n, k = 192, 512
    qw, sc, z = _weights(cuda_device, n, k, seed=m)
    x = torch.randn(m, k, generator=torch.Generator().manual_seed(7)).to(x_dtype).to(cuda_device)
    bias = None if bias_dtype is None else (torch.randn(n) * 0.02).to(bias_dtype).to(cuda_device)
    fast, slow = _both(b200, x, qw, sc, z, bias, n, k)
    assert fast.dtype == x_dtype and fast.shape == (m, n)
    assert torch.equal(fast, slow)


def test_fast_path_layouts(b200, cuda_device):
    """3-D, non-contiguous, misaligned and empty activations."""
    n, k = 128, 256
    qw, sc, z = _weights(cuda_device, n, k, seed=3)
    base = torch.randn(4, 3, 2 * k, generator=torch.Generator().manual_seed(1)).to(torch.bfloat16).to(cuda_device)
    for x in (base[..., :k],                      # non-contiguous rows
              base.reshape(-1)[1:1 + 6 * k].view(6, k),  # 2-byte offset: not 16-byte aligned
              base[:, :, k:].transpose(0, 1),     # 3-D, transposed leading dims
              base[:0, :, :k]):                   # no rows
        fast, slow = _both(b200, x, qw, sc, z, None, n, k)
        assert fast.shape == (*x.shape[:-1], n)
        assert torch.equal(fast, slow)
