"""Tied bf16 lm_head GEMV with fused argmax (qi4_bf16_gemv_argmax) on a GPU.

Logits against torch's bf16 linear (the reference's nn.Linear lm_head,
model.py:217-218) within one bf16 ulp of the FP32 sum; the argmax equal to
``torch.argmax`` of our own bf16 logits (first index on ties), and equal to
the reference logits' argmax wherever the top two reference logits differ
by more than the logits' rounding.
"""

import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("m", [1, 2, 5, 8])
@pytest.mark.parametrize("n", [151936, 1000, 7])
def test_lm_head_logits_and_argmax(b200, cuda_device, m, n):
    g = torch.Generator().manual_seed(m * 1000 + n)
    d = 1536
    w = (torch.randn(n, d, generator=g) * 0.02).to(torch.bfloat16).to(cuda_device)
    x = torch.randn(m, d, generator=g).to(torch.bfloat16).to(cuda_device)
    logits, arg = b200.b200_lm_head(x, w)
    torch.cuda.synchronize()
    exact = x.double() @ w.double().t()
    ulp = torch.exp2(torch.floor(torch.log2(exact.abs().clamp_min(2.0 ** -100))) - 7)
    assert bool(((logits.double() - exact).abs() <= ulp + 1e-6).all())
    assert torch.equal(arg, logits.argmax(dim=-1))
    ref = torch.nn.functional.linear(x, w)
    top2 = ref.float().topk(2, dim=-1).values
    clear = (top2[:, 0] - top2[:, 1]) > 2 * ulp.max()
    assert torch.equal(arg[clear], ref.argmax(dim=-1)[clear])


def test_lm_head_argmax_only_skips_logits_and_breaks_ties_to_first(b200, cuda_device):
    d, n = 256, 4096
    w = torch.zeros(n, d, dtype=torch.bfloat16, device=cuda_device)
    w[[17, 900, 3000], 0] = 1.0  # three equal maxima: the first row wins
    x = torch.zeros(2, d, dtype=torch.bfloat16, device=cuda_device)
    x[:, 0] = 2.0
    logits, arg = b200.b200_lm_head(x, w, return_logits=False)
    assert logits is None
    assert arg.tolist() == [17, 17]


def test_argmax_with_caller_workspace_leaves_it_zero(b200, cuda_device):
    """qi4_bf16_gemv_argmax_ws gives the plain call's tokens, and its 8-word
    workspace is zero again after every call (so repeated calls need no
    memset)."""
    import ctypes
    from importlib import import_module

    lib = import_module(b200.__name__ + "._lib").load()
    g = torch.Generator().manual_seed(3)
    w = (torch.randn(151936, 1536, generator=g) * 0.02).to(torch.bfloat16).to(cuda_device)
    keys = torch.zeros(8, dtype=torch.int64, device=cuda_device)
    s = torch.cuda.current_stream().cuda_stream
    for m in (1, 3, 8):
        x = torch.randn(m, 1536, generator=g).to(torch.bfloat16).to(cuda_device)
        a, b = (torch.empty(m, dtype=torch.int64, device=cuda_device) for _ in range(2))
        assert lib.qi4_bf16_gemv_argmax(w.data_ptr(), x.data_ptr(), m, 1536, 151936, None, a.data_ptr(), s) == 0
        assert lib.qi4_bf16_gemv_argmax_ws(w.data_ptr(), x.data_ptr(), m, 1536, 151936, None, b.data_ptr(),
                                           keys.data_ptr(), s) == 0
        torch.cuda.synchronize()
        assert torch.equal(a, b) and int(keys.abs().sum()) == 0
    assert lib.qi4_bf16_gemv_argmax_ws(w.data_ptr(), x.data_ptr(), 1, 1536, 151936, None, b.data_ptr(), None, s) == -1


@pytest.mark.parametrize(("b", "v", "pad", "offset"), [(64, 151936, 0, 0), (3, 1001, 7, 1), (1, 7, 0, 0), (9, 64, 8, 0)])
def test_argmax_rows_matches_torch_argmax(b200, cuda_device, b, v, pad, offset):
    """qi4_bf16_argmax_rows against torch.argmax(dim=-1) on bf16 rows: planted
    ties (the first index wins), NaN (counts as the maximum), +/-inf, rows
    with a pitch above V and a base that is not 16-byte aligned (the scalar
    path)."""
    from importlib import import_module

    lib = import_module(b200.__name__ + "._lib").load()
    g = torch.Generator().manual_seed(b * 7 + v)
    ld = v + pad
    buf = (torch.randn(b * ld + offset, generator=g) * 4).to(torch.bfloat16).to(cuda_device)
    rows = buf[offset:].view(b, ld)
    top = rows[:, :v].float().max(dim=-1).values
    for r in range(b):
        if r % 4 == 1 and v > 3:  # a tie with the existing maximum, later and earlier
            i = int(rows[r, :v].float().argmax())
            rows[r, (i + 1) % v] = top[r].to(torch.bfloat16)
            rows[r, max(i - 1, 0)] = top[r].to(torch.bfloat16)
        if r % 4 == 2:
            rows[r, v // 2] = float("nan")
            rows[r, v - 1] = float("nan")
        if r % 4 == 3:
            rows[r, 0] = float("-inf")
            rows[r, v - 1] = float("inf")
    if pad:
        rows[:, v:] = 1e4  # past V: never read
    out = torch.full((b,), -5, dtype=torch.int64, device=cuda_device)
    s = torch.cuda.current_stream().cuda_stream
    assert lib.qi4_bf16_argmax_rows(rows.data_ptr(), b, v, ld, out.data_ptr(), s) == 0
    torch.cuda.synchronize()
    assert torch.equal(out, torch.argmax(rows[:, :v], dim=-1))
    assert lib.qi4_bf16_argmax_rows(rows.data_ptr(), b, v, v - 1, out.data_ptr(), s) != 0  # ld < V
