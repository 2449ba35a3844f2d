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
