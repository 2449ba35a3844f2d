"""Decode attention with in-place KV append (qi4_gqa_decode_attention) on a GPU.

Against the reference attention's own math on the same inputs (RoPE as three
bf16 tensor ops, model.py:74-77; repeat_interleave of the KV heads and a
masked softmax in FP32, model.py:90-118): outputs within 1.5e-2 absolute /
cosine >= 0.99999 (the bf16 output's own rounding is ~4e-3 relative), the
appended cache entries bit-exact. Then the reference model itself on the
b200 backend with ``fast_attention=True``: cached decode agrees with the full
forward and with the unpatched decode, and a forked cache keeps both
continuations apart.
"""

import ctypes
import importlib

import pytest
import torch

pytestmark = pytest.mark.gpu


def _rotate_half(x):
    a, b = x.chunk(2, dim=-1)
    return torch.cat((-b, a), dim=-1)


def _reference(q, k_new, v_new, cos, sin, past_k, past_v, mask, G):
    """The reference model's decode attention (model.py:74-118), FP32 softmax."""
    q = q.unsqueeze(2)  # [B, Hq, 1, D]
    k = k_new.unsqueeze(2)
    c, s = cos[:, None, None, :], sin[:, None, None, :]
    q = q * c + _rotate_half(q) * s
    k = k * c + _rotate_half(k) * s
    K = torch.cat((past_k, k), dim=2).repeat_interleave(G, dim=1).float()
    V = torch.cat((past_v, v_new.unsqueeze(2)), dim=2).repeat_interleave(G, dim=1).float()
    scores = (q.float() @ K.transpose(-1, -2)) * q.shape[-1] ** -0.5
    if mask is not None:
        scores = scores.masked_fill(~mask.bool()[:, None, None, :], float("-inf"))
    out = torch.softmax(scores, dim=-1) @ V
    return out.squeeze(2).reshape(q.shape[0], -1).to(torch.bfloat16), k.squeeze(2)


@pytest.mark.parametrize("B,L,Hq,Hkv", [(1, 0, 12, 2), (1, 5, 12, 2), (3, 63, 12, 2), (2, 64, 12, 2),
                                        (2, 130, 8, 8), (4, 700, 12, 2), (64, 333, 12, 2)])
def test_decode_attention_matches_reference_math(b200, cuda_device, B, L, Hq, Hkv):
    g = torch.Generator(device="cpu").manual_seed(L * 7 + B)
    D, cap = 128, L + 1 + 37
    bf = dict(dtype=torch.bfloat16, device=cuda_device)
    q = torch.randn(B, Hq, D, generator=g).to(**bf)
    k_new = torch.randn(B, Hkv, D, generator=g).to(**bf)
    v_new = torch.randn(B, Hkv, D, generator=g).to(**bf)
    pos = torch.arange(B) + L
    inv = 1.0 / (1e6 ** (torch.arange(0, D, 2, dtype=torch.float32) / D))
    f = pos[:, None].float() * inv[None, :]
    emb = torch.cat((f, f), dim=-1)
    cos, sin = emb.cos().to(**bf), emb.sin().to(**bf)
    kc = torch.randn(B, Hkv, cap, D, generator=g).to(**bf)
    vc = torch.randn(B, Hkv, cap, D, generator=g).to(**bf)
    past_k, past_v = kc[:, :, :L].clone(), vc[:, :, :L].clone()
    mask = torch.ones(B, L + 1, dtype=torch.bool)
    for b in range(B):  # left padding: the first (b * 3) % (L + 1) keys invalid
        mask[b, : (b * 3) % (L + 1)] = False
    mask = mask.to(cuda_device)
    lengths = torch.full((B,), L, dtype=torch.int32, device=cuda_device)
    out = b200.b200_gqa_decode_attention(q, k_new, v_new, kc, vc, lengths, cos=cos, sin=sin, key_mask=mask)
    torch.cuda.synchronize()
    ref, k_roped = _reference(q, k_new, v_new, cos, sin, past_k, past_v, mask, Hq // Hkv)
    cosine = torch.nn.functional.cosine_similarity(out.float().flatten(), ref.float().flatten(), dim=0)
    assert float((out.float() - ref.float()).abs().max()) <= 1.5e-2
    assert float(cosine) >= 0.99999
    assert torch.equal(kc[:, :, L], k_roped) and torch.equal(vc[:, :, L], v_new)  # appended in place
    assert torch.equal(kc[:, :, :L], past_k) and torch.equal(vc[:, :, :L], past_v)  # past untouched


def test_full_cache_gives_zero_output_and_a_status(b200, cuda_device):
    lib = importlib.import_module(b200.__name__ + "._lib").load()
    bf = dict(dtype=torch.bfloat16, device=cuda_device)
    q, kv = torch.randn(1, 12, 128).to(**bf), torch.randn(1, 2, 128).to(**bf)
    kc, vc = torch.zeros(1, 2, 8, 128, **bf), torch.zeros(1, 2, 8, 128, **bf)
    lengths = torch.tensor([8], dtype=torch.int32, device=cuda_device)  # no room for key 8
    out = b200.b200_gqa_decode_attention(q, kv, kv, kc, vc, lengths)
    assert torch.count_nonzero(out) == 0
    assert lib.qi4_device_status(torch.cuda.current_stream().cuda_stream) == 2
    assert lib.qi4_device_status(torch.cuda.current_stream().cuda_stream) == 0


def _cos(a, b):
    return float(torch.nn.functional.cosine_similarity(a.float().flatten(), b.float().flatten(), dim=0))


def test_reference_model_decode_with_fast_attention(b200, cuda_device):
    """The reference model (2 layers) on b200 with the decode attention
    patched in: each cached step agrees with the full forward, and with the
    same steps through the reference's own attention code."""
    q2 = importlib.import_module(b200.__name__ + ".qwen2")
    cfg = q2.qwen2_config(num_hidden_layers=2, vocab_size=512)
    model = q2.build_random_qwen2(cfg, device=cuda_device, seed=3, fast_attention=True)
    ref_name = q2.reference_package().__name__
    tokens = torch.randint(0, 512, (2, 12), generator=torch.Generator().manual_seed(1)).to(cuda_device)
    mask = torch.ones(2, 12, dtype=torch.bool, device=cuda_device)
    mask[1, :3] = False  # left padding of the second sequence
    try:
        with torch.inference_mode():
            full = model(tokens, attention_mask=mask)
            fast_steps = []
            _, cache = model(tokens[:, :6], attention_mask=mask[:, :6], use_cache=True)
            for t in range(6, 12):
                logits, cache = model(tokens[:, t:t + 1], attention_mask=mask[:, :t + 1], past_key_values=cache,
                                      use_cache=True)
                fast_steps.append(logits[:, -1])
            assert cache[0][0].shape[2] == 12
            q2.register_with_reference(ref_name, fast_attention=False)
            _, cache = model(tokens[:, :6], attention_mask=mask[:, :6], use_cache=True)
            for i, t in enumerate(range(6, 12)):
                logits, cache = model(tokens[:, t:t + 1], attention_mask=mask[:, :t + 1], past_key_values=cache,
                                      use_cache=True)
                assert _cos(fast_steps[i], logits[:, -1]) > 0.9999
                assert _cos(fast_steps[i], full[:, t]) > 0.9999
    finally:
        q2.register_with_reference(ref_name, fast_attention=False)


def test_forked_cache_continuations_stay_apart(b200, cuda_device):
    q2 = importlib.import_module(b200.__name__ + ".qwen2")
    cfg = q2.qwen2_config(num_hidden_layers=2, vocab_size=512)
    model = q2.build_random_qwen2(cfg, device=cuda_device, seed=4, fast_attention=True)
    ref_name = q2.reference_package().__name__
    prompt = torch.randint(0, 512, (1, 7), generator=torch.Generator().manual_seed(2)).to(cuda_device)
    a, b = torch.tensor([[5]], device=cuda_device), torch.tensor([[9]], device=cuda_device)
    try:
        with torch.inference_mode():
            _, cache = model(prompt, use_cache=True)
            _, cache = model(a, past_key_values=cache, use_cache=True)  # capacity buffers from here on
            la, ca = model(a, past_key_values=cache, use_cache=True)
            lb, cb = model(b, past_key_values=cache, use_cache=True)  # same prefix: must copy, not overwrite
            la2, _ = model(b, past_key_values=ca, use_cache=True)
            full_a = model(torch.cat((prompt, a, a, b), dim=1))
            full_b = model(torch.cat((prompt, a, b), dim=1))
        assert _cos(la2[:, -1], full_a[:, -1]) > 0.9999
        assert _cos(lb[:, -1], full_b[:, -1]) > 0.9999
        assert not torch.equal(ca[0][0], cb[0][0])
    finally:
        q2.register_with_reference(ref_name, fast_attention=False)


def test_workspace_and_early_cache_read_give_the_same_result(b200, cuda_device):
    """qi4_gqa_decode_attention_ex with a caller workspace (and the early cache
    read a decode step may use) equals the plain call bit for bit; a workspace
    that is too small is rejected before any launch."""
    lm = importlib.import_module(b200.__name__ + "._lib")
    lib = lm.load()
    g = torch.Generator(device="cpu").manual_seed(12)
    B, L, Hq, Hkv, D, cap = 3, 200, 12, 2, 128, 256
    bf = dict(dtype=torch.bfloat16, device=cuda_device)
    q = torch.randn(B, Hq, D, generator=g).to(**bf)
    kn, vn = torch.randn(B, Hkv, D, generator=g).to(**bf), torch.randn(B, Hkv, D, generator=g).to(**bf)
    kc0, vc0 = torch.randn(B, Hkv, cap, D, generator=g).to(**bf), torch.randn(B, Hkv, cap, D, generator=g).to(**bf)
    lengths = torch.tensor([L, L - 77, 5], dtype=torch.int32, device=cuda_device)
    s = torch.cuda.current_stream().cuda_stream
    outs = []
    for mode in ("plain", "ws", "ws_early"):
        kc, vc = kc0.clone(), vc0.clone()
        out = torch.empty(B, Hq * D, **bf)
        args = (q.data_ptr(), kn.data_ptr(), vn.data_ptr(), None, None, None, kc.data_ptr(), vc.data_ptr(),
                kc.stride(0), kc.stride(1), cap, lengths.data_ptr(), None, 0, out.data_ptr(), B, Hq, Hkv, D,
                ctypes.c_float(D ** -0.5))
        if mode == "plain":
            assert lib.qi4_gqa_decode_attention(*args, s) == 0
        else:
            n = lib.qi4_gqa_decode_attention_workspace(B, Hq, Hkv, cap)
            ws = torch.empty(n, dtype=torch.uint8, device=cuda_device)
            flags = lm.ATTN_EARLY_CACHE_READ if mode == "ws_early" else 0
            assert lib.qi4_gqa_decode_attention_ex(*args, flags, ws.data_ptr(), n - 16, s) == -1  # too small
            assert lib.qi4_gqa_decode_attention_ex(*args, flags, ws.data_ptr(), n, s) == 0
        torch.cuda.synchronize()
        outs.append((out, kc, vc))
    for out, kc, vc in outs[1:]:
        assert torch.equal(out, outs[0][0]) and torch.equal(kc, outs[0][1]) and torch.equal(vc, outs[0][2])


@pytest.mark.parametrize(("cap", "lengths", "big"), [(1000, [998, 300, 0, 1000], 10), (100, [99, 64, 63, 7], 80)])
def test_cluster_merge_equals_the_combine_kernel(b200, cuda_device, cap, lengths, big):
    """Small grids merge the splits of a (sequence, KV head) inside one
    thread-block cluster (no combine launch); large grids use the combine
    kernel. The same sequences, alone (cluster path: 16 or 2 splits, so one
    or three heads per merging CTA) and as the first rows of a batch large
    enough for the two-kernel path, give bit-identical outputs and caches; a
    full cache gives zeros and QI4_DEVICE_CACHE_FULL on both paths; splits
    without keys (short sequences) still take part in the cluster."""
    lm = importlib.import_module(b200.__name__ + "._lib")
    lib = lm.load()
    g = torch.Generator(device="cpu").manual_seed(cap)
    Hq, Hkv, D = 12, 2, 128
    bf = dict(dtype=torch.bfloat16, device=cuda_device)
    q = torch.randn(big, Hq, D, generator=g).to(**bf)
    kn, vn = torch.randn(big, Hkv, D, generator=g).to(**bf), torch.randn(big, Hkv, D, generator=g).to(**bf)
    kc0, vc0 = torch.randn(big, Hkv, cap, D, generator=g).to(**bf), torch.randn(big, Hkv, cap, D, generator=g).to(**bf)
    small = len(lengths)
    lens = torch.tensor(lengths + [cap // 2] * (big - small), dtype=torch.int32, device=cuda_device)
    s = torch.cuda.current_stream().cuda_stream
    full = any(x >= cap for x in lengths)
    res = []
    for B in (small, big):
        kc, vc = kc0[:B].clone(), vc0[:B].clone()
        out = torch.full((B, Hq * D), float("nan"), **bf)
        n = lib.qi4_gqa_decode_attention_workspace(B, Hq, Hkv, cap)
        ws = torch.empty(n, dtype=torch.uint8, device=cuda_device)
        rc = lib.qi4_gqa_decode_attention_ex(
            q.data_ptr(), kn.data_ptr(), vn.data_ptr(), None, None, None, kc.data_ptr(), vc.data_ptr(), kc.stride(0),
            kc.stride(1), cap, lens.data_ptr(), None, 0, out.data_ptr(), B, Hq, Hkv, D, ctypes.c_float(D ** -0.5), 0,
            ws.data_ptr(), n, s)
        assert rc == 0
        torch.cuda.synchronize()
        assert lib.qi4_device_status(s) == (2 if full else 0)
        res.append((out[:small], kc[:small], vc[:small]))
    (o1, k1, v1), (o2, k2, v2) = res
    assert not bool(o1.isnan().any())
    assert torch.equal(o1, o2) and torch.equal(k1, k2) and torch.equal(v1, v2)
    for i, L in enumerate(lengths):
        if L >= cap:
            assert bool((o1[i] == 0).all())
