"""GPU parity of the CUDA kernels against the reference (golden vectors) and the oracle.

Tolerances (stated per the north-star contract):
* unpack and FP32 dequantisation: bit-exact;
* linear, GEMV kernel: |out - ref_f32| <= 1e-3 + 1 ulp of the output dtype
  (FP32 dequantised weights, FP32 accumulation - only the summation order
  differs from the reference);
* linear, tensor-core kernel (bf16/fp16 operands): |out - ref_f32| <= 2e-2 +
  1 ulp of the output dtype, ref_f32 = FP32 dequantise-then-matmul (f64 sum);
* and, for every case with a recorded reference output, the reference's own
  Triton-test tolerances (tests/test_triton_unpack.py:112: fp16 rtol 0.01 /
  atol 0.0625, bf16 rtol 0.02 / atol 0.25).
"""

import importlib

import numpy as np
import pytest
import torch

from oracle import w4g64 as orc

import _golden as G

pytestmark = pytest.mark.gpu

ALGOS = {"auto": 0, "gemv": 1, "gemv_fma": 3}


def _ulp(ref: np.ndarray, dtype: torch.dtype) -> np.ndarray:
    mant = {torch.float16: 10, torch.bfloat16: 7, torch.float32: 23}[dtype]
    mag = np.maximum(np.abs(ref), 2.0 ** -14)
    return np.exp2(np.floor(np.log2(mag)) - mant)


def assert_linear_close(got: torch.Tensor, ref_f32: np.ndarray, atol: float, what=""):
    g = got.detach().float().cpu().numpy().reshape(ref_f32.shape)
    err = np.abs(g - ref_f32)
    budget = atol + _ulp(ref_f32, got.dtype)
    worst = np.argmax(err - budget)
    assert np.all(err <= budget), (
        f"{what}: max err {err.max():.3e} at {np.unravel_index(worst, err.shape)} "
        f"(got {g.flat[worst]!r}, ref {ref_f32.flat[worst]!r}, budget {budget.flat[worst]:.3e})")


def to_dev(a, device):
    return torch.from_numpy(np.ascontiguousarray(a)).to(device)


# --------------------------------------------------------------------------
# unpack (bit-exact)
# --------------------------------------------------------------------------

@pytest.mark.parametrize("i", [0, 1])
def test_unpack_boundary_patterns(b200, cuda_device, i):
    a = G.arrays()
    packed = to_dev(a[f"kat_boundary{i}_bytes"], cuda_device)
    got = b200.unpack_canonical_signed_int4_b200(packed)
    np.testing.assert_array_equal(got.cpu().numpy(), a[f"kat_boundary{i}_codes"])


def test_unpack_random_bytes_odd_count(b200, cuda_device):
    a = G.arrays()
    packed = to_dev(a["unpack_random_bytes"], cuda_device)
    got = b200.unpack_canonical_signed_int4_b200(packed, elements=1025)
    assert got.dtype == torch.int8
    np.testing.assert_array_equal(got.cpu().numpy(), a["unpack_random_codes"])


@pytest.mark.parametrize("count", [0, 1, 31, 32, 33, 4095, 1 << 20, (1 << 20) + 17])
def test_unpack_sizes_and_ragged_tails(b200, cuda_device, count):
    rng = np.random.default_rng(count)
    nbytes = (count + 1) // 2 + (count % 3)
    raw = rng.integers(0, 256, size=max(nbytes, 1), dtype=np.uint8)
    got = b200.unpack_canonical_signed_int4_b200(to_dev(raw, cuda_device), elements=count)
    np.testing.assert_array_equal(got.cpu().numpy(), orc.unpack_int4(raw, elements=count))


def test_unpack_rejects_invalid_contracts(b200, cuda_device):
    packed = torch.zeros(4, dtype=torch.uint8, device=cuda_device)
    with pytest.raises(ValueError, match="dtype"):
        b200.unpack_canonical_signed_int4_b200(packed.to(torch.int8))
    with pytest.raises(ValueError, match="elements"):
        b200.unpack_canonical_signed_int4_b200(packed, elements=9)
    with pytest.raises(ValueError, match="contiguous"):
        b200.unpack_canonical_signed_int4_b200(packed.repeat(2)[::2])


# --------------------------------------------------------------------------
# FP32 dequantisation (bit-exact)
# --------------------------------------------------------------------------

@pytest.mark.parametrize("shape", [(3, 64), (5, 128), (256, 1536)])
def test_dequant_bit_exact_against_reference(b200, cuda_device, shape):
    n, k = shape
    key = f"deq_{n}x{k}"
    a, meta = G.arrays(), G.manifest()[key]
    got = b200.dequantize_canonical_w4g64_b200(
        to_dev(a[f"{key}_qweight"], cuda_device), to_dev(a[f"{key}_scales"], cuda_device),
        to_dev(a[f"{key}_zeros"], cuda_device), out_features=n, in_features=k)
    assert got.dtype == torch.float32 and got.shape == (n, k)
    assert G.sha256(got.cpu().numpy()) == meta["expected_sha256"]


@pytest.mark.parametrize("which", ["cfg0", "cfg2"])
def test_dequant_bit_exact_on_config_weights(b200, cuda_device, which):
    qw, sc, z = G.cfg0_weights() if which == "cfg0" else G.cfg2_weights()
    n, g = sc.shape
    k = g * 64
    got = b200.dequantize_canonical_w4g64_b200(to_dev(qw, cuda_device), to_dev(sc, cuda_device),
                                               to_dev(z, cuda_device), out_features=n, in_features=k)
    exp = orc.dequantize_groupwise(qw, sc, out_features=n, in_features=k, zeros=z)
    assert np.array_equal(got.cpu().numpy().view(np.uint32), exp.view(np.uint32))


def test_dequant_rejects_layout_and_dtype_drift(b200, cuda_device):
    qweight = torch.zeros(64, dtype=torch.uint8, device=cuda_device)
    scales = torch.ones(2, dtype=torch.float16, device=cuda_device)
    zeros = torch.zeros(1, dtype=torch.uint8, device=cuda_device)
    with pytest.raises(ValueError, match="divisible"):
        b200.dequantize_canonical_w4g64_b200(qweight, scales, zeros, out_features=1, in_features=96)
    with pytest.raises(ValueError, match="scales.*dtype"):
        b200.dequantize_canonical_w4g64_b200(qweight, scales.float(), zeros, out_features=1, in_features=128)
    with pytest.raises(ValueError, match="qweight must contain"):
        b200.dequantize_canonical_w4g64_b200(qweight[:-1], scales, zeros, out_features=1, in_features=128)


# --------------------------------------------------------------------------
# Linear forward against the reference's recorded outputs
# --------------------------------------------------------------------------

def _run_case(b200, c, device, algo):
    x = c["x"].to(device)
    bias = None if c["bias"] is None else c["bias"].to(device)
    return b200.b200_w4g64_linear(
        x, to_dev(c["qweight"], device), to_dev(c["scales"], device), to_dev(c["zeros"], device), bias,
        out_features=c["n"], in_features=c["k"], group_size=64, packing="canonical", algo=algo)


def _oracle_f32(c):
    x = c["x"].to(torch.float32).numpy()
    bias = None if c["bias"] is None else c["bias"].to(torch.float32).numpy()
    return orc.linear(x, c["qweight"], c["scales"], c["zeros"], bias,
                      out_features=c["n"], in_features=c["k"], accumulate="f64")


@pytest.mark.parametrize("algo", list(ALGOS))
@pytest.mark.parametrize("key", G.LINEAR_CASES)
def test_linear_matches_reference_outputs(b200, cuda_device, key, algo):
    c = G.linear_case(key)
    got = _run_case(b200, c, cuda_device, ALGOS[algo])
    exp = c["expected"]
    assert got.dtype == exp.dtype and tuple(got.shape) == tuple(exp.shape)
    rtol, atol = (0.02, 0.25) if exp.dtype == torch.bfloat16 else (0.01, 0.0625)
    if exp.dtype == torch.float32:
        rtol, atol = 1e-5, 1e-4
    torch.testing.assert_close(got.cpu(), exp, rtol=rtol, atol=atol)
    ref = _oracle_f32(c)
    # The GEMV keeps FP32 weights and FP32 sums; AUTO may pick the tensor-core
    # kernel for large M (none of these cases has M > 16).
    assert_linear_close(got, ref, 1e-3, key)


def test_boundary_zero_points_exact(b200, cuda_device):
    c = G.linear_case("lin_bzp")
    got = _run_case(b200, c, cuda_device, ALGOS["gemv"])
    assert torch.equal(got.cpu(), c["expected"])


# --------------------------------------------------------------------------
# Shape sweeps against the oracle (seeded; BASELINE config 1 and 2 shapes)
# --------------------------------------------------------------------------

QWEN_SHAPES = {"q": (1536, 1536), "k": (1536, 256), "v": (1536, 256), "o": (1536, 1536),
               "gate": (1536, 8960), "up": (1536, 8960), "down": (8960, 1536)}
_WCACHE = {}


def _weights(k, n, kind, seed):
    key = (k, n, kind, seed)
    if key not in _WCACHE:
        torch.manual_seed(seed)
        w = (torch.randn(n, k) * 0.02).to(torch.bfloat16).float().numpy()
        if kind == "sym":
            qw, sc = orc.quantize_symmetric_rtn(w)
            z = np.zeros(((n * (k // 64) + 1) // 2, 1), dtype=np.uint8)
        else:
            qw, sc, z = orc.quantize_asymmetric_rtn(w)
        _WCACHE[key] = (qw, sc, z)
    return _WCACHE[key]


@pytest.mark.parametrize("algo", ["gemv", "gemv_fma"])
@pytest.mark.parametrize("m", [1, 2, 3, 4, 5, 8, 13, 16])
@pytest.mark.parametrize("name", list(QWEN_SHAPES))
def test_gemv_shape_sweep(b200, cuda_device, name, m, algo):
    k, n = QWEN_SHAPES[name]
    qw, sc, z = _weights(k, n, "sym", 11)
    g = torch.Generator().manual_seed(1000 + m)
    x = torch.randn(m, k, generator=g).to(torch.bfloat16)
    bias = (torch.randn(n, generator=g) * 0.02).to(torch.bfloat16) if name in "qkv" else None
    got = b200.b200_w4g64_linear(
        x.to(cuda_device), to_dev(qw, cuda_device), to_dev(sc, cuda_device), to_dev(z, cuda_device),
        None if bias is None else bias.to(cuda_device), out_features=n, in_features=k, group_size=64,
        packing="canonical", algo=ALGOS[algo])
    ref = orc.linear(x.float().numpy(), qw, sc, z, None if bias is None else bias.float().numpy(),
                     out_features=n, in_features=k, accumulate="f64")
    assert_linear_close(got, ref, 1e-3, f"{name} m={m} {algo}")


@pytest.mark.parametrize("algo", ["gemv", "gemv_fma"])
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16, torch.float32])
@pytest.mark.parametrize("m", [1, 13, 16])
def test_gemv_awq_down_proj_all_dtypes(b200, cuda_device, dtype, m, algo):
    qw, sc, z = G.cfg2_weights()
    chan = torch.from_numpy(G.arrays()["cfg2_chan"])
    g = torch.Generator().manual_seed(300 + m)
    x = (torch.randn(m, 8960, generator=g) / chan).to(dtype)
    got = b200.b200_w4g64_linear(
        x.to(cuda_device), to_dev(qw, cuda_device), to_dev(sc, cuda_device), to_dev(z, cuda_device), None,
        out_features=1536, in_features=8960, group_size=64, packing="canonical", algo=ALGOS[algo])
    assert got.dtype == dtype
    ref = orc.linear(x.float().numpy(), qw, sc, z, None, out_features=1536, in_features=8960,
                     accumulate="f64")
    assert_linear_close(got, ref, 1e-3, f"awq down {dtype} m={m} {algo}")


@pytest.mark.parametrize("bias_dtype", [torch.float16, torch.bfloat16, torch.float32])
def test_bias_dtypes(b200, cuda_device, bias_dtype):
    qw, sc, z = _weights(1536, 256, "asym", 5)
    x = torch.randn(3, 1536, generator=torch.Generator().manual_seed(4)).to(torch.bfloat16)
    bias = (torch.randn(256, generator=torch.Generator().manual_seed(6)) * 0.1).to(bias_dtype)
    got = b200.b200_w4g64_linear(
        x.to(cuda_device), to_dev(qw, cuda_device), to_dev(sc, cuda_device), to_dev(z, cuda_device),
        bias.to(cuda_device), out_features=256, in_features=1536, group_size=64, packing="canonical")
    ref = orc.linear(x.float().numpy(), qw, sc, z, bias.float().numpy(), out_features=256,
                     in_features=1536, accumulate="f64")
    assert_linear_close(got, ref, 1e-3, str(bias_dtype))


def test_non_contiguous_three_d_and_empty_inputs(b200, cuda_device):
    qw, sc, z = _weights(128, 64, "asym", 9)
    args = dict(out_features=64, in_features=128, group_size=64, packing="canonical")
    dev = [to_dev(t, cuda_device) for t in (qw, sc, z)]
    x = torch.arange(4 * 128, dtype=torch.float32).reshape(128, 4).t().to(torch.bfloat16) / 100
    assert not x.is_contiguous()
    got = b200.b200_w4g64_linear(x.to(cuda_device), *dev, None, **args)
    ref = orc.linear(x.float().numpy(), qw, sc, z, None, out_features=64, in_features=128, accumulate="f64")
    assert_linear_close(got, ref, 1e-3, "non-contiguous")
    x3 = torch.randn(2, 3, 128, generator=torch.Generator().manual_seed(2)).to(torch.float16)
    got3 = b200.b200_w4g64_linear(x3.to(cuda_device), *dev, None, **args)
    assert got3.shape == (2, 3, 64)
    ref3 = orc.linear(x3.float().numpy(), qw, sc, z, None, out_features=64, in_features=128, accumulate="f64")
    assert_linear_close(got3, ref3, 1e-3, "3-d")
    empty = b200.b200_w4g64_linear(torch.zeros(0, 128, dtype=torch.bfloat16, device=cuda_device), *dev,
                                   None, **args)
    assert empty.shape == (0, 64)
    empty3 = b200.b200_w4g64_linear(torch.zeros(2, 0, 128, dtype=torch.bfloat16, device=cuda_device),
                                    *dev, None, **args)
    assert empty3.shape == (2, 0, 64)


def test_pdl_on_and_off_give_identical_bits(b200, cuda_device):
    qw, sc, z = _weights(1536, 8960, "sym", 3)
    dev = [to_dev(t, cuda_device) for t in (qw, sc, z)]
    x = torch.randn(4, 1536, device=cuda_device).to(torch.bfloat16)
    args = dict(out_features=8960, in_features=1536, group_size=64, packing="canonical", algo=ALGOS["gemv"])
    a = b200.b200_w4g64_linear(x, *dev, None, pdl=True, **args)
    b = b200.b200_w4g64_linear(x, *dev, None, pdl=False, **args)
    assert torch.equal(a, b)


def test_reference_quantlinear_dispatches_to_b200(b200, cuda_device):
    """The reference's own QuantLinear (src/qwen_int4/linear.py:17-72) on the
    b200 backend after ``register_with_reference``: its forward reaches the
    CUDA kernels and matches the recorded reference output and the oracle."""
    q2 = importlib.import_module(b200.__name__ + ".qwen2")
    ref = q2.reference_package()
    q2.register_with_reference(ref.__name__)
    linear = importlib.import_module(ref.__name__ + ".linear")
    c = G.linear_case("lin_d3")
    layer = linear.QuantLinear(128, 64, group_size=64, bias=True, packing="canonical").to(cuda_device)
    layer.qweight.copy_(torch.from_numpy(c["qweight"]).view_as(layer.qweight))
    layer.scales.copy_(torch.from_numpy(c["scales"]))
    layer.zeros.copy_(torch.from_numpy(c["zeros"]).view_as(layer.zeros))
    layer.bias.copy_(c["bias"])
    layer.set_backend("b200")
    got = layer(c["x"].to(cuda_device))
    torch.testing.assert_close(got.cpu(), c["expected"], rtol=0.02, atol=0.25)
    assert_linear_close(got, _oracle_f32(c), 1e-3, "QuantLinear")


def test_wrong_device_mix_is_rejected(b200, cuda_device):
    qw, sc, z = _weights(128, 64, "asym", 9)
    with pytest.raises(ValueError, match="CUDA tensors|same device"):
        b200.b200_w4g64_linear(torch.zeros(1, 128, dtype=torch.bfloat16, device=cuda_device),
                               torch.from_numpy(qw), to_dev(sc, cuda_device), to_dev(z, cuda_device), None,
                               out_features=64, in_features=128, group_size=64, packing="canonical")


@pytest.mark.parametrize(("rows", "warps"), [(16, 2), (16, 4), (16, 16), (32, 2), (32, 4), (64, 4), (64, 8), (64, 16), (128, 8)])
@pytest.mark.parametrize("ksplit", [1, 2, 3, 5])
def test_gemv_launch_shapes_agree(b200, cuda_device, rows, warps, ksplit):
    """Every forced launch shape (rows per CTA, warps, cluster K split) gives the oracle's answer."""
    from importlib import import_module

    lib = import_module(b200.__name__ + "._lib").load()
    k, n = 1536, 1000  # N not a multiple of any tile: exercises the ragged last CTA
    qw, sc, z = _weights(k, n, "asym", 21)
    x = torch.randn(5, k, generator=torch.Generator().manual_seed(22)).to(torch.bfloat16)
    ref = orc.linear(x.float().numpy(), qw, sc, z, None, out_features=n, in_features=k, accumulate="f64")
    assert lib.qi4_gemv_mma_plan_override(rows, ksplit, warps) == 0
    try:
        got = b200.b200_w4g64_linear(
            x.to(cuda_device), to_dev(qw, cuda_device), to_dev(sc, cuda_device), to_dev(z, cuda_device), None,
            out_features=n, in_features=k, group_size=64, packing="canonical", algo=ALGOS["gemv"])
    finally:
        lib.qi4_gemv_mma_plan_override(0, 0, 0)
    assert_linear_close(got, ref, 1e-3, f"rows={rows} warps={warps} ksplit={ksplit}")


def test_device_status_clean_after_kernels(b200, cuda_device):
    from importlib import import_module

    lib = import_module(b200.__name__ + "._lib").load()
    qw, sc, z = _weights(1536, 256, "sym", 2)
    x = torch.randn(1, 1536, device=cuda_device).to(torch.bfloat16)
    b200.b200_w4g64_linear(x, to_dev(qw, cuda_device), to_dev(sc, cuda_device), to_dev(z, cuda_device), None,
                           out_features=256, in_features=1536, group_size=64, packing="canonical")
    assert lib.qi4_device_status(torch.cuda.current_stream().cuda_stream) == 0


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("n", [100, 200, 1536])
@pytest.mark.parametrize("m", [1, 3, 9])
def test_gemv_output_stores_aligned_and_not(b200, cuda_device, dtype, n, m):
    """The decode GEMV writes 16-bit outputs of whole, 16-byte-aligned tiles
    as 16-byte stores and falls back to element stores for a partial last
    tile, a row pitch that is not a multiple of 8 outputs, or an output
    pointer off the 16-byte grid (C ABI call into an offset buffer)."""
    import ctypes

    k = 256
    qw, sc, z = _weights(k, n, "asym", 5)
    g = torch.Generator().manual_seed(77 + m)
    x = torch.randn(m, k, generator=g).to(dtype)
    ref = orc.linear(x.float().numpy(), qw, sc, z, None, out_features=n, in_features=k, accumulate="f64")
    lib = importlib.import_module(b200.__name__ + "._lib").load()
    xd, qwd, scd, zd = x.to(cuda_device), to_dev(qw, cuda_device), to_dev(sc, cuda_device), to_dev(z, cuda_device)
    code = {torch.bfloat16: 1, torch.float16: 0}[dtype]
    stream = torch.cuda.current_stream(cuda_device).cuda_stream
    for offset in (0, 1):  # elements: 0 = aligned buffer, 1 = 2-byte offset
        buf = torch.full((m * n + 8,), float("nan"), dtype=dtype, device=cuda_device)
        out = buf[offset:offset + m * n]
        rc = lib.qi4_w4g64_linear_ex(xd.data_ptr(), code, m, k, qwd.data_ptr(), scd.data_ptr(), zd.data_ptr(),
                                     None, -1, out.data_ptr(), n, ctypes.c_void_p(stream), 1, 1)
        torch.cuda.synchronize()
        assert rc == 0
        assert_linear_close(out.view(m, n), ref, 1e-3, f"n={n} m={m} offset={offset}")
        assert torch.isnan(buf[:offset]).all() and torch.isnan(buf[offset + m * n:]).all()


def test_bounded_wait_runs_out_as_a_status_not_a_hang(b200, cuda_device):
    """Failure detection without a GPU fault: a wait on a barrier that nothing
    arrives on ends after its limit (10 ms here) and shows up as
    QI4_DEVICE_WAIT_TIMEOUT in qi4_device_status; the flag is cleared by the
    read, and the context still runs a linear correctly afterwards."""
    import time

    lib = importlib.import_module(b200.__name__ + "._lib").load()
    stream = torch.cuda.current_stream(cuda_device).cuda_stream
    assert lib.qi4_device_status(stream) >= 0  # clear leftovers
    t0 = time.perf_counter()
    assert lib.qi4_selftest_bounded_wait(10_000_000, stream) == 0
    torch.cuda.synchronize()
    waited = time.perf_counter() - t0
    assert 0.009 <= waited < 5.0, waited
    assert lib.qi4_device_status(stream) == 1  # QI4_DEVICE_WAIT_TIMEOUT
    assert lib.qi4_device_status(stream) == 0  # cleared by the read
    k, n = 128, 64
    qw, sc, z = _weights(k, n, "asym", 9)
    x = torch.randn(2, k, generator=torch.Generator().manual_seed(3)).to(torch.bfloat16)
    got = b200.b200_w4g64_linear(x.to(cuda_device), to_dev(qw, cuda_device), to_dev(sc, cuda_device),
                                 to_dev(z, cuda_device), None, out_features=n, in_features=k, group_size=64,
                                 packing="canonical")
    ref = orc.linear(x.float().numpy(), qw, sc, z, None, out_features=n, in_features=k, accumulate="f64")
    assert_linear_close(got, ref, 1e-3, "after the self-test")
    assert lib.qi4_device_status(stream) == 0
