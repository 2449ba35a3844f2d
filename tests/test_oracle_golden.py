"""Pin the CPU oracle to the reference: golden vectors and known-answer tests.

Every fixture was produced by the reference implementation itself
(``tests/golden/make_golden.py``); these tests run on the CPU only.
"""

import numpy as np
import pytest
import torch

from oracle import torch_port
from oracle import w4g64 as orc

import _golden as G


def test_canonical_byte_layout_kat():
    a = G.arrays()
    assert orc.pack_int4(a["kat_pack_codes"]).tolist() == a["kat_pack_bytes"].tolist() == [0x2F]
    assert orc.pack_int4(a["kat_zero_codes"]).tolist() == a["kat_zero_bytes"].tolist()
    assert a["kat_zero_bytes"].tolist() == [0xF8, 0x70]
    for i in range(2):
        codes, packed = a[f"kat_boundary{i}_codes"], a[f"kat_boundary{i}_bytes"]
        assert orc.pack_int4(codes).tolist() == packed.tolist()
        assert orc.unpack_int4(packed).tolist() == codes.tolist()


def test_unpack_random_bytes_odd_count():
    a = G.arrays()
    got = orc.unpack_int4(a["unpack_random_bytes"], elements=1025)
    assert got.dtype == np.int8
    np.testing.assert_array_equal(got, a["unpack_random_codes"])
    with pytest.raises(ValueError, match="element count"):
        orc.unpack_int4(a["unpack_random_bytes"], elements=1027)


def test_group_scale_indexing_kat():
    a = G.arrays()
    got = orc.dequantize_groupwise(
        a["kat_group2_qweight"], a["kat_group2_scales"], out_features=2, in_features=4,
        group_size=2, zeros=np.zeros(2, dtype=np.uint8))
    np.testing.assert_array_equal(got, a["kat_group2_expected"])
    np.testing.assert_array_equal(
        got, np.array([[0.5, 1.0, 6.0, 8.0], [-1.0, -2.0, -0.75, -1.0]], dtype=np.float32))


def test_asymmetric_group_zero_and_scale_kat():
    a = G.arrays()
    got = orc.dequantize_groupwise(
        a["kat_asym_qweight"], a["kat_asym_scales"], out_features=1, in_features=128,
        zeros=a["kat_asym_zeros"])
    np.testing.assert_array_equal(got, a["kat_asym_expected"])
    assert np.all(got[:, :64] == -0.25) and np.all(got[:, 64:] == 4.0)


@pytest.mark.parametrize("key", ["q_sym_small", "q_asym_small", "q_asym_odd", "q_sym_gate"])
def test_oracle_quantisers_match_reference_bytes(key):
    meta = G.manifest()[key]
    qw, sc, z = G.regen_quant(meta["n"], meta["k"], meta["kind"], meta["seed"], meta["std"])
    assert G.sha256(qw) == meta["qweight_sha256"]
    assert G.sha256(sc) == meta["scales_sha256"]
    assert G.sha256(z) == meta["zeros_sha256"]


@pytest.mark.parametrize("shape", [(3, 64), (5, 128), (256, 1536)])
def test_dequant_bit_exact_against_reference(shape):
    n, k = shape
    a, meta = G.arrays(), G.manifest()[f"deq_{n}x{k}"]
    key = f"deq_{n}x{k}"
    got = orc.dequantize_groupwise(a[f"{key}_qweight"], a[f"{key}_scales"],
                                   out_features=n, in_features=k, zeros=a[f"{key}_zeros"])
    assert got.dtype == np.float32
    assert G.sha256(got) == meta["expected_sha256"]
    port = torch_port.dequantize(torch.from_numpy(a[f"{key}_qweight"]),
                                 torch.from_numpy(a[f"{key}_scales"]),
                                 torch.from_numpy(a[f"{key}_zeros"]),
                                 out_features=n, in_features=k)
    assert G.sha256(port.numpy()) == meta["expected_sha256"]


def _ulp_budget(expected: torch.Tensor) -> np.ndarray:
    """One unit in the last place of the output dtype, per element."""
    e = expected.to(torch.float32).numpy()
    mant = {torch.float16: 10, torch.bfloat16: 7, torch.float32: 23}[expected.dtype]
    mag = np.maximum(np.abs(e), np.float32(2.0 ** -14))
    return np.exp2(np.floor(np.log2(mag)) - mant) * 1.0001 + 1e-6


@pytest.mark.parametrize("key", G.LINEAR_CASES)
def test_linear_oracle_matches_reference_outputs(key):
    c = G.linear_case(key)
    x = c["x"].to(torch.float32).numpy()
    bias = None if c["bias"] is None else c["bias"].to(torch.float32).numpy()
    raw = orc.linear(x, c["qweight"], c["scales"], c["zeros"], bias,
                     out_features=c["n"], in_features=c["k"])
    got = orc.round_to_dtype(raw, c["dtype"])
    exp = c["expected"].to(torch.float32).numpy()
    # Same algorithm, different BLAS summation order: at most one output ulp.
    assert np.all(np.abs(got - exp) <= _ulp_budget(c["expected"])), key


@pytest.mark.parametrize("key", ["lin_bzp", "lin_adv_zero", "lin_f32", "lin_d3",
                                 "lin_triton_8x1536x1536_bf16"])
def test_torch_port_matches_reference_outputs(key):
    c = G.linear_case(key)
    got = torch_port.linear(c["x"], torch.from_numpy(c["qweight"]),
                            torch.from_numpy(c["scales"]), torch.from_numpy(c["zeros"]),
                            c["bias"], out_features=c["n"], in_features=c["k"])
    assert got.dtype == c["expected"].dtype and got.shape == c["expected"].shape
    diff = np.abs(got.to(torch.float32).numpy() - c["expected"].to(torch.float32).numpy())
    assert np.all(diff <= _ulp_budget(c["expected"])), key


def test_boundary_zero_points_are_exact():
    c = G.linear_case("lin_bzp")
    raw = orc.linear(c["x"].float().numpy(), c["qweight"], c["scales"], c["zeros"], None,
                     out_features=2, in_features=128)
    np.testing.assert_array_equal(orc.round_to_dtype(raw, "f16"),
                                  c["expected"].float().numpy())


def test_bf16_rounding_helper_matches_torch():
    rng = np.random.default_rng(5)
    v = np.concatenate([rng.standard_normal(4096).astype(np.float32) * 100,
                        np.array([0.0, -0.0, 1e-40, 3.0e38, np.inf, -np.inf], np.float32)])
    ours = orc.f32_to_bf16_bits(v)
    theirs = torch.from_numpy(v).to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
    np.testing.assert_array_equal(ours, theirs)
    np.testing.assert_array_equal(orc.bf16_to_f32(ours),
                                  torch.from_numpy(v).to(torch.bfloat16).float().numpy())
