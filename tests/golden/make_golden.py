"""Generate golden W4G64 vectors by running the reference implementation.

Run once, in a checkout that has the reference project
(ryanyue-16/qwen2-int4-systems) available:

    python tests/golden/make_golden.py --reference-src <reference>/src

It imports the reference's own ``qwen_int4`` package and records, for seeded
inputs, what the reference's quantisers, ``unpack_int4``,
``dequantize_groupwise`` and ``torch_reference_linear`` return. Outputs:

* ``w4g64_golden.npz`` - arrays (inputs where small, outputs, digests);
* ``manifest.json``    - one entry per case: shape, dtype, seed, the
  reference test it mirrors (file:line in the reference project).

Large weight tensors are not stored. They are regenerated from a seed with
``torch.randn`` on the CPU and the oracle quantiser, and the fixture keeps the
SHA-256 of the reference quantiser's bytes so the regeneration is checked.
The GPU host never runs this script; it only reads the committed fixtures.
"""

from __future__ import annotations

import argparse
import hashlib
import json
import math
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent


def sha256(array: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(array).tobytes()).hexdigest()


def as_bits(t: torch.Tensor) -> np.ndarray:
    """Store fp16/bf16 tensors as uint16 bit patterns, fp32 as float32."""
    t = t.detach().cpu().contiguous()
    if t.dtype in (torch.float16, torch.bfloat16):
        return t.view(torch.int16).numpy().view(np.uint16)
    if t.dtype == torch.float32:
        return t.numpy()
    return t.numpy()


DTYPES = {"f16": torch.float16, "bf16": torch.bfloat16, "f32": torch.float32}


def main() -> None:
    parser = argparse.ArgumentParser(description=__doc__)
    parser.add_argument("--reference-src", required=True,
                        help="path to the reference project's src/ directory")
    args = parser.parse_args()
    sys.path.insert(0, str(Path(args.reference_src).resolve()))
    from qwen_int4.backends import torch_reference_linear
    from qwen_int4.quantization import (
        PackingFormat,
        dequantize_groupwise,
        pack_int4,
        quantize_asymmetric_rtn,
        quantize_symmetric_rtn,
        unpack_int4,
    )

    canonical = PackingFormat.CANONICAL
    arrays: dict[str, np.ndarray] = {}
    manifest: dict[str, dict] = {}

    # --- known-answer vectors from the reference's tests -----------------
    arrays["kat_pack_codes"] = np.array([-1, 2], dtype=np.int8)
    arrays["kat_pack_bytes"] = pack_int4(torch.tensor([-1, 2], dtype=torch.int8),
                                         packing=canonical).numpy()
    manifest["kat_pack"] = {"mirrors": "tests/test_quantization.py:22-25"}

    zero_codes = torch.tensor([-8, -1, 0, 7], dtype=torch.int8)
    arrays["kat_zero_codes"] = zero_codes.numpy()
    arrays["kat_zero_bytes"] = pack_int4(zero_codes, packing=canonical).numpy()
    manifest["kat_zero"] = {"mirrors": "tests/test_phase_e_correctness.py:102-108"}

    for i, codes in enumerate((
        [-8, -7, -1, 0, 1, 6, 7, -8],
        [7, -8, 0, -1, 3, -4, -5, 6],
    )):
        t = torch.tensor(codes, dtype=torch.int8)
        arrays[f"kat_boundary{i}_codes"] = t.numpy()
        arrays[f"kat_boundary{i}_bytes"] = pack_int4(t, packing=canonical).numpy()
    manifest["kat_boundary"] = {"mirrors": "tests/test_triton_unpack.py:28-38"}

    torch.manual_seed(20260831)
    rnd = torch.randint(0, 256, (513,), dtype=torch.uint8)
    arrays["unpack_random_bytes"] = rnd.numpy()
    arrays["unpack_random_codes"] = unpack_int4(rnd, packing=canonical, elements=1025).numpy()
    manifest["unpack_random"] = {"mirrors": "tests/test_triton_unpack.py:41-46",
                                 "seed": 20260831, "elements": 1025}

    codes = torch.tensor([[1, 2, 3, 4], [-1, -2, -3, -4]], dtype=torch.int8)
    scales = torch.tensor([[0.5, 2.0], [1.0, 0.25]], dtype=torch.float16)
    packed = pack_int4(codes, packing=canonical)
    arrays["kat_group2_qweight"] = packed.numpy()
    arrays["kat_group2_scales"] = scales.numpy()
    arrays["kat_group2_expected"] = dequantize_groupwise(
        packed, scales, out_features=2, in_features=4, group_size=2,
        packing=canonical, zeros=torch.zeros(2, dtype=torch.uint8),
    ).numpy()
    manifest["kat_group2"] = {"mirrors": "tests/test_quantization.py:35-49"}

    codes = torch.tensor([[[-8] * 64, [7] * 64]], dtype=torch.int8).reshape(1, 128)
    scales = torch.tensor([[0.25, 2.0]], dtype=torch.float16)
    zeros = pack_int4(torch.tensor([-7, 5], dtype=torch.int8), packing=canonical)
    packed = pack_int4(codes, packing=canonical)
    arrays["kat_asym_qweight"] = packed.numpy()
    arrays["kat_asym_scales"] = scales.numpy()
    arrays["kat_asym_zeros"] = zeros.numpy()
    arrays["kat_asym_expected"] = dequantize_groupwise(
        packed, scales, out_features=1, in_features=128, group_size=64,
        packing=canonical, zeros=zeros,
    ).numpy()
    manifest["kat_asym"] = {"mirrors": "tests/test_phase_e_correctness.py:111-121"}

    # --- quantiser digests (regeneration check) --------------------------
    quant_cases = []
    for name, (n, k, kind, seed, std) in {
        "q_sym_small": (6, 128, "sym", 7, 0.1),
        "q_asym_small": (6, 128, "asym", 8, 0.1),
        "q_asym_odd": (3, 64, "asym", 9, 0.1),
        "q_sym_gate": (8960, 1536, "sym", 0, 0.02),
    }.items():
        torch.manual_seed(seed)
        w = torch.randn(n, k, dtype=torch.float32) * std
        if kind == "sym":
            qw, sc = quantize_symmetric_rtn(w, group_size=64, packing=canonical)
            z = torch.zeros((n * (k // 64) + 1) // 2, 1, dtype=torch.uint8)
        else:
            qw, sc, z = quantize_asymmetric_rtn(w, group_size=64, packing=canonical)
        manifest[name] = {"n": n, "k": k, "kind": kind, "seed": seed, "std": std,
                          "qweight_sha256": sha256(qw.numpy()),
                          "scales_sha256": sha256(sc.numpy()),
                          "zeros_sha256": sha256(z.numpy())}
        quant_cases.append(name)

    # --- dequantisation, bit-exact shapes --------------------------------
    for shape in ((3, 64), (5, 128), (256, 1536)):
        n, k = shape
        torch.manual_seed(n * 10000 + k)
        w = torch.randn(shape, dtype=torch.float32) * 0.1
        qw, sc, z = quantize_asymmetric_rtn(w, group_size=64)
        expected = dequantize_groupwise(qw, sc, zeros=z, out_features=n, in_features=k,
                                        group_size=64, packing=canonical)
        key = f"deq_{n}x{k}"
        arrays[f"{key}_qweight"] = qw.numpy()
        arrays[f"{key}_scales"] = sc.numpy()
        arrays[f"{key}_zeros"] = z.numpy()
        if n * k <= 1024:
            arrays[f"{key}_expected"] = expected.numpy()
        manifest[key] = {"mirrors": "tests/test_triton_unpack.py:59-72", "n": n, "k": k,
                         "seed": n * 10000 + k, "expected_sha256": sha256(expected.numpy())}

    # --- linear forward --------------------------------------------------
    def record_linear(key, x, qw, sc, z, bias, n, k, meta):
        out = torch_reference_linear(x, qw, sc, z, bias, out_features=n, in_features=k,
                                     group_size=64, packing=canonical)
        arrays[f"{key}_out"] = as_bits(out)
        meta.update({"n": n, "k": k, "x_shape": list(x.shape),
                     "dtype": {v: kk for kk, v in DTYPES.items()}[x.dtype],
                     "bias": bias is not None})
        manifest[key] = meta

    # Triton-test shapes (asymmetric, bias), inputs regenerated from the seed.
    for rows, n, k, dt in ((1, 256, 1536, "f16"), (8, 1536, 1536, "bf16"),
                           (4, 1536, 8960, "f16")):
        seed = rows + n + k
        torch.manual_seed(seed)
        w = torch.randn(n, k, dtype=torch.float32) * 0.02
        qw, sc, z = quantize_asymmetric_rtn(w, group_size=64)
        x = torch.randn(rows, k, dtype=DTYPES[dt])
        bias = torch.randn(n, dtype=DTYPES[dt]) * 0.01
        key = f"lin_triton_{rows}x{n}x{k}_{dt}"
        arrays[f"{key}_x"] = as_bits(x)
        arrays[f"{key}_bias"] = as_bits(bias)
        record_linear(key, x, qw, sc, z, bias, n, k, {
            "mirrors": "tests/test_triton_unpack.py:93-119", "seed": seed,
            "weight": "randn*0.02 asym", "qweight_sha256": sha256(qw.numpy()),
            "scales_sha256": sha256(sc.numpy()), "zeros_sha256": sha256(z.numpy())})

    # Config 0: gate 1536->8960 symmetric RTN, bf16 W ~ N(0, 0.02), x bf16 ~ N(0,1).
    torch.manual_seed(0)
    w = (torch.randn(8960, 1536) * 0.02).to(torch.bfloat16)
    qw, sc = quantize_symmetric_rtn(w.float(), group_size=64)
    z = torch.zeros((8960 * 24 + 1) // 2, 1, dtype=torch.uint8)
    manifest["cfg0_weights"] = {"seed": 0, "weight": "(randn(8960,1536)*0.02).bf16 sym",
                                "qweight_sha256": sha256(qw.numpy()),
                                "scales_sha256": sha256(sc.numpy())}
    for m in (1, 4, 16):
        g = torch.Generator().manual_seed(100 + m)
        x = torch.randn(m, 1536, generator=g).to(torch.bfloat16)
        key = f"lin_cfg0_m{m}"
        arrays[f"{key}_x"] = as_bits(x)
        record_linear(key, x, qw, sc, z, None, 8960, 1536,
                      {"mirrors": "BASELINE config 0", "x_seed": 100 + m})

    # Config 2: AWQ-style asymmetric down_proj 8960->1536 with channel scales.
    torch.manual_seed(2)
    chan = torch.exp(torch.empty(8960).uniform_(math.log(0.5), math.log(2.0)))
    w = (torch.randn(1536, 8960) * 0.02).to(torch.bfloat16).float() * chan
    qw, sc, z = quantize_asymmetric_rtn(w, group_size=64)
    arrays["cfg2_chan"] = chan.numpy()
    manifest["cfg2_weights"] = {"seed": 2, "weight": "bf16(randn*0.02)*chan asym",
                                "qweight_sha256": sha256(qw.numpy()),
                                "scales_sha256": sha256(sc.numpy()),
                                "zeros_sha256": sha256(z.numpy())}
    for m in (1, 16):
        g = torch.Generator().manual_seed(200 + m)
        x = (torch.randn(m, 8960, generator=g) / chan).to(torch.bfloat16)
        key = f"lin_cfg2_m{m}"
        arrays[f"{key}_x"] = as_bits(x)
        record_linear(key, x, qw, sc, z, None, 1536, 8960,
                      {"mirrors": "BASELINE config 2", "x_seed": 200 + m})

    # Adversarial activations on a small asymmetric layer (fp16).
    torch.manual_seed(81)
    qw, sc, z = quantize_asymmetric_rtn(torch.randn(64, 128) * 0.05, group_size=64)
    arrays["adv_qweight"], arrays["adv_scales"], arrays["adv_zeros"] = (
        qw.numpy(), sc.numpy(), z.numpy())
    for kind in ("zero", "alternating", "bounded_large"):
        if kind == "zero":
            x = torch.zeros((2, 128), dtype=torch.float16)
        elif kind == "alternating":
            x = torch.tensor([1.0, -1.0]).repeat(2, 64).to(torch.float16)
        else:
            x = torch.linspace(-8, 8, 128).repeat(2, 1).to(torch.float16)
        key = f"lin_adv_{kind}"
        arrays[f"{key}_x"] = as_bits(x)
        record_linear(key, x, qw, sc, z, None, 64, 128,
                      {"mirrors": "tests/test_triton_unpack.py:133-154"})

    # Boundary zero points -8 / 7 (expected bit-exact in the reference's tests).
    bcodes = torch.tensor([-8, 7]).repeat(2 * 128 // 2)
    qw = pack_int4(bcodes, packing=canonical)
    z = pack_int4(torch.tensor([-8, 7, 7, -8], dtype=torch.int8), packing=canonical)
    sc = torch.tensor([[0.25, 0.5], [1.0, 2.0]], dtype=torch.float16)
    x = torch.tensor([1.0, -1.0]).repeat(64).reshape(1, 128).to(torch.float16)
    arrays["bzp_qweight"], arrays["bzp_scales"], arrays["bzp_zeros"] = (
        qw.numpy(), sc.numpy(), z.numpy())
    arrays["lin_bzp_x"] = as_bits(x)
    record_linear("lin_bzp", x, qw, sc, z, None, 2, 128,
                  {"mirrors": "tests/test_backends.py:91-104"})

    # FP32 activations (the model's down_proj input dtype) and a 3-D input with bias.
    torch.manual_seed(118)
    qw, sc, z = quantize_asymmetric_rtn(torch.randn(64, 128) * 0.1, group_size=64)
    x = torch.randn(2, 128, dtype=torch.float32)
    arrays["f32_qweight"], arrays["f32_scales"], arrays["f32_zeros"] = (
        qw.numpy(), sc.numpy(), z.numpy())
    arrays["lin_f32_x"] = as_bits(x)
    record_linear("lin_f32", x, qw, sc, z, None, 64, 128,
                  {"mirrors": "tests/test_triton_unpack.py:173-189"})

    torch.manual_seed(117)
    qw, sc, z = quantize_asymmetric_rtn(torch.randn(64, 128) * 0.1, group_size=64)
    bias = torch.randn(64, dtype=torch.bfloat16) * 0.01
    x = torch.randn(2, 3, 128, dtype=torch.bfloat16)
    arrays["d3_qweight"], arrays["d3_scales"], arrays["d3_zeros"] = (
        qw.numpy(), sc.numpy(), z.numpy())
    arrays["lin_d3_x"] = as_bits(x)
    arrays["lin_d3_bias"] = as_bits(bias)
    record_linear("lin_d3", x, qw, sc, z, bias, 64, 128,
                  {"mirrors": "tests/test_triton_unpack.py:157-170"})

    np.savez_compressed(HERE / "w4g64_golden.npz", **arrays)
    (HERE / "manifest.json").write_text(json.dumps(manifest, indent=1, sort_keys=True) + "\n")
    size = (HERE / "w4g64_golden.npz").stat().st_size
    print(f"wrote {len(arrays)} arrays ({size} bytes) and {len(manifest)} manifest entries")


if __name__ == "__main__":
    main()
