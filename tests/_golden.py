"""Load the committed golden fixtures and rebuild the seeded inputs they describe.

The fixtures were produced by ``tests/golden/make_golden.py`` from the
reference implementation. Large weights are regenerated here from their seed
with ``torch.randn`` and the oracle quantiser; ``regen_*`` checks the bytes
against the SHA-256 digests of the reference quantiser's output.
"""

from __future__ import annotations

import hashlib
import json
import math
from functools import lru_cache
from pathlib import Path

import numpy as np
import torch

from oracle import w4g64 as orc

GOLDEN = Path(__file__).resolve().parent / "golden"
DTYPES = {"f16": torch.float16, "bf16": torch.bfloat16, "f32": torch.float32}


@lru_cache(maxsize=1)
def arrays() -> dict:
    with np.load(GOLDEN / "w4g64_golden.npz") as data:
        return {k: data[k] for k in data.files}


@lru_cache(maxsize=1)
def manifest() -> dict:
    return json.loads((GOLDEN / "manifest.json").read_text())


def sha256(array: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(array).tobytes()).hexdigest()


def to_tensor(bits: np.ndarray, dtype: str) -> torch.Tensor:
    """Rebuild a torch tensor from the stored representation of ``dtype``."""
    if dtype in ("f16", "bf16"):
        return torch.from_numpy(bits.astype(np.uint16).view(np.int16).copy()).view(DTYPES[dtype])
    return torch.from_numpy(np.ascontiguousarray(bits, dtype=np.float32).copy())


def to_f32(bits: np.ndarray, dtype: str) -> np.ndarray:
    return to_tensor(bits, dtype).to(torch.float32).numpy()


def regen_quant(n: int, k: int, kind: str, seed: int, std: float, bf16_weight: bool = False):
    """Seeded weights through the oracle quantiser -> (qweight, scales, zeros) numpy."""
    torch.manual_seed(seed)
    w = torch.randn(n, k, dtype=torch.float32) * std
    if bf16_weight:
        w = w.to(torch.bfloat16).float()
    w = w.numpy()
    if kind == "sym":
        qw, sc = orc.quantize_symmetric_rtn(w)
        z = np.zeros(((n * (k // 64) + 1) // 2, 1), dtype=np.uint8)
    else:
        qw, sc, z = orc.quantize_asymmetric_rtn(w)
    return qw, sc, z


@lru_cache(maxsize=None)
def linear_case(key: str):
    """Inputs and reference output of a recorded linear case.

    Returns a dict with numpy ``qweight``, ``scales``, ``zeros``; torch ``x``
    and ``bias`` (CPU, original dtype); ``expected`` (torch, x dtype); ``n``,
    ``k``, ``dtype``.
    """
    a, meta = arrays(), manifest()[key]
    n, k, dt = meta["n"], meta["k"], meta["dtype"]
    if key.startswith("lin_triton_"):
        torch.manual_seed(meta["seed"])
        w = (torch.randn(n, k, dtype=torch.float32) * 0.02).numpy()
        qw, sc, z = orc.quantize_asymmetric_rtn(w)
        assert sha256(qw) == meta["qweight_sha256"]
        assert sha256(sc) == meta["scales_sha256"]
        assert sha256(z) == meta["zeros_sha256"]
    elif key.startswith("lin_cfg0_"):
        qw, sc, z = cfg0_weights()
    elif key.startswith("lin_cfg2_"):
        qw, sc, z = cfg2_weights()
    else:
        prefix = {"lin_adv": "adv", "lin_bzp": "bzp", "lin_f32": "f32", "lin_d3": "d3"}[
            "_".join(key.split("_")[:2])]
        qw, sc, z = a[f"{prefix}_qweight"], a[f"{prefix}_scales"], a[f"{prefix}_zeros"]
    x = to_tensor(a[f"{key}_x"], dt).reshape(meta["x_shape"])
    bias = to_tensor(a[f"{key}_bias"], dt) if meta["bias"] else None
    if key == "lin_d3":
        bias = to_tensor(a["lin_d3_bias"], "bf16")
    expected = to_tensor(a[f"{key}_out"], dt).reshape(*meta["x_shape"][:-1], n)
    return {"qweight": qw, "scales": sc, "zeros": z, "x": x, "bias": bias,
            "expected": expected, "n": n, "k": k, "dtype": dt}


@lru_cache(maxsize=1)
def cfg0_weights():
    meta = manifest()["cfg0_weights"]
    qw, sc, z = regen_quant(8960, 1536, "sym", 0, 0.02, bf16_weight=True)
    assert sha256(qw) == meta["qweight_sha256"]
    assert sha256(sc) == meta["scales_sha256"]
    return qw, sc, z


@lru_cache(maxsize=1)
def cfg2_weights():
    meta = manifest()["cfg2_weights"]
    torch.manual_seed(2)
    chan = torch.exp(torch.empty(8960).uniform_(math.log(0.5), math.log(2.0)))
    assert np.array_equal(chan.numpy(), arrays()["cfg2_chan"])
    w = ((torch.randn(1536, 8960) * 0.02).to(torch.bfloat16).float() * chan).numpy()
    qw, sc, z = orc.quantize_asymmetric_rtn(w)
    assert sha256(qw) == meta["qweight_sha256"]
    assert sha256(sc) == meta["scales_sha256"]
    assert sha256(z) == meta["zeros_sha256"]
    return qw, sc, z


LINEAR_CASES = sorted(k for k in manifest() if k.startswith("lin_"))
