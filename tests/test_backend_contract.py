"""Host-side contract of the b200 backend (CPU only).

Mirrors the fail-closed rejections of the reference's backend tests
(ryanyue-16/qwen2-int4-systems tests/test_backends.py:178-270 and
tests/test_triton_unpack.py:319-326,345-360,392-400): every bad input raises
before any launch, with the same error class and message fragment.
"""

import importlib
import sys
import types

import numpy as np
import pytest
import torch

from oracle import w4g64 as orc

GROUP = 64


def _tensors(n=6, k=128):
    values = np.arange(n * k, dtype=np.float32)
    w = ((np.remainder(values, 31) - 15) / 8).reshape(n, k)
    qw, sc, z = orc.quantize_asymmetric_rtn(w)
    return torch.from_numpy(qw), torch.from_numpy(sc), torch.from_numpy(z)


def _call(b200, x, qw, sc, z, bias=None, **override):
    args = {"out_features": 6, "in_features": 128, "group_size": GROUP, "packing": "canonical"}
    args.update(override)
    return b200.b200_w4g64_linear(x, qw, sc, z, bias, **args)


@pytest.mark.parametrize(("override", "error", "message"), [
    ({"group_size": 128}, ValueError, "W4G64"),
    ({"packing": "legacy_signed_add"}, ValueError, "canonical INT4 packing"),
    ({"in_features": 64}, ValueError, "activation feature dimension"),
    ({"in_features": 96}, ValueError, "divisible by group size 64"),
])
def test_rejects_incompatible_mapping(b200, override, error, message):
    qw, sc, z = _tensors()
    with pytest.raises(error, match=message):
        _call(b200, torch.ones(1, 128, dtype=torch.bfloat16), qw, sc, z, **override)


@pytest.mark.parametrize("target", ["qweight", "scales", "zeros", "bias"])
def test_rejects_inconsistent_tensor_shapes(b200, target):
    qw, sc, z = _tensors()
    tensors = {"qweight": qw, "scales": sc, "zeros": z, "bias": torch.zeros(6, dtype=torch.bfloat16)}
    tensors[target] = tensors[target][:-1]
    with pytest.raises(ValueError, match=target):
        _call(b200, torch.ones(1, 128, dtype=torch.bfloat16), tensors["qweight"], tensors["scales"],
              tensors["zeros"], tensors["bias"])


@pytest.mark.parametrize(("mutation", "error", "message"), [
    ("qweight_dtype", TypeError, "uint8"),
    ("zeros_dtype", TypeError, "uint8"),
    ("scales_dtype", TypeError, "FP16"),
    ("x_dtype", TypeError, "FP16, BF16, or FP32"),
])
def test_rejects_malformed_dtypes(b200, mutation, error, message):
    qw, sc, z = _tensors()
    x = torch.ones(1, 128, dtype=torch.bfloat16)
    if mutation == "qweight_dtype":
        qw = qw.to(torch.int8)
    elif mutation == "zeros_dtype":
        z = z.to(torch.int8)
    elif mutation == "scales_dtype":
        sc = sc.to(torch.float32)
    else:
        x = x.to(torch.float64)
    with pytest.raises(error, match=message):
        _call(b200, x, qw, sc, z)


def test_value_checks_reject_bad_scales_when_enabled(b200):
    qw, sc, z = _tensors()
    sc[0, 0] = float("nan")
    b200.set_value_checks(True)
    try:
        # Value checks run after the device check, so on a CPU host the device
        # error comes first; the flag itself must round-trip.
        with pytest.raises(ValueError):
            _call(b200, torch.ones(1, 128, dtype=torch.bfloat16), qw, sc, z)
    finally:
        b200.set_value_checks(False)


def test_cpu_tensors_are_rejected_not_computed(b200):
    qw, sc, z = _tensors()
    with pytest.raises(ValueError, match="CUDA tensors"):
        _call(b200, torch.ones(1, 128, dtype=torch.bfloat16), qw, sc, z)


def test_prims_reject_invalid_contracts_on_cpu_tensors(b200):
    packed = torch.zeros(4, dtype=torch.uint8)
    with pytest.raises((ValueError, RuntimeError)):
        b200.unpack_canonical_signed_int4_b200(packed)
    with pytest.raises((ValueError, RuntimeError)):
        b200.dequantize_canonical_w4g64_b200(torch.zeros(64, dtype=torch.uint8),
                                             torch.ones(2, dtype=torch.float16),
                                             torch.zeros(1, dtype=torch.uint8),
                                             out_features=1, in_features=96)


def _reference_or_skip(b200):
    q2 = importlib.import_module(b200.__name__ + ".qwen2")
    try:
        return q2, q2.reference_package()
    except ImportError:
        pytest.skip("reference package not installed here (build() installs it into baseline/_ref)")


def test_reference_quantlinear_selects_b200_backend(b200):
    """The reference's own QuantLinear (src/qwen_int4/linear.py:17-72) after
    registration: ``b200`` is an accepted backend name, unknown names are
    still rejected, and the checkpoint buffers are the ones the kernels read."""
    q2, ref = _reference_or_skip(b200)
    q2.register_with_reference(ref.__name__)
    linear = importlib.import_module(ref.__name__ + ".linear")
    layer = linear.QuantLinear(1536, 256, group_size=64, bias=True, packing="canonical")
    layer.set_backend("b200")
    assert layer.backend == "b200"
    assert "b200" in importlib.import_module(ref.__name__ + ".backends").SUPPORTED_BACKENDS
    assert layer.qweight.shape == (256 * 1536 // 2, 1) and layer.qweight.dtype == torch.uint8
    assert layer.scales.shape == (256, 24) and layer.scales.dtype == torch.float16
    assert layer.zeros.shape == ((256 * 24 + 1) // 2, 1)
    with pytest.raises(ValueError):
        layer.set_backend("environment-variable-magic")
    # On CPU tensors the b200 path fails closed (no CPU fallback).
    with pytest.raises((ValueError, RuntimeError)):
        layer(torch.zeros(1, 1536, dtype=torch.bfloat16))


def _fake_reference_package(name):
    """A stand-in with the reference's dispatch structure (backends.py:11, linear.py:51-72)."""
    pkg = types.ModuleType(name)
    pkg.__path__ = []
    backends = types.ModuleType(name + ".backends")
    backends.SUPPORTED_BACKENDS = ("torch", "lpu", "triton")
    backends.torch_reference_linear = lambda *a, **k: "torch"
    linear = types.ModuleType(name + ".linear")
    linear.SUPPORTED_BACKENDS = backends.SUPPORTED_BACKENDS

    class QuantLinear(torch.nn.Module):
        def __init__(self):
            super().__init__()
            self.backend = "torch"

        def set_backend(self, backend):
            if backend not in linear.SUPPORTED_BACKENDS:
                raise ValueError(f"unknown backend {backend!r}")
            self.backend = backend

        def forward(self, x):
            return {"torch": backends.torch_reference_linear}[self.backend](x)

    linear.QuantLinear = QuantLinear
    sys.modules[name] = pkg
    sys.modules[name + ".backends"] = backends
    sys.modules[name + ".linear"] = linear
    return backends, linear


def test_register_with_reference_adds_explicit_backend(b200):
    name = "fake_qwen_int4_for_registration"
    backends, linear = _fake_reference_package(name)
    try:
        b200.register_with_reference(name)
        b200.register_with_reference(name)  # idempotent
        assert backends.SUPPORTED_BACKENDS.count("b200") == 1
        assert linear.SUPPORTED_BACKENDS == backends.SUPPORTED_BACKENDS
        layer = linear.QuantLinear()
        assert layer(torch.zeros(1)) == "torch"  # other backends untouched
        layer.set_backend("b200")
        assert layer.backend == "b200"
        with pytest.raises(ValueError):
            layer.set_backend("b201")
    finally:
        for key in [k for k in sys.modules if k.startswith(name)]:
            del sys.modules[key]


def test_fuse_mlp_switch_routes_only_b200_projections(b200, monkeypatch):
    """``fuse_mlp`` patches the reference MLP (model.py:133-136): on the b200
    backend the fused call feeds down_proj; on other backends, or with the
    switch off again, the reference forward runs unchanged."""
    integration = importlib.import_module(b200.__name__ + ".integration")
    name = "fake_qwen_int4_for_mlp_fusion"
    backends, linear = _fake_reference_package(name)
    model = types.ModuleType(name + ".model")
    calls = []

    class QwenMLP(torch.nn.Module):
        def __init__(self):
            super().__init__()
            self.gate_proj, self.up_proj = linear.QuantLinear(), linear.QuantLinear()
            self.down_proj = lambda h: h * 2  # FP32 in, FP32 out

        def forward(self, x):
            return "reference"

    model.QwenMLP = QwenMLP
    sys.modules[name + ".model"] = model
    monkeypatch.setattr(integration, "b200_w4g64_gate_up_silu",
                        lambda x, g, u: calls.append((g, u)) or torch.ones(2, dtype=torch.float32))
    try:
        b200.register_with_reference(name, fuse_mlp=True)
        mlp = QwenMLP()
        x = torch.zeros(2, dtype=torch.bfloat16)
        assert mlp(x) == "reference"  # torch backend: untouched
        mlp.gate_proj.set_backend("b200")
        assert mlp(x) == "reference"  # only one projection on b200
        mlp.up_proj.set_backend("b200")
        b200.register_with_reference(name, fuse_mlp=True)  # idempotent
        out = mlp(x)
        assert calls == [(mlp.gate_proj, mlp.up_proj)]
        assert out.dtype == torch.bfloat16 and out.tolist() == [2.0, 2.0]
        b200.register_with_reference(name)  # switch off
        assert mlp(x) == "reference"
    finally:
        for key in [k for k in sys.modules if k.startswith(name)]:
            del sys.modules[key]


def test_grouped_linear_rejects_bad_groups_without_a_gpu(b200):
    from types import SimpleNamespace

    qw, sc, z = _tensors(64, 128)
    lay = SimpleNamespace(qweight=qw, scales=sc, zeros=z, bias=None, in_features=128, out_features=64)
    other = SimpleNamespace(qweight=qw, scales=sc, zeros=z, bias=None, in_features=192, out_features=64)
    x = torch.ones(1, 128, dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="one to three"):
        b200.b200_w4g64_linear_multi(x, [])
    with pytest.raises(ValueError, match="one to three"):
        b200.b200_w4g64_linear_multi(x, [lay] * 4)
    with pytest.raises(ValueError, match="share in_features"):
        b200.b200_w4g64_linear_multi(x, [lay, other])
    with pytest.raises(ValueError, match="CUDA tensors"):
        b200.b200_w4g64_linear_multi(x, [lay, lay])


def test_fused_gate_up_rejects_mismatched_projections_without_a_gpu(b200):
    from types import SimpleNamespace

    qw, sc, z = _tensors(64, 128)
    gate = SimpleNamespace(qweight=qw, scales=sc, zeros=z, bias=None, in_features=128, out_features=64)
    other = SimpleNamespace(qweight=qw, scales=sc, zeros=z, bias=None, in_features=192, out_features=64)
    biased = SimpleNamespace(qweight=qw, scales=sc, zeros=z, bias=torch.zeros(64), in_features=128, out_features=64)
    x = torch.ones(1, 128, dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="same shape"):
        b200.b200_w4g64_gate_up_silu(x, gate, other)
    with pytest.raises(ValueError, match="without bias"):
        b200.b200_w4g64_gate_up_silu(x, gate, biased)
    with pytest.raises(ValueError, match="CUDA tensors"):
        b200.b200_w4g64_gate_up_silu(x, gate, gate)


def _fast_and_python_errors(b200, *args, **kwargs):
    """Error type and message from the C++ fast path and from the Python checks."""
    backends = importlib.import_module(b200.__name__ + ".backends")
    results = []
    for use_fast in (True, False):
        saved = backends._fast
        if not use_fast:
            backends._fast = None
        try:
            b200.b200_w4g64_linear(*args, **kwargs)
            results.append(None)
        except (ValueError, TypeError, RuntimeError) as exc:
            results.append((type(exc), str(exc)))
        finally:
            backends._fast = saved
    return results


def test_fast_path_is_built_and_raises_like_the_python_checks(b200):
    """The C++ fast path of b200_w4g64_linear (csrc/torch_binding.cpp) is part
    of the build and rejects every malformed call with the Python wrapper's
    exception class and message (the reference's validator contract)."""
    backends = importlib.import_module(b200.__name__ + ".backends")
    assert backends._fast is not None, "the _qi4_torch fast path was not built"
    qw, sc, z = _tensors()
    x = torch.zeros(2, 128, dtype=torch.bfloat16)
    kw = {"out_features": 6, "in_features": 128, "group_size": GROUP, "packing": "canonical"}
    cases = [
        ((x, qw, sc, z, None), kw),  # CPU tensors
        ((x.int(), qw, sc, z, None), kw),
        ((torch.zeros(2, 64, dtype=torch.bfloat16), qw, sc, z, None), kw),
        ((x, qw[:-1], sc, z, None), kw),
        ((x, qw, sc[:, :1], z, None), kw),
        ((x, qw, sc.reshape(-1), z, None), kw),
        ((x, qw, sc, z[:-1], None), kw),
        ((x, qw, sc.float(), z, None), kw),
        ((x, qw.to(torch.int8), sc, z, None), kw),
        ((x, qw, sc, z, torch.zeros(5, dtype=torch.bfloat16)), kw),
        ((x, qw, sc, z, torch.zeros(6, dtype=torch.int32)), kw),
        ((x, qw, sc, z, None), dict(kw, out_features=0)),
        ((x, qw, sc, z, None), dict(kw, in_features=96)),
    ]
    for args, kwargs in cases:
        fast, python = _fast_and_python_errors(b200, *args, **kwargs)
        assert fast is not None and fast == python, (fast, python)
