"""C-ABI library: loads without a GPU, exports every declared entry point, and
rejects bad arguments before touching a device (no compute calls here)."""

import ctypes
import re
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
HEADER = ROOT / "include" / "qi4_b200.h"


def declared_symbols():
    text = HEADER.read_text()
    return re.findall(r"QI4_API\s+int\s+(qi4_\w+)\s*\(", text)


def test_header_declares_the_boundary():
    names = declared_symbols()
    for required in ("qi4_w4g64_linear", "qi4_w4g64_linear_ex", "qi4_w4g64_dequant_f32",
                     "qi4_w4_unpack", "qi4_last_error", "qi4_version"):
        assert required in names
    assert len(names) == len(set(names))


def test_library_exports_every_declared_symbol(b200):
    from importlib import import_module

    lib_mod = import_module(b200.__name__ + "._lib")
    lib = lib_mod.load()
    raw = ctypes.CDLL(str(lib_mod.LIB_PATH))
    for name in declared_symbols():
        assert hasattr(raw, name), name
        assert name in lib_mod.SIGNATURES, name
    assert lib.qi4_version() == 100


def _lib(b200):
    from importlib import import_module

    mod = import_module(b200.__name__ + "._lib")
    return mod, mod.load()


def test_argument_errors_return_status_without_a_device(b200):
    mod, lib = _lib(b200)
    fake = 1 << 20  # never dereferenced: every call below fails validation first
    assert lib.qi4_w4g64_linear(None, 0, 1, 64, None, None, None, None, -1, None, 1, None) == -1
    assert "non-null" in mod.last_error()
    assert lib.qi4_w4g64_linear(fake, 0, 1, 96, fake, fake, None, None, -1, fake, 4, None) == -3
    assert "divisible by 64" in mod.last_error()
    assert lib.qi4_w4g64_linear(fake, 7, 1, 64, fake, fake, None, None, -1, fake, 4, None) == -2
    assert lib.qi4_w4g64_linear(fake, 0, 0, 64, fake, fake, None, None, -1, fake, 4, None) == -1
    assert lib.qi4_w4g64_linear(fake, 0, 1, 64, fake + 8, fake, None, None, -1, fake, 4, None) == -4
    assert "16-byte" in mod.last_error()
    assert lib.qi4_w4g64_dequant_f32(fake, fake, None, fake, 2, 100, None) == -3
    assert lib.qi4_w4_unpack(fake, fake, -1, None) == -1
    assert lib.qi4_w4_unpack(None, None, 0, None) == 0  # empty is a no-op
    with pytest.raises(ValueError, match="SHAPE"):
        mod.check(-3, "probe")
    with pytest.raises(TypeError):
        mod.check(-2, "probe")
    with pytest.raises(RuntimeError):
        mod.check(-5, "probe")


def test_last_error_truncates_and_reports_length(b200):
    mod, lib = _lib(b200)
    lib.qi4_w4g64_linear(None, 0, 1, 64, None, None, None, None, -1, None, 1, None)
    buf = ctypes.create_string_buffer(8)
    n = lib.qi4_last_error(buf, 8)
    assert n > 8 and len(buf.value) == 7


@pytest.mark.timeout(120)
def test_gemv_planner_always_terminates_with_a_valid_plan(b200):
    """The decode-GEMV launch planner, queried without a GPU over every M of the
    GEMV path, all activation dtypes and a spread of shapes: it returns, every
    CTA of a K split gets at least one 128-byte box, and the plan fits the
    shared memory the kernel is configured for."""
    _, lib = _lib(b200)
    plan = (ctypes.c_int64 * 6)()
    shapes = [(n, k) for n in (1, 7, 100, 256, 1000, 1536, 8960, 151936)
              for k in (64, 128, 192, 960, 1536, 4096, 8960, 64 * 141)]
    for sms in (148, 132, 8):
        for m in range(1, 17):
            for dtype in (0, 1, 2):
                for n, k in shapes:
                    assert lib.qi4_gemv_mma_plan(m, n, k, dtype, sms, plan) == 0, (m, n, k, dtype)
                    rows, ks, warps, bps, smem, pre = list(plan)
                    nboxes = (k // 64 + 3) // 4
                    assert rows in (16, 32, 64, 128) and warps in (2, 4, 8, 16, 32) and rows // 16 <= warps
                    # up to 16 (a non-portable cluster) only for FP32 activations that
                    # would otherwise need more than 110 KB per CTA
                    assert 1 <= ks <= (16 if dtype == 2 else 8) and bps * (ks - 1) < nboxes <= bps * ks, (m, n, k, ks, bps)
                    if ks > 8:
                        assert dtype == 2 and smem <= 110 * 1024, (m, n, k, ks, smem)
                    assert smem <= 200 * 1024, (m, n, k, dtype, smem)
                    if pre:  # single wave, at most 4 groups per warp
                        assert warps == 8 and -(-n // rows) * ks <= sms
                        assert -(-(bps * 4) // (warps // (rows // 16))) <= 4
    assert lib.qi4_gemv_mma_plan(17, 64, 64, 1, 148, plan) == -3
    assert lib.qi4_gemv_mma_plan(1, 64, 100, 1, 148, plan) == -3


def test_gemv_planner_honours_and_validates_overrides(b200):
    _, lib = _lib(b200)
    plan = (ctypes.c_int64 * 6)()
    assert lib.qi4_gemv_mma_plan_override(32, 5, 4) == 0
    try:
        assert lib.qi4_gemv_mma_plan(1, 1000, 1536, 1, 148, plan) == 0
        # 6 boxes split 5 ways: 2 boxes per CTA, so only 3 CTAs carry work
        assert list(plan)[:4] == [32, 3, 4, 2] and plan[5] == 0
    finally:
        lib.qi4_gemv_mma_plan_override(0, 0, 0)
    for bad in ((24, 1, 4), (16, 0, 4), (16, 9, 4), (16, 1, 3), (64, 1, 2)):
        assert lib.qi4_gemv_mma_plan_override(*bad) == -1


def test_gemm_override_validates_without_a_gpu(b200):
    """qi4_gemm_tc_plan_override: token-tile widths 32/64/128/192/256, K split
    1..8 only for tiles of at most 128 tokens; bn = 0 restores the planner."""
    _, lib = _lib(b200)
    try:
        for ok in ((32, 1), (64, 8), (128, 2), (192, 1), (256, 1), (0, 0)):
            assert lib.qi4_gemm_tc_plan_override(*ok) == 0, ok
        for bad in ((96, 1), (64, 0), (64, 9), (192, 2), (256, 4), (-1, 1)):
            assert lib.qi4_gemm_tc_plan_override(*bad) == -1, bad
    finally:
        lib.qi4_gemm_tc_plan_override(0, 0)


def test_bounded_wait_selftest_validates_its_limit_without_a_gpu(b200):
    """qi4_selftest_bounded_wait takes a wait limit of 1 us .. 1 s and rejects
    anything else before touching a device."""
    _, lib = _lib(b200)
    for bad in (0, 999, 1_000_000_001, 2**63):
        assert lib.qi4_selftest_bounded_wait(bad, None) == -1


def test_fused_norm_entry_points_validate_before_any_launch(b200):
    """The norm-prologue calls reject bad descriptors on the host (no GPU needed)."""
    mod, lib = _lib(b200)
    lm = __import__("importlib").import_module(b200.__name__ + "._lib")
    one = (ctypes.c_void_p * 1)(16)
    ns = (ctypes.c_int64 * 1)(64)
    assert lib.qi4_w4g64_linear_multi_norm(None, 1, 64, 1, one, one, one, one, -1, one, ns, None) == -1
    base = 1 << 20
    overlap = lm.RmsNormPrologue(base, None, -1, 1e-6, base + 4096, base + 64)  # h_out inside h_in
    assert lib.qi4_w4g64_linear_multi_norm(ctypes.byref(overlap), 1, 64, 1, one, one, one, one, -1, one, ns, None) == -1
    big = lm.RmsNormPrologue(base, None, -1, 1e-6, base + 8192, base + (1 << 16))
    assert lib.qi4_w4g64_gate_up_silu_norm(ctypes.byref(big), 17, 64, 16, 16, None, 16, 16, None, 16, 64, None) == -3
    bad_dt = lm.RmsNormPrologue(base, base + (1 << 16), 0, 1e-6, base + 8192, base + (1 << 17))
    assert lib.qi4_w4g64_gate_up_silu_norm(ctypes.byref(bad_dt), 1, 64, 16, 16, None, 16, 16, None, 16, 64, None) == -2
    misaligned = lm.RmsNormPrologue(base + 2, None, -1, 1e-6, base + 8192, base + (1 << 17))
    assert lib.qi4_w4g64_linear_multi_norm(ctypes.byref(misaligned), 1, 64, 1, one, one, one, one, -1, one, ns,
                                           None) == -4
