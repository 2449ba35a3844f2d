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
