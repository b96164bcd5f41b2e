"""CPU-side checks of the native library: it is built, loads and exports every entry point that
include/sumac_b200.h declares (no compute: there is no GPU here)."""
import ctypes
import os
import re

from sumac_b200 import _native

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def header_symbols():
    text = open(os.path.join(ROOT, "include", "sumac_b200.h")).read()
    return set(re.findall(r"\b(sumac_[a-z0-9_]+)\s*\(", text))


def test_library_exports_all_header_symbols():
    from sumac_b200 import build
    build.build()
    lib = ctypes.CDLL(_native.LIB_PATH)
    for name in header_symbols():
        assert hasattr(lib, name), name


def test_binding_covers_header():
    assert header_symbols() == set(_native.exported_symbols())


def test_padded_rank_without_gpu():
    lib = _native.lib()
    assert [lib.sumac_padded_rank(d) for d in (1, 8, 16, 17, 33, 100, 256, 257)] == \
        [16, 16, 16, 32, 64, 128, 256, 0]
