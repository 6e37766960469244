"""The C-ABI library loads without a GPU and exports every entry point that
include/*.h declares (no compute calls)."""
import ctypes
import glob
import os
import re

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    names = set()
    for h in glob.glob(os.path.join(ROOT, "include", "*.h")):
        src = open(h).read()
        src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
        names |= set(re.findall(r"\b(iw_[a-z0-9_]+)\s*\(", src))
    return names


def test_header_declares_entry_points():
    names = declared_symbols()
    for required in ("iw_linear8", "iw_linear32_residual15", "iw_layernorm32", "iw_attention", "iw_conv1d",
                     "iw_classifier", "iw_last_error"):
        assert required in names


def test_library_exports_every_declared_symbol():
    from i_whisper_b200.build import LIB_PATH, build
    build()
    lib = ctypes.CDLL(LIB_PATH)
    missing = [n for n in sorted(declared_symbols()) if not hasattr(lib, n)]
    assert not missing, missing


def test_python_binding_covers_header():
    from i_whisper_b200 import _lib
    names = declared_symbols() - {"iw_last_error"}
    assert names <= set(_lib.SIGNATURES), names - set(_lib.SIGNATURES)
    assert _lib.LIB.iw_abi_version() == 1
    assert isinstance(_lib.last_error(), str)  # other tests may have left a message
