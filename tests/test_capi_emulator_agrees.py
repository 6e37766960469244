"""The C-ABI emulator used by the CPU tests (capi_emulator.py) rejects
arguments exactly as the product library does.

Each case below is rejected by libiwhisper_b200.so before it touches a
device, so both run here without a GPU: the real call's status code and
``iw_last_error()`` message must equal the emulator's. This keeps the
emulator's restated argument checks from drifting from capi.cu."""
import pytest

from i_whisper_b200.build import build

build()
from i_whisper_b200 import _lib  # noqa: E402

from capi_emulator import CapiEmulator  # noqa: E402

F = 0x1000  # placeholder address; never dereferenced on these paths
LIN = (F, F, F, F, F, F, F)
CASES = [
    ("iw_linear8", LIN + (-1, 16, 16, None)),
    ("iw_linear8", LIN + (4, 16, 0, None)),
    ("iw_linear8", LIN + (4, 0, 16, None)),
    ("iw_linear8_accum", (F, F, F, F, F, -1, 16, 16, None)),
    ("iw_linear32", LIN + (4, -5, 16, None)),
    ("iw_linear32_residual15", (F, F, F, F, F, F, None, 7, F, 4, 16, 16, None)),
    ("iw_linear32_residual15", (F, F, F, F, F, F, F, 7, F, 4, 16, -3, None)),
    ("iw_residual15", (F, F, 3, F, -1, None)),
    ("iw_layernorm32", (F, F, F, 1, 1, 1, 1, F, 4, 100, None)),
    ("iw_layernorm32", (F, F, F, 1, 1, 1, 1, F, -1, 1024, None)),
    ("iw_layernorm64", (F, F, F, 1, 1, 1, 1, F, 4, 96, None)),
    ("iw_layernorm64", (F, F, F, 1, 1, 1, 1, F, -2, 384, None)),
    ("iw_layernorm32_stats", (F, F, F, F, 4, 640, None)),
    ("iw_layernorm64_stats", (F, F, F, 4, 2048, None)),
    ("iw_layernorm64_stats", (F, F, F, -1, 512, None)),
    ("iw_gelu", (F, F, F, F, F, F, F, 10, 0, 1, 1, None)),
    ("iw_gelu", (F, F, F, F, F, F, F, 10, 5, 3, 1, None)),
    ("iw_gelu", (F, F, F, F, F, F, F, 10, 5, 5, 2, None)),
    ("iw_qk_requant_rowmax", (F, F, None, 1, 1, F, F, -1, 1, 1, 1, 64, None)),
    ("iw_shift_exp", (F, F, None, 0, F, F, 1, 1, 1, 1, None)),
    ("iw_shift_exp", (F, F, None, 14, F, F, 1, 1, 1, 1, None)),
    ("iw_pv_norm_requant", (F, F, F, 1, 1, 30, F, 1, 1, 1, 1, 64, None)),
    ("iw_pv_norm_requant", (F, F, F, 1, 1, -1, F, 1, 1, 1, 1, 64, None)),
    ("iw_conv1d", (F, F, F, 1, 1, 0, 1, F, 1, 4, 8, 4, 3, None)),
    ("iw_conv1d", (F, F, F, 1, 1, 1, -1, F, 1, 4, 8, 4, 3, None)),
    ("iw_conv1d", (F, F, F, 1, 1, 1, 1, F, 1, 0, 8, 4, 3, None)),
    ("iw_conv1d", (F, F, F, 1, 1, 1, 1, F, 1, 4, 0, 4, 3, None)),
    ("iw_conv1d", (F, F, F, 1, 1, 1, 1, F, 1, 4, 8, 0, 3, None)),
    ("iw_conv1d", (F, F, F, 1, 1, 1, 1, F, 1, 4, 8, 4, 0, None)),
    ("iw_conv1d", (F, F, F, 1, 1, 1, 0, F, 1, 4, 2, 4, 3, None)),
    ("iw_im2col", (F, F, 1, 4, 8, 3, 1, 1, 8, 11, 0, None)),
    ("iw_add_requant15", (F, F, F, F, F, 1, 2, 8, 3, 1, None)),
    ("iw_add_requant15", (F, F, F, F, F, 1, 2, 8, 8, 2, None)),
    ("iw_embed_add_requant15", (F, F, F, 0, F, F, F, 1, 2, 8, 4, 1, None)),
    ("iw_linear8_requant", (F, F, F, F, -1, 8, None)),
    ("iw_linear8_requant", (F, F, F, F, 2, 0, None)),
    ("iw_linear8_requant", (F, None, F, F, 2, 8, None)),
    ("iw_rounding_rshift", (F, 3, F, -1, None)),
]


@pytest.mark.parametrize("name,args", CASES, ids=[f"{n}-{i}" for i, (n, _) in enumerate(CASES)])
def test_emulator_rejects_like_the_library(name, args):
    rc = getattr(_lib.LIB, name)(*args)
    assert rc != _lib.IW_OK
    msg = _lib.last_error()
    emu = CapiEmulator()
    exc = {_lib.IW_EVALUE: ValueError, _lib.IW_EOVERFLOW: OverflowError}.get(rc, _lib.IWhisperError)
    with pytest.raises(exc) as info:
        emu.call(name, *args)
    assert str(info.value) == msg


def test_emulator_covers_the_mirror_entry_points():
    """Every C-ABI entry point the torch-facing mirror calls is emulated, so
    the reference's kernel tests exercise all of it on the CPU (the fused
    attention entry, which no reference op maps to, excepted)."""
    import os
    import re
    src = open(os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "i_whisper_b200",
                            "ops.py")).read()
    called = set(re.findall(r'_lib\.call\(\s*"(iw_[a-z0-9_]+)"', src)) | set(re.findall(r'_entry="(iw_[a-z0-9_]+)"', src))
    missing = sorted(n for n in called - {"iw_attention"} if not hasattr(CapiEmulator, n))
    assert len(called) > 15 and not missing, missing
