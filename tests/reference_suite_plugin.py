"""pytest plugin: serve the reference's ``i_whisper.kernels._C`` from this
repository's torch-facing mirror (test helper).

Loaded with ``-p reference_suite_plugin`` by tests/test_reference_kernel_suite.py
when it runs the reference's own kernel tests (tests/kernels/test_*.py of
vcsd-lab/I-Whisper). Every ``_C.<op>_scalar`` / ``_C.<op>_simd`` the mirror
covers becomes ``i_whisper_b200.ops.<op>_cuda`` running on CPU tensors through
the C-ABI emulator (tests/capi_emulator.py, the oracle behind the C ABI), so
the reference tests exercise the mirror's argument checks, error classes,
output shapes and dtypes, and the oracle's arithmetic against their
hand-written expected values. Ops the mirror does not provide are absent from
the module, as they would be from a build without them. The reference root
comes from IWHISPER_REFERENCE; the packages its top-level import needs and
the CPU path never calls (bitsandbytes, matplotlib, librosa) are stubbed.
"""
import os
import sys
import types

from capi_emulator import install
from i_whisper_b200 import ops

# reference _C name (without the _scalar/_simd suffix) -> mirror function
MIRROR = {
    "linear8": ops.linear8_cuda,
    "linear8_accum_{}_debug": ops.linear8_accum_cuda_debug,
    "linear32": ops.linear32_cuda,
    "linear32_accum_{}_debug": ops.linear32_accum_cuda_debug,
    "linear8_requant_{}_debug": ops.linear8_requant_cuda_debug,
    "linear32_requant_{}_debug": ops.linear32_requant_cuda_debug,
    "residual15": ops.residual15_cuda,
    "layernorm32": ops.layernorm32_cuda,
    "layernorm32_stats": ops.layernorm32_stats_cuda,
    "layernorm32_rsqrt": ops.layernorm32_rsqrt_cuda,
    "layernorm64": ops.layernorm64_cuda,
    "layernorm64_stats": ops.layernorm64_stats_cuda,
    "gelu": ops.gelu_cuda,
    "qk": ops.qk_cuda,
    "qk_requant_rowmax": ops.qk_requant_rowmax_cuda,
    "shift_exp": ops.shift_exp_cuda,
    "pv": ops.pv_cuda,
    "pv_norm_requant": ops.pv_norm_requant_cuda,
    "conv1d_accum": ops.conv1d_accum_cuda,
    "conv1d": ops.conv1d_cuda,
    "add_requant15": ops.add_requant15_cuda,
    "classifier_accum": ops.classifier_accum_cuda,
    "classifier": ops.classifier_cuda,
}


def _make_C():
    C = types.ModuleType("i_whisper.kernels._C")
    C.rounding_rshift_debug = ops.rounding_rshift_debug_cuda
    for name, fn in MIRROR.items():
        for backend in ("scalar", "simd"):
            key = name.format(backend) if "{}" in name else f"{name}_{backend}"
            setattr(C, key, fn)
    return C


def _install_reference():
    sys.path.insert(0, os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden"))
    import make_golden
    make_golden.import_reference(os.environ["IWHISPER_REFERENCE"], bridge=_make_C)


def pytest_configure(config):
    install(lambda obj, name, value: setattr(obj, name, value))
    _install_reference()
