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

from capi_emulator import install
from reference_c_names import make_C as _make_C


def _install_reference():
    sys.path.insert(0, os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden"))
    import make_golden
    make_golden.import_reference(os.environ["IWHISPER_REFERENCE"], bridge=_make_C)


def pytest_configure(config):
    install(lambda obj, name, value: setattr(obj, name, value))
    _install_reference()
