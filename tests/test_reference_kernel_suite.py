"""The reference's own kernel test suite, run against this repository's
torch-facing mirror on the CPU.

vcsd-lab/I-Whisper tests every ``_C`` op in tests/kernels/test_*.py
(hand-written known answers, rounding boundaries, shape and dtype errors and
their exception classes, scalar ≡ SIMD cross-checks). This test runs that
suite unmodified in a child pytest, with ``i_whisper.kernels._C`` served by
``i_whisper_b200.ops`` over the C-ABI emulator (reference_suite_plugin.py,
capi_emulator.py): the mirror's argument checks, error classes and output
shapes are the product's, the arithmetic is the oracle's. The only test
expected to fail is the reference extension's greeting string
(``_C.hello``), which has no counterpart here. Skipped when the reference
checkout is absent."""
import os
import subprocess
import sys
import xml.etree.ElementTree as ET

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF = os.environ.get("IWHISPER_REFERENCE", os.path.join(os.path.dirname(ROOT), "reference"))
SUITE = os.path.join(REF, "tests", "kernels")
EXPECTED_FAILURES = {"test_cpp_extension_hello"}

pytestmark = pytest.mark.skipif(not os.path.isdir(SUITE), reason="reference checkout not available")


def test_reference_kernel_suite_passes_on_the_mirror(tmp_path):
    env = dict(os.environ, IWHISPER_REFERENCE=REF, PYTHONDONTWRITEBYTECODE="1",
               PYTHONPATH=os.pathsep.join([os.path.join(ROOT, "tests"), ROOT]))
    xml = tmp_path / "suite.xml"
    r = subprocess.run([sys.executable, "-m", "pytest", "-q", "-p", "no:cacheprovider", "-p", "reference_suite_plugin",
                        "-c", os.devnull, "--rootdir", str(tmp_path), SUITE, f"--junitxml={xml}"],
                       cwd=str(tmp_path), env=env, capture_output=True, text=True, timeout=900)
    assert xml.exists(), r.stdout[-3000:] + r.stderr[-3000:]
    passed, failed = [], []
    for case in ET.parse(xml).getroot().iter("testcase"):
        name = case.get("name").split("[")[0]
        bad = case.find("failure") is not None or case.find("error") is not None
        skipped = case.find("skipped") is not None
        if bad:
            failed.append(case.get("name"))
        elif not skipped:
            passed.append(name)
    unexpected = [n for n in failed if n.split("[")[0] not in EXPECTED_FAILURES]
    assert not unexpected, (unexpected, r.stdout[-3000:])
    assert len(passed) >= 1400, (len(passed), r.stdout[-2000:])

