"""The operator mirror as a drop-in ``_C`` under the reference's own model.

A child process builds the reference ``Whisper_int`` (each golden case) and runs
its encoder and its ``DecodingTask`` greedy loop with every ``_C.<op>_scalar``
call served by ``i_whisper_b200.ops`` (argument checks, shapes and dtypes of
the product; arithmetic of the oracle behind the emulated C ABI), and must
reproduce the digests and token ids that the reference's compiled kernels
produced (tests/golden/model_golden.json). Skipped when the reference
checkout is absent."""
import json
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF = os.environ.get("IWHISPER_REFERENCE", os.path.join(os.path.dirname(ROOT), "reference"))

pytestmark = pytest.mark.skipif(not os.path.isdir(os.path.join(REF, "i_whisper")),
                                reason="reference checkout not available")


GOLDENS = [os.path.join(ROOT, "tests", "golden", f) for f in ("model_golden.json", "model_golden_ln64.json")]
CASES = [(p, c) for p in GOLDENS for c in json.load(open(p))]


@pytest.mark.parametrize("path,case", CASES, ids=[c for _, c in CASES])
def test_reference_model_runs_on_the_mirror(path, case):
    r = subprocess.run([sys.executable, os.path.join(ROOT, "tests", "reference_model_on_mirror.py"), REF, case],
                       capture_output=True, text=True, timeout=900, env=dict(os.environ, PYTHONDONTWRITEBYTECODE="1"))
    assert r.returncode == 0, r.stderr[-3000:]
    got = json.loads(r.stdout.strip().splitlines()[-1])
    gold = json.load(open(path))[case]
    for key in ("mel_sha256", "encoder_sha256", "block_sha256", "tokens"):
        assert got[key] == gold[key], key
