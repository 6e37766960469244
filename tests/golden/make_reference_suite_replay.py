"""Generate tests/golden/reference_suite_calls.{npz,json}: the ``_C`` calls of
the reference's own kernel test suite, for replay on the GPU.

The reference checkout cannot travel to a GPU box, so its test files cannot
run there. This script runs them here (vcsd-lab/I-Whisper tests/kernels,
unmodified, in a child pytest) with ``i_whisper.kernels._C`` served by this
repository's operator mirror over the C-ABI emulator, and records every call
of every passing test with reference_suite_recorder.py: inputs (deduplicated
arrays in the .npz), and the digest of each output or the exception class.
tests/test_gpu_reference_suite.py replays the calls on the CUDA kernels.

Usage: python tests/golden/make_reference_suite_replay.py [REFERENCE_ROOT]
"""
import json
import os
import subprocess
import sys
import tempfile

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, HERE)
from refroot import reference_root  # noqa: E402

OUT = os.path.join(HERE, "reference_suite_calls")


def main():
    ref = reference_root(sys.argv[1] if len(sys.argv) > 1 else None)
    env = dict(os.environ, IWHISPER_REFERENCE=ref, IWHISPER_RECORD_OUT=OUT, PYTHONDONTWRITEBYTECODE="1",
               PYTHONPATH=os.pathsep.join([HERE, os.path.join(ROOT, "tests"), ROOT]))
    with tempfile.TemporaryDirectory() as tmp:
        r = subprocess.run([sys.executable, "-m", "pytest", "-q", "-p", "no:cacheprovider", "-p",
                            "reference_suite_recorder", "-c", os.devnull, "--rootdir", tmp,
                            os.path.join(ref, "tests", "kernels")], cwd=tmp, env=env, capture_output=True, text=True)
    print(r.stdout.strip().splitlines()[-1])
    calls = json.load(open(OUT + ".json"))["calls"]
    n_err = sum("raises" in c for c in calls)
    tests = len({c["test"] for c in calls})
    print(f"{len(calls)} distinct calls ({n_err} expected errors) from {tests} passing tests; "
          f"{os.path.getsize(OUT + '.npz') / 1e6:.1f} MB of inputs")


if __name__ == "__main__":
    main()
