"""Location of the vcsd-lab/I-Whisper checkout used by the fixture
generators and the reference-backed CPU tests.

Resolution order: an explicit argument, then the ``IWHISPER_REFERENCE``
environment variable, then a checkout named ``reference`` next to this
repository. Generators fail with a clear message when none exists; tests
skip.
"""
import os

REPO = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))


def reference_root(arg: str = None, required: bool = True) -> str:
    for cand in (arg, os.environ.get("IWHISPER_REFERENCE"), os.path.join(os.path.dirname(REPO), "reference")):
        if cand and os.path.isdir(os.path.join(cand, "i_whisper")):
            return os.path.abspath(cand)
    if required:
        raise SystemExit("vcsd-lab/I-Whisper checkout not found: pass its path or set IWHISPER_REFERENCE")
    return None
