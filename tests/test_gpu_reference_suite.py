"""The reference's own kernel test suite, replayed on the CUDA kernels.

vcsd-lab/I-Whisper's tests/kernels/test_*.py cannot run on a GPU box (the
reference checkout does not travel there), so tests/golden/make_reference_suite_replay.py
ran them here and recorded every ``_C`` call of every passing test
(tests/golden/reference_suite_calls.{json,npz}): the inputs, and the digest of
each output the test accepted -- hand-written known answers, rounding
boundaries, torch-golden comparisons -- or the exception class it expected.
Each recorded call is replayed here through the same ``_C`` name served by
``i_whisper_b200.ops`` on CUDA tensors (same sizes and strides, so the
non-contiguous cases stay non-contiguous) running the sm_100a kernels, and
must give the same output bytes or raise the same exception class.
"""
import pytest

from reference_replay import CALLS, replay

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def C():
    from reference_c_names import make_C
    return make_C()


@pytest.mark.parametrize("i", range(len(CALLS)), ids=[f"{i}-{c['op']}" for i, c in enumerate(CALLS)])
def test_reference_call_on_gpu(C, i):
    from i_whisper_b200 import _lib
    replay(CALLS[i], C, "cuda")
    assert _lib.device_status(clear=True) == 0
