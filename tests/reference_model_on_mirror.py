"""Run the reference's own ``Whisper_int`` graph and greedy loop with this
repository's operator mirror as its ``_C`` (test helper, run as a script).

Builds the reference model exactly as tests/golden/make_golden.py does
(one of its golden cases, synthetic checkpoint, every module on the ``scalar``
backend), but with ``i_whisper.kernels._C.<op>_scalar`` served by
``i_whisper_b200.ops.<op>_cuda`` over the C-ABI emulator
(capi_emulator.py) instead of the reference's compiled kernels. Prints one
JSON object with the same digests and token ids as model_golden.json.

Usage: python tests/reference_model_on_mirror.py REFERENCE_ROOT [CASE]
"""
import json
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path[:0] = [HERE, os.path.join(HERE, "golden"), os.path.dirname(HERE)]

import capi_emulator  # noqa: E402
import reference_suite_plugin as plugin  # noqa: E402

capi_emulator.install(lambda obj, name, value: setattr(obj, name, value))
REF, CASE = sys.argv[1], (sys.argv[2] if len(sys.argv) > 2 else "mini")
import make_golden as G  # noqa: E402

MI, ML, DEC = G.import_reference(REF, bridge=plugin._make_C)
cases = dict(G.GOLDEN_CASES, **G.GOLDEN_CASES_LN64)
print(json.dumps(G.run_reference(MI, ML, DEC, cases[CASE], "scalar")))
