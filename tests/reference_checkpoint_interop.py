"""Checkpoint interchange with the reference (test helper, run as a script).

1. A checkpoint written by ``checkpoint.save_int_checkpoint`` loads in the
   reference's own ``i_whisper.load_int_model`` (i_whisper/__init__.py:339-417,
   strict key set) with every tensor bit-identical.
2. That model saved again by the reference's ``save_int_model`` (:281-335)
   loads in ``checkpoint.load_int_checkpoint`` bit-identical.

The reference is imported as tests/golden/make_golden.py imports it.
Prints "interop ok" on success.

Usage: python tests/reference_checkpoint_interop.py REFERENCE_ROOT WORK_DIR
"""
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path[:0] = [os.path.join(HERE, "golden"), os.path.dirname(HERE)]
ref_root, work = sys.argv[1], sys.argv[2]
import make_golden as G  # noqa: E402
from i_whisper_b200 import checkpoint as ck  # noqa: E402

G.import_reference(ref_root)
import i_whisper  # noqa: E402  (the reference package, with its stubs in place)

dims = ck.DIMS["tiny"]
sd = ck.synthetic_state_dict(dims, seed=5)
ours = ck.save_int_checkpoint(dims, sd, os.path.join(work, "ours"), "tiny")
model = i_whisper.load_int_model(ours, device="cpu")
ref_sd = {k: v.numpy() for k, v in model.state_dict().items()}
assert ref_sd.keys() == sd.keys()
for k in sd:
    assert ref_sd[k].dtype == sd[k].dtype and ref_sd[k].shape == sd[k].shape, k
    assert np.array_equal(ref_sd[k], sd[k]), k
i_whisper.save_int_model(model, os.path.join(work, "theirs"), "tiny")
dims2, sd2 = ck.load_int_checkpoint(os.path.join(work, "theirs", "iwhisper-tiny"))
assert dims2 == dims and sd2.keys() == sd.keys()
for k in sd:
    assert sd2[k].dtype == sd[k].dtype and np.array_equal(sd2[k], sd[k]), k
print("interop ok")
