"""Replay of the recorded ``_C`` calls of the reference's kernel test suite
(tests/golden/reference_suite_calls.{json,npz}, made by
tests/golden/make_reference_suite_replay.py) through the operator mirror
(test helper, used by the GPU replay and by its CPU check on the emulator)."""
import hashlib
import json
import os

import numpy as np
import torch

HERE = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
CALLS = json.load(open(os.path.join(HERE, "reference_suite_calls.json")))["calls"]
_ARRAYS = {}


def _array(d):
    if not _ARRAYS:
        with np.load(os.path.join(HERE, "reference_suite_calls.npz")) as z:
            _ARRAYS.update({k: z[k] for k in z.files})
    return _ARRAYS[d]


def digest(a: np.ndarray) -> str:
    h = hashlib.sha256()
    h.update(str(a.dtype).encode())
    h.update(str(a.shape).encode())
    h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()


def _arg(spec, device):
    if "py" in spec:
        return spec["py"]
    vals = torch.from_numpy(_array(spec["tensor"]).copy()).reshape(spec["size"])
    # same sizes and strides as the recorded argument (non-contiguous stays so)
    t = torch.empty_strided(spec["size"], spec["stride"], dtype=vals.dtype, device=device)
    t.copy_(vals)
    assert t.is_contiguous() == spec["contiguous"]
    return t


def replay(c, C, device):
    """Run recorded call ``c`` through module ``C`` on ``device``; assert the
    recorded output digests, or the recorded exception class."""
    fn = getattr(C, c["op"])
    args = [_arg(a, device) for a in c["args"]]
    kwargs = {k: _arg(v, device) for k, v in c["kwargs"].items()}
    if "raises" in c:
        try:
            fn(*args, **kwargs)
            if device != "cpu":
                torch.cuda.synchronize()
        except Exception as e:  # noqa: BLE001 -- the class is what is checked
            assert type(e).__name__ == c["raises"], (c["test"], repr(e))
            return
        raise AssertionError(f"{c['test']}: expected {c['raises']}")
    out = fn(*args, **kwargs)
    outs = out if isinstance(out, tuple) else (out,)
    assert isinstance(out, tuple) == c["result"]["tuple"], c["test"]
    assert len(outs) == len(c["result"]["outputs"]), c["test"]
    for t, spec in zip(outs, c["result"]["outputs"]):
        assert t.device.type == torch.device(device).type, c["test"]
        a = t.cpu().numpy()
        assert str(t.dtype).replace("torch.", "") == spec["dtype"] and list(a.shape) == spec["size"], c["test"]
        assert digest(a) == spec["sha256"], c["test"]
