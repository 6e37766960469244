"""pytest plugin (fixture generator): record every ``_C`` call the
reference's own kernel test suite makes, for replay on the GPU.

Loaded by tests/golden/make_reference_suite_replay.py when it runs the
reference's tests/kernels/test_*.py (vcsd-lab/I-Whisper) here, with ``_C``
served by this repository's operator mirror over the C-ABI emulator (the
setup of tests/reference_suite_plugin.py). Each call is recorded with the
test that made it: the positional and keyword arguments (tensors with their
sizes, strides and bytes; Python values as they are), and either the
sha256 digest, dtype and shape of every tensor it returned or the class of
the exception it raised. Only calls of tests that passed are kept: their
results are the ones the reference's tests accept (hand-written known
answers, rounding boundaries, torch-golden comparisons, error classes).
Identical calls (the suites call ``*_scalar`` and ``*_simd`` with the same
inputs, and the mirror serves both) are stored once, and calls whose inputs
exceed MAX_CALL_BYTES are left out to keep the fixture small (the count is
recorded).
"""
import hashlib
import json
import os

import numpy as np
import torch

import reference_suite_plugin as base

OUT = os.environ["IWHISPER_RECORD_OUT"]
MAX_CALL_BYTES = 64 * 1024
_records = []      # (nodeid, record)
_pending = []
_arrays = {}       # digest -> numpy array (inputs, deduplicated)
_current = {"id": None}


def _digest(a: np.ndarray) -> str:
    h = hashlib.sha256()
    h.update(str(a.dtype).encode())
    h.update(str(a.shape).encode())
    h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()


def _np(t: torch.Tensor) -> np.ndarray:
    return t.detach().contiguous().cpu().numpy()


def _arg_spec(v):
    if isinstance(v, torch.Tensor):
        a = _np(v)
        d = _digest(a)
        _arrays.setdefault(d, a)
        return {"tensor": d, "dtype": str(v.dtype).replace("torch.", ""), "size": list(v.shape),
                "stride": list(v.stride()), "contiguous": bool(v.is_contiguous())}
    if v is None or isinstance(v, (bool, int, float, str)):
        return {"py": v}
    raise TypeError(f"unrecorded argument type {type(v)}")


def _out_spec(o):
    outs = o if isinstance(o, tuple) else (o,)
    specs = []
    for t in outs:
        a = _np(t)
        specs.append({"sha256": _digest(a), "dtype": str(t.dtype).replace("torch.", ""), "size": list(t.shape)})
    return {"tuple": isinstance(o, tuple), "outputs": specs}


def _wrap(op, fn):
    def call(*args, **kwargs):
        try:
            rec = {"op": op, "args": [_arg_spec(a) for a in args],
                   "kwargs": {k: _arg_spec(v) for k, v in kwargs.items()}}
        except TypeError:
            return fn(*args, **kwargs)
        try:
            out = fn(*args, **kwargs)
        except Exception as e:  # the reference tests check these classes
            rec["raises"] = type(e).__name__
            _pending.append(rec)
            raise
        rec["result"] = _out_spec(out)
        _pending.append(rec)
        return out
    return call


_orig_make_C = base._make_C


def _make_C():
    C = _orig_make_C()
    for name in dir(C):
        fn = getattr(C, name)
        if callable(fn) and not name.startswith("__"):
            setattr(C, name, _wrap(name, fn))
    return C


base._make_C = _make_C


def pytest_configure(config):
    base.pytest_configure(config)


def pytest_runtest_logreport(report):
    if report.when == "setup":
        _pending.clear()
    if report.when == "call":
        if report.passed:
            _records.extend((report.nodeid, r) for r in _pending)
        _pending.clear()


def pytest_sessionfinish(session, exitstatus):
    seen, calls, too_big = set(), [], 0
    for nodeid, r in _records:
        ins = {a["tensor"] for a in list(r["args"]) + list(r["kwargs"].values()) if "tensor" in a}
        if sum(_arrays[d].nbytes for d in ins) > MAX_CALL_BYTES:
            too_big += 1
            continue
        key = json.dumps({k: v for k, v in r.items() if k != "op"}, sort_keys=True) + r["op"].replace("_simd", "_scalar")
        if key in seen:
            continue
        seen.add(key)
        calls.append(dict(r, test=nodeid))
    used = {a["tensor"] for c in calls for a in list(c["args"]) + list(c["kwargs"].values()) if "tensor" in a}
    np.savez_compressed(OUT + ".npz", **{d: _arrays[d] for d in sorted(used)})
    with open(OUT + ".json", "w") as f:
        json.dump({"calls": calls, "left_out_over_max_bytes": too_big, "max_call_bytes": MAX_CALL_BYTES}, f,
                  separators=(",", ":"))
