"""The ``i-whisper-int`` v1 checkpoint contract, on the CPU.

The reference loads ``model.safetensors`` into ``Whisper_int`` with
``load_state_dict(strict=True)`` after checking ``config.json``'s format and
version (i_whisper/__init__.py:339-417). These tests check that
``expected_keys`` reproduces the reference model's own ``state_dict()``
(keys, shapes and dtypes, from the fixture that
tests/golden/make_state_dict_contract.py writes by instantiating the
reference for every size), that a saved checkpoint loads back bit for bit,
and that the loader rejects what the reference rejects."""
import hashlib
import json
import os

import numpy as np
import pytest

from i_whisper_b200 import checkpoint as ck

HERE = os.path.dirname(os.path.abspath(__file__))
CONTRACT = json.load(open(os.path.join(HERE, "golden", "state_dict_contract.json")))


def _listing(dims):
    exp = ck.expected_keys(dims)
    return "".join(f"{k} {'x'.join(map(str, s))} {d}\n" for k, (s, d) in sorted(exp.items()))


@pytest.mark.parametrize("name", sorted(ck.DIMS))
def test_expected_keys_match_reference_state_dict(name):
    fx = CONTRACT[name]
    dims = ck.DIMS[name]
    assert fx["dims"] == dims.__dict__
    text = _listing(dims)
    if "listing" in fx:
        got, want = text.splitlines(), fx["listing"]
        assert sorted(set(got) ^ set(want)) == []
    assert len(ck.expected_keys(dims)) == fx["entries"]
    assert hashlib.sha256(text.encode()).hexdigest() == fx["sha256"]


@pytest.fixture(scope="module")
def tiny():
    dims = ck.DIMS["tiny"]
    return dims, ck.synthetic_state_dict(dims, seed=3)


def test_save_load_round_trip(tiny, tmp_path):
    dims, sd = tiny
    d = ck.save_int_checkpoint(dims, sd, str(tmp_path), "tiny")
    assert os.path.basename(d) == "iwhisper-tiny"
    for name, root in ((d, "CKPT"), ("tiny", str(tmp_path)), (os.path.join(d, "model.safetensors"), "CKPT")):
        dims2, sd2 = ck.load_int_checkpoint(name, root=root)
        assert dims2 == dims
        assert sd2.keys() == sd.keys()
        for k in sd:
            assert sd2[k].dtype == sd[k].dtype and np.array_equal(sd2[k], sd[k]), k


def test_synthetic_checkpoint_is_deterministic(tiny):
    dims, sd = tiny
    again = ck.synthetic_state_dict(dims, seed=3)
    assert all(np.array_equal(again[k], sd[k]) for k in sd)
    other = ck.synthetic_state_dict(dims, seed=4)
    assert not np.array_equal(other["encoder.conv1.weight"], sd["encoder.conv1.weight"])


def test_strict_key_and_dtype_checks(tiny):
    dims, sd = tiny
    bad = dict(sd)
    del bad["decoder.ln.bias"]
    with pytest.raises(RuntimeError, match="missing keys"):
        ck.check_state_dict(dims, bad)
    bad = dict(sd, **{"decoder.extra": np.zeros(1, np.int8)})
    with pytest.raises(RuntimeError, match="unexpected"):
        ck.check_state_dict(dims, bad)
    bad = dict(sd, **{"encoder.conv1.bias": sd["encoder.conv1.bias"].astype(np.int64)})
    with pytest.raises(RuntimeError, match="encoder.conv1.bias: expected int32"):
        ck.check_state_dict(dims, bad)
    bad = dict(sd, **{"encoder.ln_post.weight": sd["encoder.ln_post.weight"][:-1]})
    with pytest.raises(RuntimeError, match="encoder.ln_post.weight"):
        ck.check_state_dict(dims, bad)


def test_config_format_checks(tiny, tmp_path):
    dims, sd = tiny
    d = ck.save_int_checkpoint(dims, sd, str(tmp_path), "tiny")
    cfg_p = os.path.join(d, "config.json")
    cfg = json.load(open(cfg_p))
    for field, value, needle in (("format", "whisper-fp16", "Unsupported model format:"),
                                 ("format_version", 2, "Unsupported model format version")):
        json.dump(dict(cfg, **{field: value}), open(cfg_p, "w"))
        with pytest.raises(RuntimeError, match=needle):
            ck.load_int_checkpoint(d)
    json.dump(cfg, open(cfg_p, "w"))
    os.remove(os.path.join(d, "model.safetensors"))
    with pytest.raises(RuntimeError, match="Missing model tensors"):
        ck.load_int_checkpoint(d)
    with pytest.raises(RuntimeError, match="not found"):
        ck.load_int_checkpoint("no-such-size", root=str(tmp_path))
    with pytest.raises(RuntimeError, match="Expected model.safetensors"):
        ck.load_int_checkpoint(cfg_p)


REF = os.environ.get("IWHISPER_REFERENCE", os.path.join(os.path.dirname(os.path.dirname(HERE)), "reference"))


@pytest.mark.skipif(not os.path.isdir(os.path.join(REF, "i_whisper")), reason="reference checkout not available")
def test_checkpoints_interchange_with_the_reference(tmp_path):
    """Our saver's output loads in the reference's load_int_model, and the
    reference's save_int_model output loads here, bit for bit (child process:
    the reference import installs module stubs)."""
    import subprocess
    import sys
    r = subprocess.run([sys.executable, os.path.join(HERE, "reference_checkpoint_interop.py"), REF, str(tmp_path)],
                       capture_output=True, text=True, timeout=600, env=dict(os.environ, PYTHONDONTWRITEBYTECODE="1"))
    assert r.returncode == 0 and "interop ok" in r.stdout, r.stderr[-3000:]
