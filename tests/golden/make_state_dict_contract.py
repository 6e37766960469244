"""Generate tests/golden/state_dict_contract.json from the REFERENCE itself.

Instantiates vcsd-lab/I-Whisper's own ``Whisper_int`` (i_whisper/model_int.py)
for every model size and records its ``state_dict()`` contract: the number
of entries and a SHA-256 of the sorted ``key shape dtype`` listing, plus the
full listing for ``tiny``. ``load_state_dict(strict=True)`` accepts exactly
this key set, so the checkpoint loader's ``expected_keys`` must reproduce it.
The reference is imported the way make_golden.py imports it (stubbed
bitsandbytes, matplotlib and librosa; the scalar kernels of oracle/_ref behind
``_C``, although construction calls none of them).

Usage: python tests/golden/make_state_dict_contract.py [REFERENCE_ROOT]
"""
import hashlib
import json
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)

import make_golden as G  # noqa: E402  (also puts the repo root on sys.path)
from i_whisper_b200.checkpoint import DIMS  # noqa: E402


def listing(entries):
    """Canonical text of a {key: (shape, dtype)} contract."""
    return "".join(f"{k} {'x'.join(map(str, s))} {d}\n" for k, (s, d) in sorted(entries.items()))


def main():
    MI, _, _ = G.import_reference()
    out = {}
    for name, dims in DIMS.items():
        model = MI.Whisper_int(MI.ModelDimensions(**dims.__dict__))
        sd = {k: (tuple(v.shape), str(v.dtype).replace("torch.", "")) for k, v in model.state_dict().items()}
        del model
        text = listing(sd)
        out[name] = dict(dims=dims.__dict__, entries=len(sd), sha256=hashlib.sha256(text.encode()).hexdigest())
        if name == "tiny":
            out[name]["listing"] = text.splitlines()
        print(name, len(sd), out[name]["sha256"][:16])
    with open(os.path.join(HERE, "state_dict_contract.json"), "w") as f:
        json.dump(out, f, indent=1)


if __name__ == "__main__":
    main()
