"""Generate ``decode_tokens.json``: the special-token ids the greedy loop of
vcsd-lab/I-Whisper uses, read from the reference's own tokenizer.

DecodingTask (i_whisper/decoding.py:517-632) derives from the tokenizer:
the SOT sequence for ``language="en", task="transcribe"``, EOT, the
timestamp range, ``encode(" ")`` (SuppressBlank), and the SuppressTokens set
for ``suppress_tokens="-1"`` (non_speech_tokens + transcribe, translate, sot,
sot_prev, sot_lm, no_speech). They depend only on the vocabulary size
(51865 multilingual, 51866 for large-v3), so they are computed once here, in
a checkout that has the reference, and shipped as data.

Usage: python i_whisper_b200/assets/make_decode_tokens.py [REFERENCE_ROOT]
(default: $IWHISPER_REFERENCE, else a checkout named ``reference`` next to
this repository; it is an error when neither exists)
"""
import json
import os
import sys

import types

_repo = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
ref = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("IWHISPER_REFERENCE",
                                                           os.path.join(os.path.dirname(_repo), "reference"))
if not os.path.isdir(os.path.join(ref, "i_whisper")):
    sys.exit(f"vcsd-lab/I-Whisper checkout not found at {ref!r}: pass its path or set IWHISPER_REFERENCE")
# The reference package imports bitsandbytes, matplotlib and librosa at
# import time; none is used by the tokenizer, so empty stand-ins suffice.
for name in ("bitsandbytes", "bitsandbytes.functional", "matplotlib", "matplotlib.pyplot", "librosa"):
    sys.modules.setdefault(name, types.ModuleType(name))
sys.modules["bitsandbytes"].functional = sys.modules["bitsandbytes.functional"]
sys.modules["bitsandbytes.functional"].int8_linear_matmul = None
sys.modules["matplotlib"].pyplot = sys.modules["matplotlib.pyplot"]
_k = types.ModuleType("i_whisper.kernels")
_k._C = types.ModuleType("_C")
sys.modules["i_whisper.kernels"] = _k
sys.modules["i_whisper.kernels._C"] = _k._C
sys.path.insert(0, ref)
from i_whisper.tokenizer import get_tokenizer  # noqa: E402

out = {}
for n_vocab in (51865, 51866):
    is_multilingual = n_vocab >= 51865
    num_languages = n_vocab - 51765 - int(is_multilingual)
    tok = get_tokenizer(is_multilingual, num_languages=num_languages, language="en", task="transcribe")
    suppress = [t for t in [-1] if t >= 0]
    suppress.extend(tok.non_speech_tokens)
    suppress.extend([tok.transcribe, tok.translate, tok.sot, tok.sot_prev, tok.sot_lm])
    if tok.no_speech is not None:
        suppress.append(tok.no_speech)
    out[str(n_vocab)] = {
        "sot": tok.sot,
        "eot": tok.eot,
        "sot_sequence": list(tok.sot_sequence),
        "no_timestamps": tok.no_timestamps,
        "timestamp_begin": tok.timestamp_begin,
        "blank": tok.encode(" "),
        "suppress": sorted(set(suppress)),
        "no_speech": tok.no_speech,
    }
path = os.path.join(os.path.dirname(os.path.abspath(__file__)), "decode_tokens.json")
with open(path, "w") as f:
    json.dump(out, f, indent=1)
print(path)
