"""The oracle's greedy filter chain against the reference's own logit
filters (test helper, run as a script).

Builds the reference's own DecodingTask (i_whisper/decoding.py:517-632,
``language="en"``, greedy) for each vocabulary size and checks that its
tokenizer ids, SOT sequence, blank tokens, SuppressTokens set and
max_initial_timestamp index are those of i_whisper_b200/assets/
decode_tokens.json; then applies the task's own logit filters
(SuppressBlank, SuppressTokens, ApplyTimestampRules, :426-510) and
``oracle.apply_filters_torch`` to the same float logits for token histories
of every kind (text, timestamps, pairs, EOT; 0-5 sampled tokens, with and
without a dominant timestamp block). The filtered logits must be identical.
Prints "filters ok".

Usage: python tests/reference_filters_check.py REFERENCE_ROOT
"""
import os
import sys
import types

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path[:0] = [os.path.join(HERE, "golden"), os.path.dirname(HERE)]
import make_golden as G  # noqa: E402
from oracle import oracle as O  # noqa: E402
from i_whisper_b200.model import decode_tokens  # noqa: E402

MI, _, DEC = G.import_reference(sys.argv[1], bridge=lambda: types.ModuleType("_C"))

for V, n_mels in ((51865, 80), (51866, 128)):
    t = decode_tokens(V)
    tb, eot = t["timestamp_begin"], t["eot"]
    # the reference's own DecodingTask (decoding.py:517-632) for this vocabulary
    model = MI.Whisper_int(MI.ModelDimensions(n_mels, 1500, 384, 6, 1, V, 448, 384, 6, 1))
    task = DEC.DecodingTask(model, DEC.DecodingOptions(fp16=False, language="en"))
    tok = task.tokenizer
    assert list(task.sot_sequence) == t["sot_sequence"] and task.sample_begin == len(t["sot_sequence"])
    assert (tok.sot, tok.eot, tok.no_timestamps, tok.timestamp_begin) == (t["sot"], eot, t["no_timestamps"], tb)
    assert tok.encode(" ") == t["blank"]
    kinds = [type(f).__name__ for f in task.logit_filters]
    assert kinds == ["SuppressBlank", "SuppressTokens", "ApplyTimestampRules"], kinds
    assert sorted(task.logit_filters[1].suppress_tokens) == t["suppress"]
    assert task.logit_filters[2].max_initial_timestamp_index == 50
    spec = O.DecodeTokens(sot=t["sot"], eot=eot, sot_sequence=t["sot_sequence"], no_timestamps=t["no_timestamps"],
                          timestamp_begin=tb, blank=t["blank"], suppress=t["suppress"])
    Tp = task.sample_begin
    for n_hist in (0, 1, 2, 3, 5):
        rng = np.random.default_rng(V + n_hist)
        B = 48
        logits = rng.integers(-128, 128, (B, V)).astype(np.float32) / 2.5
        logits[::3, tb:tb + 40] = rng.integers(90, 128, (len(logits[::3]), 40)) / 2.5
        hist = np.zeros((B, n_hist), np.int64)
        for b in range(B):
            for j in range(n_hist):
                r = rng.random()
                hist[b, j] = (tb + int(rng.integers(0, 1500))) if r < 0.45 else (
                    eot if r < 0.55 else int(rng.integers(0, eot)))
        tokens = torch.from_numpy(np.concatenate([np.tile(np.array(t["sot_sequence"]), (B, 1)), hist], 1))
        ref = torch.from_numpy(logits.copy())
        for f in task.logit_filters:
            f.apply(ref, tokens)
        got = torch.from_numpy(logits.copy())
        O.apply_filters_torch(got, tokens, spec, Tp)
        assert torch.equal(ref, got), (V, n_hist)
        assert torch.equal(ref.argmax(-1), got.argmax(-1))
print("filters ok")
