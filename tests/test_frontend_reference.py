"""The float64 log-mel restatement (i_whisper_b200.synthetic.log_mel, the
checker of the GPU frontend) against the reference's own
log_mel_spectrogram (i_whisper/audio.py:216-265) run here on CPU, with its
librosa mel filterbank supplied by the same Slaney construction (librosa is
not installed). Skipped without the reference checkout."""
import os
import sys
import types

import numpy as np
import pytest
import torch

from i_whisper_b200.frontend import mel_filterbank
from i_whisper_b200.synthetic import log_mel, synthetic_audio

REF = os.environ.get("IWHISPER_REFERENCE",
                     os.path.join(os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))),
                                  "reference"))
pytestmark = pytest.mark.skipif(not os.path.isdir(os.path.join(REF, "i_whisper")), reason="no reference checkout")


@pytest.fixture(scope="module")
def ref_audio():
    sys.path.insert(0, os.path.join(os.path.dirname(__file__), "golden"))
    import make_golden as MG  # module stubs + scalar-kernel bridge for importing the reference
    from oracle import oracle as O
    if not os.path.exists(O.REF_PATH):
        pytest.skip("oracle/_ref not built")
    MG.REF = REF
    MG.import_reference()
    lib = sys.modules["librosa"]
    lib.filters = types.SimpleNamespace(mel=lambda sr, n_fft, n_mels: mel_filterbank(n_mels, n_fft, sr))
    import i_whisper.audio as A
    return A


@pytest.mark.parametrize("seed,n_mels", [(1, 80), (5, 128)])
def test_log_mel_matches_reference(ref_audio, seed, n_mels):
    audio = synthetic_audio(seed)
    want = ref_audio.log_mel_spectrogram(torch.from_numpy(audio), n_mels=n_mels).numpy()
    got = log_mel(audio, n_mels)
    assert want.shape == got.shape == (n_mels, 3000)
    assert np.max(np.abs(want - got)) < 2e-4
    q = lambda m: np.clip(np.rint(m * np.float32(100.0)), -127, 127)
    d = np.abs(q(want) - q(got))
    assert d.max() <= 1 and (d == 0).mean() > 0.999
