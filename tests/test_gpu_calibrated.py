"""Model-level parity on the reference-calibrated checkpoints.

The checkpoints are random-init float models calibrated and quantised by the
reference's own quantiser on 8 synthetic windows (tests/golden/make_calibrated.py,
``CKPT/iwhisper-<size>-calib-seed0``, or rebuilt from the committed compact
record i_whisper_b200/assets/calib_<size>_seed0.npz where the full checkpoint
is absent), i.e. the weights the benchmark configurations name. Unlike the hand-made synthetic checkpoint they carry
per-layer requantisation parameters from calibration: qk_frac_bits 13-15,
qk multipliers 64-127 with shifts 6-8, per-channel GeLU shifts 11-18 and so on.

* config 0 exactly (tiny, 4 + 4 layers, the seed-1 window, 32 greedy
  tokens) against digests of the reference's own Whisper_int graph and
  DecodingTask loop on its scalar C++ kernels;
* whisper-medium, all 24 + 24 layers, two windows, against the oracle
  (per-block and encoder-output digests, 8 greedy tokens);
* whisper-medium at the benchmark's batch of 256 windows (M = 384000-row
  GEMMs, the persistent schedules over ~1500 tiles per SM wave, an 18.9 GB
  head-major cross-K/V cache): windows 0 and 1 of the batch reproduce the
  same oracle digests and tokens, and the last window equals a batch-1 run;
* whisper-small and whisper-large, one window each, against the oracle
  (encoder output, 8 greedy tokens).
"""
import hashlib
import json
import os

import numpy as np
import pytest
import torch

from i_whisper_b200.checkpoint import load_calibrated, state_digest
from i_whisper_b200.synthetic import synthetic_mel_batch

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "calibrated_golden.json")


def sha(a):
    if isinstance(a, torch.Tensor):
        a = a.cpu().numpy()
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


_MODELS = {}


def calibrated_model(size):
    """(model, state dict, golden) for a calibrated checkpoint, once per size;
    skipped when the checkpoint has not been generated here."""
    if size in _MODELS:
        return _MODELS[size]
    g = json.load(open(GOLDEN))
    try:
        dims, sd = load_calibrated(size)  # the full checkpoint, or rebuilt from its committed record
    except FileNotFoundError as e:
        pytest.skip(str(e))
    assert state_digest(sd) == g["checkpoints"][size]["state_digest"], "checkpoint differs from the golden's"
    from i_whisper_b200.model import WhisperIntB200
    _MODELS.clear()  # one model on the device at a time
    torch.cuda.empty_cache()
    _MODELS[size] = (WhisperIntB200(dims, sd), sd, g)
    return _MODELS[size]


@pytest.mark.parametrize("use_graph", [False, True])
def test_config0_matches_reference_golden(use_graph):
    """tiny, seed-1 window, 32 greedy tokens."""
    from i_whisper_b200 import _lib
    model, sd, g = calibrated_model("tiny")
    c = g["tiny_config0"]
    mel = synthetic_mel_batch(80, c["mel_seeds"], float(sd["encoder.input_alpha"][0]))
    assert sha(mel) == c["mel_sha256"]
    trace = {}
    xa = model.encoder(torch.from_numpy(mel).cuda(), trace=trace)
    for k, h in enumerate(c["block_sha256"]):
        assert sha(trace[f"encoder.blocks.{k}"]) == h, f"encoder block {k}"
    assert sha(xa) == c["encoder_sha256"]
    toks = model.decode(xa, model._enc_ws[1]["rs_xa"], c["sample_len"], use_graph=use_graph, stop_when_done=True)
    assert toks.cpu().numpy().tolist() == c["tokens"]
    assert _lib.device_status(clear=True) == 0


def test_medium_all_layers_matches_oracle():
    """whisper-medium, 24 + 24 layers, windows seeded 0 and 1."""
    from i_whisper_b200 import _lib
    model, sd, g = calibrated_model("medium")
    c = g["medium_w2"]
    mel = synthetic_mel_batch(80, c["mel_seeds"], float(sd["encoder.input_alpha"][0]))
    assert [sha(m) for m in mel] == c["mel_sha256"]
    trace = {}
    xa = model.encoder(torch.from_numpy(mel).cuda(), trace=trace)
    nb = len(c["mel_seeds"])
    for b in range(nb):
        for k, h in enumerate(c["block_sha256"][b]):
            x16 = trace[f"encoder.blocks.{k}"].view(nb, 1500, -1)  # the INT15 stream, [B*T, d] on the device
            assert sha(x16[b]) == h, f"window {b}, encoder block {k}"
        assert sha(xa[b]) == c["encoder_sha256"][b], f"window {b}"
    toks = model.decode(xa, model._enc_ws[len(mel)]["rs_xa"], c["sample_len"], use_graph=True)
    assert toks.cpu().numpy().tolist() == c["tokens"]
    assert _lib.device_status(clear=True) == 0


def test_medium_batch256_matches_oracle_and_batch1():
    """The benchmark's batch: 256 windows (seeds recycled modulo 32, as the
    benchmark does) through the encoder and 8 greedy steps. Windows 0 and 1
    (seeds 0 and 1) give the oracle's digests and tokens; window 255 (seed
    31) gives what a batch of one gives."""
    from i_whisper_b200 import _lib
    from i_whisper_b200.sharding import window_seeds
    model, sd, g = calibrated_model("medium")
    c = g["medium_w2"]
    alpha = float(sd["encoder.input_alpha"][0])
    seeds = window_seeds(0, 256)
    mels = synthetic_mel_batch(80, sorted(set(seeds)), alpha)
    mel = torch.from_numpy(np.stack([mels[s] for s in seeds])).cuda()
    xa = model.encoder(mel)
    toks = model.decode(xa, model._enc_ws[256]["rs_xa"], c["sample_len"], use_graph=True)
    xa_h, toks_h = xa.cpu().numpy(), toks.cpu().numpy()
    for b in (0, 1):
        assert sha(xa_h[b]) == c["encoder_sha256"][b], f"window {b}"
        assert toks_h[b].tolist() == c["tokens"][b], f"window {b}"
    # the same window alone
    x1 = model.encoder(mel[255:].contiguous())
    t1 = model.decode(x1, model._enc_ws[1]["rs_xa"], c["sample_len"], use_graph=True)
    assert np.array_equal(x1.cpu().numpy()[0], xa_h[255])
    assert t1.cpu().numpy()[0].tolist() == toks_h[255].tolist()
    assert _lib.device_status(clear=True) == 0


def test_graphed_encoder_equals_eager():
    """encoder_graphed (one CUDA graph per batch size) gives the eager
    encoder's bytes, on two calls in a row with different inputs."""
    from i_whisper_b200 import _lib
    model, sd, g = calibrated_model("tiny")
    alpha = float(sd["encoder.input_alpha"][0])
    for seeds in ([3, 4], [5, 6]):
        mel = torch.from_numpy(synthetic_mel_batch(80, seeds, alpha)).cuda()
        ref = model.encoder(mel).clone()
        got = model.encoder_graphed(mel)
        assert torch.equal(got, ref), seeds
    assert model.graph_launches[("encoder", 2)] > 0
    assert _lib.device_status(clear=True) == 0


def test_config0_zero_point_form_matches_folded():
    """The zero-point form of every Linear_int (row sums produced by the
    LayerNorms, the attention and fc1; the GEMMs subtracting wz * rowsum),
    which the model keeps for checkpoints whose zero points do not fold into
    int8 weights, gives config 0's golden bytes as the folded form does."""
    from i_whisper_b200 import _lib
    from i_whisper_b200.model import WhisperIntB200
    g = json.load(open(GOLDEN))
    try:
        dims, sd = load_calibrated("tiny")
    except FileNotFoundError as e:
        pytest.skip(str(e))
    model = WhisperIntB200(dims, sd, fold_zero_points=False)
    assert all(L[k].wz is not None for L in model.enc_layers for k in ("qkv", "out", "fc1"))
    c = g["tiny_config0"]
    mel = synthetic_mel_batch(80, c["mel_seeds"], float(sd["encoder.input_alpha"][0]))
    xa = model.encoder(torch.from_numpy(mel).cuda())
    assert sha(xa) == c["encoder_sha256"]
    toks = model.decode(xa, model._enc_ws[1]["rs_xa"], c["sample_len"], use_graph=True, stop_when_done=True)
    assert toks.cpu().numpy().tolist() == c["tokens"]
    assert _lib.device_status(clear=True) == 0


@pytest.mark.parametrize("size", ["small", "large"])
def test_small_and_large_match_oracle(size):
    """whisper-small (12 + 12 layers, d = 768) and whisper-large (32 + 32
    layers, d = 1280, 128 mel bins, the 51866-token vocabulary) on their
    calibrated checkpoints: the seed-0 window's encoder output and 8 greedy
    tokens equal the oracle's (the windows BASELINE configurations 2 and 4
    start from)."""
    from i_whisper_b200 import _lib
    model, sd, g = calibrated_model(size)
    c = g[f"{size}_w1"]
    mel = synthetic_mel_batch(model.dims.n_mels, c["mel_seeds"], float(sd["encoder.input_alpha"][0]))
    assert [sha(m) for m in mel] == c["mel_sha256"]
    xa = model.encoder(torch.from_numpy(mel).cuda())
    for b in range(len(mel)):
        assert sha(xa[b]) == c["encoder_sha256"][b], f"window {b}"
    toks = model.decode(xa, model._enc_ws[len(mel)]["rs_xa"], c["sample_len"], use_graph=True)
    assert toks.cpu().numpy().tolist() == c["tokens"]
    assert _lib.device_status(clear=True) == 0
