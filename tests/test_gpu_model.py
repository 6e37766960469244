"""Model-level parity on the GPU: WhisperIntB200 (encoder + greedy decoder)
against the reference golden fixture and against the oracle dataflow."""
import hashlib
import json
import os

import numpy as np
import pytest
import torch

from oracle import oracle as O
from i_whisper_b200.checkpoint import ModelDims, synthetic_state_dict
from i_whisper_b200.model import decode_tokens
from i_whisper_b200.synthetic import synthetic_mel_batch

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "model_golden.json")


def sha(a):
    if isinstance(a, torch.Tensor):
        a = a.cpu().numpy()
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def decode_spec(n_vocab):
    t = decode_tokens(n_vocab)
    return O.DecodeTokens(sot=t["sot"], eot=t["eot"], sot_sequence=t["sot_sequence"], no_timestamps=t["no_timestamps"],
                          timestamp_begin=t["timestamp_begin"], blank=t["blank"], suppress=t["suppress"])


@pytest.mark.parametrize("case", list(json.load(open(GOLDEN))))
@pytest.mark.parametrize("use_graph", [False, True])
def test_model_matches_reference_golden(case, use_graph):
    from i_whisper_b200.model import WhisperIntB200
    g = json.load(open(GOLDEN))[case]
    dims = ModelDims(**g["dims"])
    sd = synthetic_state_dict(dims, g["seed"])
    mel = synthetic_mel_batch(dims.n_mels, g["mel_seeds"], float(sd["encoder.input_alpha"][0]))
    model = WhisperIntB200(dims, sd)
    trace = {}
    xa = model.encoder(torch.from_numpy(mel).cuda(), trace=trace)
    for k, h in enumerate(g["block_sha256"]):
        assert sha(trace[f"encoder.blocks.{k}"].reshape(len(g["mel_seeds"]), dims.n_audio_ctx, -1)) == h, f"block {k}"
    assert sha(xa) == g["encoder_sha256"]
    toks = model.decode(xa, model._enc_ws[xa.shape[0]]["rs_xa"], g["sample_len"], use_graph=use_graph)
    ref = g["tokens"]
    assert toks.cpu().tolist() == ref


CASES = [
    # (dims, seed, mel seeds, decode steps)
    (ModelDims(80, 1500, 384, 6, 2, 51865, 448, 384, 6, 2), 3, [5, 6], 12),
    (ModelDims(80, 1500, 512, 8, 1, 51865, 448, 512, 8, 1), 4, [7], 10),
    (ModelDims(80, 1500, 768, 12, 1, 51865, 448, 768, 12, 1), 5, [8], 6),
    (ModelDims(128, 1500, 1280, 20, 1, 51866, 448, 1280, 20, 1), 6, [9], 6),
]


@pytest.mark.parametrize("dims,seed,mel_seeds,steps", CASES)
def test_model_matches_oracle(dims, seed, mel_seeds, steps):
    from i_whisper_b200.model import WhisperIntB200
    sd = synthetic_state_dict(dims, seed)
    mel = synthetic_mel_batch(dims.n_mels, mel_seeds, float(sd["encoder.input_alpha"][0]))
    odims = O.Dims(**dims.__dict__)
    xa_ref = O.encoder_forward(sd, odims, mel)
    model = WhisperIntB200(dims, sd)
    xa = model.encoder(torch.from_numpy(mel).cuda())
    assert np.array_equal(xa.cpu().numpy(), xa_ref)
    ref = O.greedy_decode(sd, odims, xa_ref, decode_spec(dims.n_vocab), steps, stop_when_done=False)
    toks = model.decode(xa, model._enc_ws[xa.shape[0]]["rs_xa"], steps, use_graph=True)
    assert toks.cpu().numpy().tolist() == ref.tolist()


def test_device_status_clean_after_model():
    from i_whisper_b200 import _lib
    assert _lib.device_status(clear=True) == 0


def test_model_layernorm64_matches_oracle():
    """Every LayerNorm_int on its LayerNorm64 backend: encoder output and
    greedy tokens against the oracle dataflow with the same variant."""
    from i_whisper_b200 import _lib
    from i_whisper_b200.model import WhisperIntB200
    dims = ModelDims(80, 1500, 512, 8, 2, 51865, 448, 512, 8, 2)
    sd = synthetic_state_dict(dims, 11)
    mel = synthetic_mel_batch(dims.n_mels, [4, 5], float(sd["encoder.input_alpha"][0]))
    odims = O.Dims(**dims.__dict__)
    xa_ref = O.encoder_forward(sd, odims, mel, layernorm="64")
    model = WhisperIntB200(dims, sd, layernorm="64")
    xa = model.encoder(torch.from_numpy(mel).cuda())
    assert np.array_equal(xa.cpu().numpy(), xa_ref)
    ref = O.greedy_decode(sd, odims, xa_ref, decode_spec(dims.n_vocab), 6, stop_when_done=False, layernorm="64")
    toks = model.decode(xa, model._enc_ws[2]["rs_xa"], 6, use_graph=True)
    assert toks.cpu().numpy().tolist() == ref.tolist()
    assert _lib.device_status(clear=True) == 0


def test_encode_batches_pipelined():
    """The host-buffer streaming API (uploads and downloads overlapping the
    neighbouring batches' compute) returns, batch for batch, what the
    device-resident encoder returns."""
    from i_whisper_b200.model import WhisperIntB200
    dims = ModelDims(80, 1500, 384, 6, 1, 51865, 448, 384, 6, 1)
    sd = synthetic_state_dict(dims, 3)
    alpha = float(sd["encoder.input_alpha"][0])
    model = WhisperIntB200(dims, sd)
    mels = [torch.from_numpy(synthetic_mel_batch(dims.n_mels, [s, s + 1], alpha)).pin_memory() for s in (0, 2, 4, 6, 8)]
    outs = [torch.empty(2, dims.n_audio_ctx, dims.n_audio_state, dtype=torch.int8).pin_memory() for _ in mels]
    model.encode_batches(mels, outs)
    torch.cuda.synchronize()
    for m, o in zip(mels, outs):
        want = model.encoder(m.cuda()).cpu()
        assert torch.equal(o, want)
    # again with the graphs already captured (three batches, reversed), and at
    # another batch size (its own buffers and graphs)
    outs2 = [torch.empty_like(o).pin_memory() for o in outs[:3]]
    model.encode_batches(mels[:3][::-1], outs2)
    torch.cuda.synchronize()
    for o, want in zip(outs2, outs[:3][::-1]):
        assert torch.equal(o, want)
    one = [m[1:].contiguous().pin_memory() for m in mels[:2]]
    outs1 = [torch.empty(1, dims.n_audio_ctx, dims.n_audio_state, dtype=torch.int8).pin_memory() for _ in one]
    model.encode_batches(one, outs1)
    torch.cuda.synchronize()
    for o, want in zip(outs1, outs[:2]):
        assert torch.equal(o[0], want[1])
    assert model.graph_launches[("encode_batches", 2)] > 0 and model.graph_launches[("encode_batches", 1)] > 0
    with pytest.raises(RuntimeError):
        model.encode_batches(mels[:1], [torch.empty(1, 3, dtype=torch.int8)])


def test_encoder_from_audio():
    """Raw audio -> GPU frontend -> encoder equals the encoder on the INT8 mel
    the same frontend produces (the frontend is checked separately)."""
    from i_whisper_b200.frontend import log_mel_int8_cuda
    from i_whisper_b200.model import WhisperIntB200
    from i_whisper_b200.synthetic import synthetic_audio
    dims = ModelDims(80, 1500, 384, 6, 1, 51865, 448, 384, 6, 1)
    sd = synthetic_state_dict(dims, 2)
    model = WhisperIntB200(dims, sd)
    audio = torch.from_numpy(np.stack([synthetic_audio(s) for s in (3, 4)])).cuda()
    got = model.encoder_from_audio(audio).clone()
    mel = log_mel_int8_cuda(audio, 80, float(sd["encoder.input_alpha"][0]))
    assert torch.equal(got, model.encoder(mel))
