"""The reference-calibrated benchmark checkpoints, rebuilt from a compact
record.

The benchmark configurations name "random-init weights from seed 0,
calibrated with the repo's quantize.py on 8 synthetic windows". The
full checkpoints (tests/golden/make_calibrated.py runs the reference's
quantiser to make them) hold 38 MB (tiny) to 0.77 GB (medium) of INT8
weights, too much to ship. Almost all of it is determined by torch's own
seeded initialisation: every linear weight of the reference's
``Whisper_quantized`` is ``nn.Linear``'s default init drawn in construction
order after ``torch.manual_seed(0)``, and the quantiser maps it to INT8 as
``round(W * wgt_alpha + wgt_zeros)`` clamped to +-127
(model_quant.py:652-745, ``quantize_layer``); the token embedding is
``nn.Embedding``'s normal init mapped as ``round(E * wgt_alpha)``
(model_quant.py:2046-2099). So the record (assets/calib_<size>_seed0.npz)
keeps every other tensor of the INT8 state dict as it is, plus the float32
``wgt_alpha`` scales; ``rebuild`` draws the float weights again in the
reference's construction order (model_quant.py:1112-1131, 1438-1475,
1727-1747, 1918-1985) and applies the same float32 operations. The result
is checked against the full checkpoint's content digest stored in the
record.
"""
from __future__ import annotations

import json
import os
from typing import Dict, Tuple

import numpy as np

from .checkpoint import ModelDims, check_state_dict, state_digest

ASSETS = os.path.join(os.path.dirname(os.path.abspath(__file__)), "assets")

# the linear layers whose INT8 weights are rebuilt (all of them, in order)
_ATTN = ("query", "key", "value", "out")


def record_path(size: str) -> str:
    return os.path.join(ASSETS, f"calib_{size}_seed0.npz")


def rebuilt_keys(dims: ModelDims):
    """Keys of the INT8 state dict that the record leaves out: every linear
    weight of the blocks and the token embedding."""
    keys = []
    for side, n in (("encoder", dims.n_audio_layer), ("decoder", dims.n_text_layer)):
        for i in range(n):
            pre = f"{side}.blocks.{i}"
            mhas = [pre + ".attn"] + ([pre + ".cross_attn"] if side == "decoder" else [])
            keys += [f"{m}.{p}.weight" for m in mhas for p in _ATTN]
            keys += [pre + ".mlp.0.weight", pre + ".mlp.2.weight"]
    keys.append("decoder.token_embedding.weight")
    return keys


def make_record(dims: ModelDims, sd: Dict[str, np.ndarray], alphas: Dict[str, np.ndarray], path: str):
    """Write the compact record of a calibrated checkpoint: ``sd`` without
    the rebuilt weights, plus the quantiser's float32 ``wgt_alpha`` of each
    rebuilt weight (``alphas``, keyed like the weight's module)."""
    drop = set(rebuilt_keys(dims))
    out = {k: np.asarray(v) for k, v in sd.items() if k not in drop}
    for k in drop:
        mod = k[: -len(".weight")] if k != "decoder.token_embedding.weight" else "decoder"
        out["__alpha__." + mod] = np.asarray(alphas[mod], np.float32)
    out["__dims__"] = np.frombuffer(json.dumps(dims.__dict__).encode(), np.uint8)
    out["__digest__"] = np.frombuffer(state_digest(sd).encode(), np.uint8)
    np.savez_compressed(path, **out)


def rebuild(path: str) -> Tuple[ModelDims, Dict[str, np.ndarray]]:
    """(dims, INT8 state dict) of a calibrated checkpoint from its record;
    RuntimeError if the rebuilt content differs from the recorded digest."""
    import torch

    with np.load(path) as z:
        rec = {k: z[k] for k in z.files}
    dims = ModelDims(**json.loads(rec.pop("__dims__").tobytes().decode()))
    digest = rec.pop("__digest__").tobytes().decode()
    alpha = {k[len("__alpha__."):]: v for k, v in rec.items() if k.startswith("__alpha__.")}
    sd = {k: v for k, v in rec.items() if not k.startswith("__")}

    def q_linear(pre: str, n_in: int, n_out: int, bias: bool = True):
        # nn.Linear's own init (kaiming-uniform weight, then uniform bias)
        lin = torch.nn.Linear(n_in, n_out, bias=bias)
        w = lin.weight.detach()
        a = torch.from_numpy(alpha[pre]).reshape(n_out, 1)
        z = torch.from_numpy(sd[pre + ".wgt_zeros"]).unsqueeze(-1)
        sd[pre + ".weight"] = w.mul(a).add(z).round().clamp(min=-127, max=127).to(torch.int8).numpy()

    def block(pre: str, d: int, cross: bool):
        # ResidualAttentionBlock_quantized: attn (query, key, value, out),
        # attn_ln, [cross_attn (same), cross_attn_ln], mlp (fc1, GeLU, fc2),
        # mlp_ln; LayerNorm and GeLU draw no random numbers
        for mha in ([pre + ".attn"] + ([pre + ".cross_attn"] if cross else [])):
            for p in _ATTN:
                q_linear(f"{mha}.{p}", d, d, bias=(p != "key"))
        q_linear(pre + ".mlp.0", d, 4 * d)
        q_linear(pre + ".mlp.2", 4 * d, d)

    g = torch.random.get_rng_state()
    try:
        torch.manual_seed(0)
        with torch.no_grad():
            d, td = dims.n_audio_state, dims.n_text_state
            # AudioEncoder_quantized: conv1, conv2 (their INT8 weights are in
            # the record; constructed only to draw their random numbers), blocks
            torch.nn.Conv1d(dims.n_mels, d, kernel_size=3, padding=1)
            torch.nn.Conv1d(d, d, kernel_size=3, stride=2, padding=1)
            for i in range(dims.n_audio_layer):
                block(f"encoder.blocks.{i}", d, False)
            # TextDecoder_quantized: token embedding (normal init), blocks
            emb = torch.nn.Embedding(dims.n_vocab, td).weight.detach()
            a = torch.from_numpy(alpha["decoder"])
            sd["decoder.token_embedding.weight"] = emb.mul(a).round().clamp(min=-127, max=127).to(torch.int8).numpy()
            del emb
            for i in range(dims.n_text_layer):
                block(f"decoder.blocks.{i}", td, True)
    finally:
        torch.random.set_rng_state(g)
    check_state_dict(dims, sd)
    if state_digest(sd) != digest:
        raise RuntimeError(f"{path}: rebuilt checkpoint does not match its recorded digest")
    return dims, sd
