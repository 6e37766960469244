"""Generate the model-level golden fixtures from the REFERENCE itself.

Runs vcsd-lab/I-Whisper's own ``Whisper_int`` module graph
(i_whisper/model_int.py) and its own greedy decoding loop
(i_whisper/decoding.py, DecodingTask._main_loop) with every module on the
``scalar`` backend, where ``_C.<op>_scalar`` is served by the reference's
own scalar C++ kernels compiled into oracle/_ref/libiw_ref.so (the
pybind layer is replaced by a numpy bridge; bitsandbytes, matplotlib and
librosa, which the CPU path never calls, are stubbed). The checkpoint is
``i_whisper_b200.checkpoint.synthetic_state_dict`` (deterministic), loaded
into the reference model with ``load_state_dict(strict=True)``; the input is
the deterministic synthetic INT8 mel. The same run is repeated with every
module on the ``torch`` golden backend as a cross-check.

Writes tests/golden/model_golden.json and, for the LayerNorm64 research
variant, model_golden_ln64.json (digests of the encoder output and
of each block's INT15 stream, plus the greedy token ids). Needs the
reference checkout and oracle/_ref (``make -C oracle ref``).

Usage: python tests/golden/make_golden.py [REFERENCE_ROOT]
(default: $IWHISPER_REFERENCE, else a checkout named ``reference`` next to
this repository)
"""
import hashlib
import json
import os
import sys
import types

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)
sys.path.insert(0, HERE)
from refroot import reference_root  # noqa: E402

REF = None  # resolved on first use: argv[1], $IWHISPER_REFERENCE or ../reference

from oracle import oracle as O  # noqa: E402
from i_whisper_b200.checkpoint import ModelDims, synthetic_state_dict  # noqa: E402
from i_whisper_b200.synthetic import synthetic_mel_batch  # noqa: E402

GOLDEN_CASES = {
    # reduced-depth model with the full audio context and vocabulary
    "mini": dict(dims=ModelDims(80, 1500, 384, 6, 2, 51865, 448, 384, 6, 2), seed=0, mel_seeds=[1], sample_len=24),
    # large's widths: 128 mel bins, d = 1280 (20 heads), the 51866-token vocabulary; one layer each side
    "large1": dict(dims=ModelDims(128, 1500, 1280, 20, 1, 51866, 448, 1280, 20, 1), seed=6, mel_seeds=[9],
                   sample_len=6),
}

# the LayerNorm64 research variant (set_layernorm_backend "scalar64" / "torch64"),
# kept in its own file: model_golden_ln64.json
GOLDEN_CASES_LN64 = {
    "mini_ln64": dict(dims=ModelDims(80, 1500, 384, 6, 2, 51865, 448, 384, 6, 2), seed=0, mel_seeds=[1],
                      sample_len=24, layernorm="64"),
}


def sha(a) -> str:
    a = a.numpy() if isinstance(a, torch.Tensor) else np.asarray(a)
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def _bridge_C():
    """_C.<op>_scalar with the reference scalar kernels (oracle/_ref)."""
    R = O.lib("ref")
    n = lambda t: None if t is None else t.contiguous().numpy()
    t = torch.from_numpy
    C = types.ModuleType("_C")
    C.linear8_scalar = lambda x, w, b, z, m, s: t(R.linear8(n(x), n(w), n(b), n(z), n(m), n(s)))
    C.linear32_scalar = lambda x, w, b, z, m, s: t(R.linear32(n(x), n(w), n(b), n(z), n(m), n(s)))
    C.residual15_scalar = lambda br, r, m: t(R.residual15(n(br), n(r), n(m)))
    C.layernorm32_scalar = lambda x, g, b, lm, ls, om, os_: t(R.layernorm32(n(x), n(g), n(b), n(lm), n(ls), n(om), n(os_)))
    C.layernorm64_scalar = lambda x, g, b, lm, ls, om, os_: t(R.layernorm64(n(x), n(g), n(b), n(lm), n(ls), n(om), n(os_)))
    C.gelu_scalar = lambda x, lut, mi, si, mo, so: t(R.gelu(n(x), n(lut), n(mi), n(si), n(mo), n(so)))

    def qk(q, k, mask, m, s):
        a, b = R.qk_requant_rowmax(n(q), n(k), None if mask is None else n(mask).astype(np.uint8), n(m), n(s))
        return t(a), t(b)

    def se(x, rm, mask, fb):
        a, b = R.shift_exp(n(x), n(rm), None if mask is None else n(mask).astype(np.uint8), n(fb))
        return t(a), t(b)

    C.qk_requant_rowmax_scalar = qk
    C.shift_exp_scalar = se
    C.pv_norm_requant_scalar = lambda p, v, rs, am, as_, off: t(R.pv_norm_requant(n(p), n(v), n(rs), n(am), n(as_), off))
    C.conv1d_scalar = lambda x, w, b, m, s, st, pad: t(R.conv1d(n(x), n(w), n(b), n(m), n(s), st, pad))
    C.add_requant15_scalar = lambda x, a, m, s: t(R.add_requant15(n(x), n(a), n(m), n(s)))
    C.classifier_scalar = lambda x, w, m, s: t(R.classifier(n(x), n(w), n(m), n(s)))
    return C


def import_reference(ref: str = None, bridge=None):
    """Import the reference's model_int, modules.linear and decoding with
    ``_C`` served by ``bridge()`` (default: the reference scalar kernels)."""
    ref = ref or REF or reference_root(sys.argv[1] if __name__ == "__main__" and len(sys.argv) > 1 else None)
    for name in ("bitsandbytes", "bitsandbytes.functional", "matplotlib", "matplotlib.pyplot", "librosa"):
        sys.modules.setdefault(name, types.ModuleType(name))
    sys.modules["bitsandbytes"].functional = sys.modules["bitsandbytes.functional"]
    sys.modules["bitsandbytes.functional"].int8_linear_matmul = None
    sys.modules["matplotlib"].pyplot = sys.modules["matplotlib.pyplot"]
    kern = types.ModuleType("i_whisper.kernels")
    kern._C = (bridge or _bridge_C)()
    sys.modules["i_whisper.kernels"] = kern
    sys.modules["i_whisper.kernels._C"] = kern._C
    sys.path.insert(0, ref)
    import i_whisper.model_int as MI
    import i_whisper.modules.linear as ML
    import i_whisper.decoding as DEC
    return MI, ML, DEC


def run_reference(MI, ML, DEC, case, backend, sd=None):
    """The reference's Whisper_int encoder (with per-block digests) and its
    DecodingTask greedy loop on ``backend``; ``sd`` defaults to the synthetic
    checkpoint of ``case["seed"]``."""
    dims = case["dims"]
    model = MI.Whisper_int(MI.ModelDimensions(**dims.__dict__))
    if sd is None:
        sd = synthetic_state_dict(dims, case["seed"])
    missing, unexpected = model.load_state_dict({k: torch.from_numpy(np.ascontiguousarray(v)) for k, v in sd.items()},
                                                strict=True)
    assert not missing and not unexpected
    quiet = type("L", (), {"debug": staticmethod(lambda *a, **k: None)})()
    for fn in (MI.set_residual_backend, MI.set_layernorm_backend, MI.set_gelu_backend, MI.set_attention_backend,
               MI.set_conv1d_backend, MI.set_audio_encoder_backend, MI.set_text_decoder_backend,
               ML.set_linear8_backend, ML.set_linear32_backend):
        fn(model, backend, logger=quiet)
    if case.get("layernorm") == "64":
        MI.set_layernorm_backend(model, backend + "64", logger=quiet)
    model.eval()
    mel = torch.from_numpy(synthetic_mel_batch(dims.n_mels, case["mel_seeds"], float(sd["encoder.input_alpha"][0])))
    blocks = {}
    hooks = [blk.register_forward_hook(lambda m, i, o, k=k: blocks.__setitem__(k, o.clone()))
             for k, blk in enumerate(model.encoder.blocks)]
    with torch.no_grad():
        xa = model.encoder(mel)
        for h in hooks:
            h.remove()
        opts = DEC.DecodingOptions(fp16=False, language="en", sample_len=case["sample_len"])
        task = DEC.DecodingTask(model, opts)
        tokens = torch.tensor([task.initial_tokens]).repeat(mel.shape[0], 1)
        tokens, _, _ = task._main_loop(xa, tokens)
    return dict(mel_sha256=sha(mel), encoder_sha256=sha(xa),
                block_sha256=[sha(blocks[k]) for k in sorted(blocks)], tokens=tokens.tolist())


def main():
    MI, ML, DEC = import_reference()
    for cases, fname in ((GOLDEN_CASES, "model_golden.json"), (GOLDEN_CASES_LN64, "model_golden_ln64.json")):
        out = {}
        for name, case in cases.items():
            res = run_reference(MI, ML, DEC, case, "scalar")
            res_t = run_reference(MI, ML, DEC, case, "torch")
            assert res == res_t, "reference scalar and torch backends disagree"
            out[name] = dict(dims=case["dims"].__dict__, seed=case["seed"], mel_seeds=case["mel_seeds"],
                             sample_len=case["sample_len"], **res)
            if case.get("layernorm"):
                out[name]["layernorm"] = case["layernorm"]
            print(name, res["encoder_sha256"][:16], res["tokens"])
        with open(os.path.join(HERE, fname), "w") as f:
            json.dump(out, f, indent=1)


if __name__ == "__main__":
    main()
