"""``i-whisper-int`` checkpoints: dimensions, the strict key contract, the
safetensors loader/saver, and a deterministic synthetic generator.

The on-disk format is the reference's (vcsd-lab/I-Whisper,
i_whisper/__init__.py:244-417): a directory ``iwhisper-<name>/`` holding
``config.json`` (``format == "i-whisper-int"``, ``format_version == 1``,
``dims``) and ``model.safetensors`` whose keys and integer dtypes are exactly
``Whisper_int.state_dict()`` (loaded with ``strict=True``).
"""
from __future__ import annotations

import json
import os
import zlib
from dataclasses import asdict, dataclass
from typing import Dict, Tuple

import numpy as np

FORMAT = "i-whisper-int"
FORMAT_VERSION = 1


@dataclass(frozen=True)
class ModelDims:
    """Field-for-field ``ModelDimensions`` (model_int.py:50-61)."""
    n_mels: int
    n_audio_ctx: int
    n_audio_state: int
    n_audio_head: int
    n_audio_layer: int
    n_vocab: int
    n_text_ctx: int
    n_text_state: int
    n_text_head: int
    n_text_layer: int


DIMS = {
    "tiny": ModelDims(80, 1500, 384, 6, 4, 51865, 448, 384, 6, 4),
    "base": ModelDims(80, 1500, 512, 8, 6, 51865, 448, 512, 8, 6),
    "small": ModelDims(80, 1500, 768, 12, 12, 51865, 448, 768, 12, 12),
    "medium": ModelDims(80, 1500, 1024, 16, 24, 51865, 448, 1024, 16, 24),
    "large": ModelDims(128, 1500, 1280, 20, 32, 51866, 448, 1280, 20, 32),
}


def _linear_keys(pre: str, n_in: int, n_out: int, bias: bool = True):
    k = {pre + ".weight": ((n_out, n_in), "int8")}
    if bias:
        k[pre + ".bias"] = ((n_out,), "int32")
    k[pre + ".req_multiplier"] = ((n_out,), "uint32")
    k[pre + ".req_shiftmount"] = ((n_out,), "int8")
    k[pre + ".wgt_zeros"] = ((n_out,), "int8")
    return k


def _ln_keys(pre: str, d: int):
    return {pre + ".weight": ((d,), "int8"), pre + ".bias": ((d,), "int32"),
            pre + ".ln_req_multiplier": ((1,), "uint8"), pre + ".ln_req_shiftmount": ((1,), "int8"),
            pre + ".out_req_multiplier": ((1,), "uint32"), pre + ".out_req_shiftmount": ((1,), "int8")}


def _gelu_keys(pre: str, n_in: int, n_out: int):
    return {pre + ".lut": ((16,), "uint8"), pre + ".luti_req_multiplier": ((n_in,), "uint8"),
            pre + ".luti_req_shiftmount": ((n_in,), "int8"), pre + ".luto_req_multiplier": ((n_out,), "uint8"),
            pre + ".luto_req_shiftmount": ((n_out,), "int8"), pre + ".de_smooth_vec": ((n_in,), "uint8")}


def _mha_keys(pre: str, d: int):
    k = {pre + ".qk_req_multiplier": ((1,), "uint8"), pre + ".qk_req_shiftmount": ((1,), "int8"),
         pre + ".av_req_multiplier": ((1,), "uint8"), pre + ".av_req_shiftmount": ((1,), "int8"),
         pre + ".qk_frac_bits": ((), "int32")}
    k.update(_linear_keys(pre + ".query", d, d))
    k.update(_linear_keys(pre + ".key", d, d, bias=False))
    k.update(_linear_keys(pre + ".value", d, d))
    k.update(_linear_keys(pre + ".out", d, d))
    return k


def _block_keys(pre: str, d: int):
    k = {pre + ".attn_res_req_multiplier": ((1,), "uint16"), pre + ".cross_attn_res_req_multiplier": ((1,), "uint16"),
         pre + ".mlp_res_req_multiplier": ((1,), "uint16")}
    k.update(_mha_keys(pre + ".attn", d))
    k.update(_ln_keys(pre + ".attn_ln", d))
    k.update(_linear_keys(pre + ".mlp.0", d, 4 * d))
    k.update(_gelu_keys(pre + ".mlp.1", 4 * d, 4 * d))
    k.update(_linear_keys(pre + ".mlp.2", 4 * d, d))
    k.update(_ln_keys(pre + ".mlp_ln", d))
    return k


def expected_keys(dims: ModelDims) -> Dict[str, Tuple[tuple, str]]:
    """Key -> (shape, dtype) of ``Whisper_int(dims).state_dict()``
    (model_int.py:66-1553; module order as registered)."""
    d, td = dims.n_audio_state, dims.n_text_state
    k = {"encoder.req_multiplier": ((d,), "uint16"), "encoder.req_shiftmount": ((d,), "int8"),
         "encoder.input_alpha": ((1,), "float32"), "encoder.positional_embedding": ((dims.n_audio_ctx, d), "int8")}
    k.update(_gelu_keys("encoder.gelu1", 1, 1))
    k.update(_gelu_keys("encoder.gelu2", 1, d))
    k.update({"encoder.conv1.weight": ((d, dims.n_mels * 3), "int8"), "encoder.conv1.bias": ((d,), "int32"),
              "encoder.conv1.req_multiplier": ((1,), "uint32"), "encoder.conv1.req_shiftmount": ((1,), "int8"),
              "encoder.conv2.weight": ((d, d * 3), "int8"), "encoder.conv2.bias": ((d,), "int32"),
              "encoder.conv2.req_multiplier": ((1,), "uint32"), "encoder.conv2.req_shiftmount": ((1,), "int8")})
    for i in range(dims.n_audio_layer):
        k.update(_block_keys(f"encoder.blocks.{i}", d))
    k.update(_ln_keys("encoder.ln_post", d))
    k.update({"decoder.req_multiplier": ((1,), "uint8"), "decoder.req_shiftmount": ((1,), "int8"),
              "decoder.clf_req_multiplier": ((1,), "uint32"), "decoder.clf_req_shiftmount": ((1,), "int8"),
              "decoder.act_logits_alpha": ((1,), "float32"),
              "decoder.positional_embedding": ((dims.n_text_ctx, td), "int8"),
              "decoder.token_embedding.weight": ((dims.n_vocab, td), "int8")})
    for i in range(dims.n_text_layer):
        pre = f"decoder.blocks.{i}"
        k.update(_block_keys(pre, td))
        k.update(_mha_keys(pre + ".cross_attn", td))
        k.update(_ln_keys(pre + ".cross_attn_ln", td))
    k.update(_ln_keys("decoder.ln", td))
    return k


# ---------------------------------------------------------------------------
# Loading / saving (i_whisper/__init__.py:244-417)
# ---------------------------------------------------------------------------
def resolve_dir(name: str, root: str = "CKPT") -> str:
    if os.path.isdir(name):
        return name
    if os.path.isfile(name):
        if os.path.basename(name) != "model.safetensors":
            raise RuntimeError(f"Expected model.safetensors, got: {name}")
        return os.path.dirname(name)
    d = os.path.join(root, f"iwhisper-{name}")
    if os.path.isdir(d):
        return d
    raise RuntimeError(f"I-Whisper INT model '{name}' not found. Expected directory: {d}")


def load_int_checkpoint(name: str, root: str = "CKPT"):
    """Returns (ModelDims, {key: numpy array}) after the reference's format
    checks and a strict key/dtype/shape check."""
    from safetensors.numpy import load_file
    d = resolve_dir(name, root)
    cfg_p, ten_p = os.path.join(d, "config.json"), os.path.join(d, "model.safetensors")
    if not os.path.isfile(cfg_p):
        raise RuntimeError(f"Missing model configuration: {cfg_p}")
    if not os.path.isfile(ten_p):
        raise RuntimeError(f"Missing model tensors: {ten_p}")
    cfg = json.load(open(cfg_p, encoding="utf-8"))
    if cfg.get("format") != FORMAT:
        raise RuntimeError(f"Unsupported model format: {cfg.get('format')}")
    if cfg.get("format_version") != FORMAT_VERSION:
        raise RuntimeError(f"Unsupported model format version: {cfg.get('format_version')}")
    dims = ModelDims(**cfg["dims"])
    sd = load_file(ten_p)
    check_state_dict(dims, sd)
    return dims, sd


def check_state_dict(dims: ModelDims, sd: Dict[str, np.ndarray]):
    """``load_state_dict(strict=True)`` semantics: same key set, and each
    tensor with the expected shape and integer dtype."""
    exp = expected_keys(dims)
    missing = sorted(set(exp) - set(sd))
    unexpected = sorted(set(sd) - set(exp))
    if missing or unexpected:
        raise RuntimeError(f"Error(s) in loading state_dict: missing keys {missing[:8]}..., unexpected {unexpected[:8]}...")
    for k, (shape, dt) in exp.items():
        a = np.asarray(sd[k])
        if tuple(a.shape) != tuple(shape) or a.dtype != np.dtype(dt):
            raise RuntimeError(f"{k}: expected {dt}{list(shape)}, got {a.dtype}{list(a.shape)}")


def save_int_checkpoint(dims: ModelDims, sd: Dict[str, np.ndarray], prefix: str, model_name: str) -> str:
    """``save_int_model`` (i_whisper/__init__.py:281-335)."""
    from safetensors.numpy import save_file
    d = os.path.join(prefix, f"iwhisper-{model_name}")
    os.makedirs(d, exist_ok=True)
    # np.require keeps 0-d tensors (qk_frac_bits) 0-d; ascontiguousarray would make them [1]
    save_file({k: np.require(v, requirements="C") for k, v in sd.items()}, os.path.join(d, "model.safetensors"),
              metadata={"format": FORMAT, "format_version": str(FORMAT_VERSION)})
    with open(os.path.join(d, "config.json"), "w", encoding="utf-8") as f:
        json.dump({"format": FORMAT, "format_version": FORMAT_VERSION, "model_name": model_name,
                   "dims": asdict(dims)}, f, indent=2)
    return d


def state_digest(sd: Dict[str, np.ndarray]) -> str:
    """sha256 over every tensor (sorted keys; name, dtype, shape and bytes):
    identifies a checkpoint's content independently of file layout."""
    import hashlib
    h = hashlib.sha256()
    for k in sorted(sd):
        a = np.asarray(sd[k])
        h.update(k.encode())
        h.update(str(a.dtype).encode())
        h.update(str(tuple(a.shape)).encode())
        h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()


# ---------------------------------------------------------------------------
# Reference-calibrated checkpoints (random-init float weights from seed 0,
# calibrated and quantised by the reference's own quantiser on 8 synthetic
# windows; generated by tests/golden/make_calibrated.py)
# ---------------------------------------------------------------------------
def ckpt_root() -> str:
    """Checkpoint directory: $IWHISPER_CKPT, else CKPT/ in the repository."""
    return os.environ.get("IWHISPER_CKPT") or os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))),
                                                           "CKPT")


def calibrated_name(size: str) -> str:
    return f"{size}-calib-seed0"


def calibrated_path(size: str) -> str:
    return os.path.join(ckpt_root(), f"iwhisper-{calibrated_name(size)}")


def load_calibrated(size: str):
    """(dims, state dict) of the reference-calibrated ``size`` checkpoint:
    the full checkpoint when it is present, else rebuilt from its compact
    record (calibrated.rebuild); FileNotFoundError when neither exists."""
    p = calibrated_path(size)
    if os.path.isfile(os.path.join(p, "model.safetensors")):
        return load_int_checkpoint(p)
    from .calibrated import rebuild, record_path
    if os.path.isfile(record_path(size)):
        return rebuild(record_path(size))
    raise FileNotFoundError(f"{p}: run tests/golden/make_calibrated.py --sizes {size}")


# ---------------------------------------------------------------------------
# Deterministic synthetic checkpoint
# ---------------------------------------------------------------------------
def _rng(seed: int, key: str) -> np.random.Generator:
    return np.random.default_rng([seed, zlib.crc32(key.encode())])


def _frexp_u32(scale: np.ndarray, shift_rule: str = "down"):
    """Multiplier/shift pair the way model_quant.py:626-648 derives them with
    torch.frexp: m = trunc(mantissa * 2^31), s = clamp(-exp-1, 0, 32)."""
    mant, exp = np.frexp(np.asarray(scale, np.float64))
    m = np.trunc(mant * 2.0 ** 31).astype(np.uint64).astype(np.uint32)
    s = np.clip(-exp - 1, 0, 32).astype(np.int8)
    return m, s


def synthetic_state_dict(dims: ModelDims, seed: int = 0) -> Dict[str, np.ndarray]:
    """A complete, valid ``Whisper_int`` state dict with random INT8 weights
    and requantisation parameters chosen so that activations stay inside
    their integer ranges (int8 activations of standard deviation ~30, INT15
    residual stream ~1500). Deterministic in (dims, seed) on any machine:
    every tensor has its own generator seeded by (seed, crc32(key))."""
    sd: Dict[str, np.ndarray] = {}
    act = 30.0

    def weights(key, shape, std=40.0):
        # uniform integers in [-h, h] with standard deviation ~std
        h = int(round(np.sqrt(3.0) * std))
        sd[key] = _rng(seed, key).integers(-h, h + 1, shape, dtype=np.int8)

    def linear8(pre, n_in, n_out, bias=True, out_std=act):
        weights(pre + ".weight", (n_out, n_in))
        r = _rng(seed, pre + ".q")
        acc_std = np.sqrt(n_in) * act * 40.0
        m, s = _frexp_u32(out_std / acc_std * r.uniform(0.8, 1.25, n_out))
        if bias:
            sd[pre + ".bias"] = np.rint(r.normal(0, 0.2 * acc_std, n_out)).astype(np.int32)
        sd[pre + ".req_multiplier"], sd[pre + ".req_shiftmount"] = m, s
        sd[pre + ".wgt_zeros"] = r.integers(-4, 5, n_out).astype(np.int8)

    def linear32(pre, n_in, n_out, res_std=700.0):
        # branch in residual units * 2^15: br = mulh(acc, m) << s
        weights(pre + ".weight", (n_out, n_in))
        r = _rng(seed, pre + ".q")
        acc_std = np.sqrt(n_in) * act * 40.0
        scale = res_std * 2.0 ** 15 / acc_std * r.uniform(0.8, 1.25, n_out)
        mant, exp = np.frexp(scale)
        sd[pre + ".weight"] = sd[pre + ".weight"]
        sd[pre + ".bias"] = np.rint(r.normal(0, 0.2 * acc_std, n_out)).astype(np.int32)
        sd[pre + ".req_multiplier"] = np.trunc(mant * 2.0 ** 32).astype(np.uint64).clip(0, 2 ** 32 - 1).astype(np.uint32)
        sd[pre + ".req_shiftmount"] = np.clip(exp, 0, 32).astype(np.int8)
        sd[pre + ".wgt_zeros"] = r.integers(-4, 5, n_out).astype(np.int8)

    def layernorm(pre, d):
        r = _rng(seed, pre)
        sd[pre + ".weight"] = r.integers(40, 91, d).astype(np.int8)
        sd[pre + ".bias"] = np.rint(r.normal(0, 20000, d)).astype(np.int32)
        sd[pre + ".ln_req_multiplier"] = np.array([128], np.uint8)
        sd[pre + ".ln_req_shiftmount"] = np.array([9], np.int8)
        m, s = _frexp_u32(np.array([act / (2048.0 * 65.0)]))
        sd[pre + ".out_req_multiplier"], sd[pre + ".out_req_shiftmount"] = m, s

    def gelu(pre, n_in, n_out):
        r = _rng(seed, pre)
        t = (np.arange(16) - 8) * 16.0 / act
        sd[pre + ".lut"] = np.rint(255.0 / (1.0 + np.exp(-1.702 * t))).astype(np.uint8)
        sd[pre + ".luti_req_multiplier"] = np.ones(n_in, np.uint8)
        sd[pre + ".luti_req_shiftmount"] = np.full(n_in, 4, np.int8)
        sd[pre + ".luto_req_multiplier"] = r.integers(150, 220, n_out).astype(np.uint8)
        sd[pre + ".luto_req_shiftmount"] = np.full(n_out, 15, np.int8)
        sd[pre + ".de_smooth_vec"] = np.ones(n_in, np.uint8)

    def mha(pre, d):
        sd[pre + ".qk_req_multiplier"] = np.array([182], np.uint8)
        sd[pre + ".qk_req_shiftmount"] = np.array([12], np.int8)
        sd[pre + ".av_req_multiplier"] = np.array([192], np.uint8)
        sd[pre + ".av_req_shiftmount"] = np.array([7], np.int8)
        sd[pre + ".qk_frac_bits"] = np.array(7, np.int32)
        linear8(pre + ".query", d, d)
        linear8(pre + ".key", d, d, bias=False)
        linear8(pre + ".value", d, d)
        linear32(pre + ".out", d, d)

    def block(pre, d, cross):
        sd[pre + ".attn_res_req_multiplier"] = np.array([31130], np.uint16)
        sd[pre + ".cross_attn_res_req_multiplier"] = np.array([31130], np.uint16)
        sd[pre + ".mlp_res_req_multiplier"] = np.array([31130], np.uint16)
        mha(pre + ".attn", d)
        layernorm(pre + ".attn_ln", d)
        if cross:
            mha(pre + ".cross_attn", d)
            layernorm(pre + ".cross_attn_ln", d)
        linear8(pre + ".mlp.0", d, 4 * d)
        gelu(pre + ".mlp.1", 4 * d, 4 * d)
        linear32(pre + ".mlp.2", 4 * d, d)
        layernorm(pre + ".mlp_ln", d)

    d, td = dims.n_audio_state, dims.n_text_state
    r = _rng(seed, "encoder")
    sd["encoder.req_multiplier"] = r.integers(8000, 11000, d).astype(np.uint16)
    sd["encoder.req_shiftmount"] = np.full(d, 8, np.int8)
    sd["encoder.input_alpha"] = np.array([100.0], np.float32)
    weights("encoder.positional_embedding", (dims.n_audio_ctx, d), std=act)
    gelu("encoder.gelu1", 1, 1)
    gelu("encoder.gelu2", 1, d)
    for name, cin in (("conv1", dims.n_mels), ("conv2", d)):
        pre = "encoder." + name
        weights(pre + ".weight", (d, cin * 3))
        acc_std = np.sqrt(cin * 3) * act * 40.0
        rr = _rng(seed, pre + ".q")
        sd[pre + ".bias"] = np.rint(rr.normal(0, 0.2 * acc_std, d)).astype(np.int32)
        m, s = _frexp_u32(np.array([act / acc_std]))
        sd[pre + ".req_multiplier"], sd[pre + ".req_shiftmount"] = m, s
    for i in range(dims.n_audio_layer):
        block(f"encoder.blocks.{i}", d, False)
    layernorm("encoder.ln_post", d)
    sd["decoder.req_multiplier"] = np.array([148], np.uint8)
    sd["decoder.req_shiftmount"] = np.array([2], np.int8)
    acc_std = np.sqrt(td) * act * 40.0
    m, s = _frexp_u32(np.array([25.0 / acc_std]))
    sd["decoder.clf_req_multiplier"], sd["decoder.clf_req_shiftmount"] = m, s
    sd["decoder.act_logits_alpha"] = np.array([5.0], np.float32)
    weights("decoder.positional_embedding", (dims.n_text_ctx, td), std=act)
    weights("decoder.token_embedding.weight", (dims.n_vocab, td))
    for i in range(dims.n_text_layer):
        block(f"decoder.blocks.{i}", td, True)
    layernorm("decoder.ln", td)
    check_state_dict(dims, sd)
    return sd
