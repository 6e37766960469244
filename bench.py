"""Benchmark of the B200 integer Whisper path (the repository's bench contract).

Workload (per GPU): whisper-medium integer encoder
over a batch of 256 synthetic 30 s windows (d_model 1024, 24 layers, 16
heads, 80 mels), then greedy decoding of 128 tokens per window with an INT8
self-attention KV cache and INT8 cross-attention over the 1500 encoder
states. Weights are the reference-calibrated checkpoint the configuration
names (random-init from seed 0, calibrated and quantised by the reference's
own quantiser on 8 synthetic windows: CKPT/iwhisper-medium-calib-seed0, made
by tests/golden/make_calibrated.py; the deterministic synthetic checkpoint
when it is absent, which the line then says); inputs are seeded sine+noise
windows through the float log-mel frontend (seeds recycled modulo 32).

* ``parity``: outside the timed region, windows 0 and 1 of every rank's
  batch (seeds 0 and 1) are compared with the committed golden digests of
  the oracle (encoder output and the first 8 greedy tokens).

* ``value``: encoder windows/s of the whole job (all ranks), inputs resident
  in HBM; one step = one encoder pass over the batch, replayed from a CUDA
  graph captured once for the batch (``WhisperIntB200.encoder_graphed``).
  Steps whose working set exceeds L2 run back to back; a smaller one (tiny,
  one window) is timed one step at a time after a write that flushes L2.
* ``e2e``: the same metric through the public API with host buffers
  (``WhisperIntB200.encode_batches``): each step copies its INT8 mel batch
  from pinned host memory, runs the encoder and reads the INT8 features back
  to pinned host memory; uploads and downloads run on their own streams,
  overlapping the neighbouring steps' compute.
* ``decoder``: greedy decoding tok/s (device-resident and end to end with
  the token matrix read back).
* ``roofline``: the dominant kernel, achieved work per launch from a CUDA
  event pair around every launch of a second pass over the same steps (the
  headline pass records no per-launch events: small configurations are
  bound by the host's launch rate), against the dense INT8 tensor peak taken as
  2 x the measured dense BF16 peak (MEASURED_PEAKS.json; INT8 runs at twice
  the BF16 rate on B200), with the datasheet 4500 TOPS and an in-run
  torch._int_mm probe reported beside it.
* ``cpu_baseline``: the reference's own scalar C++ kernels (oracle/_ref) on a
  bounded sample of the same workload on the host cores (rank 0, N=1).

``--config N`` selects another BASELINE configuration (default 3, the line
above): 0 whisper-tiny, the seed-1 window, encoder + 32 greedy tokens; 1 the
kernel microbench (w8a8 GEMM at M = 1500*{1,8,32} for four (K, N), integer
LayerNorm over 1500 x 1024, 16-head 1500 x 1500 attention), each kernel
timed per launch with an L2 flush in between; 2 whisper-small encoder, 32
windows; 4 whisper-large encoder + 224 greedy tokens, 64 windows per GPU
(512 over 8 GPUs).

Multi-GPU: one process per GPU (torchrun); utterances are sharded by
rank with no collective on the data path; ``scaling`` is weak (each rank
owns a fixed batch). ``--impl reference`` times the reference CPU path
instead (rank 0 only).
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "int8 encoder 30s-windows/sec (whisper-medium) + % int8 TC peak; decoder tok/s"

# model, windows per GPU, greedy tokens, window seeds
CONFIGS = {
    0: dict(model="tiny", batch=1, decode_tokens=32, seeds=[1],
            workload="whisper-tiny integer encoder + 32 greedy tokens, batch 1, the seed-1 window (BASELINE configs[0])"),
    1: dict(model="medium", batch=0, decode_tokens=0, seeds=None,
            workload="kernel microbench (BASELINE configs[1]): w8a8 GEMM M=1500*{1,8,32} x (K,N) in "
                     "{(1024,1024),(1024,4096),(4096,1024),(1280,5120)}, LayerNorm32 1500x1024, "
                     "attention 16 heads x 1500^2 x 64"),
    2: dict(model="small", batch=32, decode_tokens=0, seeds=None,
            workload="whisper-small integer encoder, 32 windows per GPU (BASELINE configs[2])"),
    3: dict(model="medium", batch=256, decode_tokens=128, seeds=None,
            workload="whisper-medium integer encoder, {batch} windows per GPU (BASELINE configs[3]); "
                     "greedy decoder {tokens} tokens"),
    4: dict(model="large", batch=64, decode_tokens=224, seeds=None,
            workload="whisper-large integer encoder, {batch} windows per GPU (512 over 8 GPUs, BASELINE "
                     "configs[4]); greedy decoder {tokens} tokens"),
}


def metric_of(model: str) -> str:
    return f"int8 encoder 30s-windows/sec (whisper-{model}) + % int8 TC peak; decoder tok/s"


DATASHEET_INT8_TOPS = 4500.0
ENC_GOP = {"tiny": 36.9, "small": 344.2, "medium": 1138.1, "large": 2273.8}


def enc_gop(d):
    """Algorithmic encoder work per window (QK^T counted once):
    L*(24*T*d^2 + 4*T^2*d) + 2*(3000*3*n_mels*d + 1500*3*d^2), in GOP."""
    T = d.n_audio_ctx
    L, dm, nm = d.n_audio_layer, d.n_audio_state, d.n_mels
    return (L * (24 * T * dm * dm + 4 * T * T * dm) + 2 * (2 * T * 3 * nm * dm + T * 3 * dm * dm)) / 1e9


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--config", type=int, default=3, choices=sorted(CONFIGS),
                    help="BASELINE.json configuration (default 3: whisper-medium, 256 windows, 128 tokens)")
    ap.add_argument("--model", default=None, help="override the configuration's model")
    ap.add_argument("--batch", type=int, default=None, help="windows per GPU (override)")
    ap.add_argument("--decode-tokens", type=int, default=None, help="greedy tokens (override)")
    ap.add_argument("--decode-runs", type=int, default=1)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-rows", type=int, default=64, help="query rows of the CPU sample")
    ap.add_argument("--phase", default="all", choices=["all", "encoder", "decoder"],
                    help="restrict the run (for profiling): encoder only, or decoder only")
    a = ap.parse_args()
    cfg = CONFIGS[a.config]
    a.model = a.model or cfg["model"]
    a.batch = cfg["batch"] if a.batch is None else a.batch
    a.decode_tokens = cfg["decode_tokens"] if a.decode_tokens is None else a.decode_tokens
    a.seeds = cfg["seeds"]
    return a


# ---------------------------------------------------------------------------
# CPU reference timing (bounded samples of the same workload)
# ---------------------------------------------------------------------------
def _cpu_sample_worker(args):
    """One process: time one medium encoder layer + stem on `rows` of the
    1500 positions, and one decoder step (1 layer + classifier), with the
    chosen kernel library; returns seconds."""
    kind, rows, seed, model = args
    from oracle import oracle as O
    from i_whisper_b200.checkpoint import DIMS
    L = O.lib(kind)
    if kind == "port":
        L.set_threads(1)
    dims = DIMS[model]
    d, H, T = dims.n_audio_state, dims.n_audio_head, dims.n_audio_ctx
    rng = np.random.default_rng(seed)
    i8 = lambda *s: rng.integers(-60, 61, s, dtype=np.int8)
    lin = lambda n_in, n_out: (i8(n_out, n_in), rng.integers(-1000, 1000, n_out, dtype=np.int32),
                               rng.integers(-4, 5, n_out).astype(np.int8),
                               rng.integers(2 ** 30, 2 ** 31, n_out, dtype=np.uint32),
                               np.full(n_out, 12, np.int8))
    wq, wk, wv, wo, w1, w2 = lin(d, d), lin(d, d), lin(d, d), lin(d, d), lin(d, 4 * d), lin(4 * d, d)
    x16 = rng.integers(-3000, 3000, (rows, d), dtype=np.int16)
    g = rng.integers(40, 90, d, dtype=np.int8)
    be = rng.integers(-1000, 1000, d, dtype=np.int32)
    kfull = i8(1, H, T, 64)
    vtfull = i8(1, H, 64, T)
    lut = np.arange(16, dtype=np.uint8) * 16
    mi, si = np.ones(4 * d, np.uint8), np.full(4 * d, 4, np.int8)
    mo, so = np.full(4 * d, 128, np.uint8), np.full(4 * d, 15, np.int8)
    mel = i8(1, dims.n_mels, 2 * rows + 2)
    wc1, wc2 = i8(d, dims.n_mels * 3), i8(d, 3 * d)

    def layer():
        h = L.layernorm32(x16, g, be, 128, 9, 2 ** 30, 10)
        q = L.linear8(h, *wq); L.linear8(h, *wk); L.linear8(h, *wv)
        q4 = np.ascontiguousarray(q.reshape(1, rows, H, 64).transpose(0, 2, 1, 3))
        s, rm = L.qk_requant_rowmax(q4, kfull, None, 182, 12)
        p, rs = L.shift_exp(s, rm, None, 7)
        a = L.pv_norm_requant(p, vtfull, rs, 192, 7, 16).reshape(rows, d)
        x = L.residual15(L.linear32(a, *wo), x16, 31130)
        h = L.layernorm32(x, g, be, 128, 9, 2 ** 30, 10)
        f = L.gelu(L.linear8(h, *w1), lut, mi, si, mo, so)
        L.residual15(L.linear32(f, *w2), x, 31130)

    def stem():
        y = L.conv1d(mel, wc1, None, 2 ** 30, 10, 1, 1)
        L.conv1d(y, wc2, None, 2 ** 30, 10, 2, 1)

    t0 = time.perf_counter(); layer(); t_layer = time.perf_counter() - t0
    t0 = time.perf_counter(); stem(); t_stem = time.perf_counter() - t0
    # one decoder step of one utterance: 1 layer (self Tk 67, cross Tk 1500) + classifier
    x1 = x16[:1]
    ks, vts = i8(1, H, 67, 64), i8(1, H, 64, 67)
    emb = i8(dims.n_vocab, d)

    def dec_layer():
        h = L.layernorm32(x1, g, be, 128, 9, 2 ** 30, 10)
        q = L.linear8(h, *wq); L.linear8(h, *wk); L.linear8(h, *wv)
        q4 = np.ascontiguousarray(q.reshape(1, 1, H, 64).transpose(0, 2, 1, 3))
        for kk, vv in ((ks, vts), (kfull, vtfull)):
            s, rm = L.qk_requant_rowmax(q4, kk, None, 182, 12)
            p, rs = L.shift_exp(s, rm, None, 7)
            a = L.pv_norm_requant(p, vv, rs, 192, 7, 16).reshape(1, d)
            x = L.residual15(L.linear32(a, *wo), x1, 31130)
            L.linear8(L.layernorm32(x, g, be, 128, 9, 2 ** 30, 10), *wq)
        f = L.gelu(L.linear8(h, *w1), lut, mi, si, mo, so)
        L.residual15(L.linear32(f, *w2), x, 31130)

    t0 = time.perf_counter(); dec_layer(); t_dec_layer = time.perf_counter() - t0
    t0 = time.perf_counter(); L.classifier(L.layernorm32(x1, g, be, 128, 9, 2 ** 30, 10), emb, 2 ** 30, 10)
    t_clf = time.perf_counter() - t0
    return t_layer, t_stem, t_dec_layer, t_clf


def cpu_baseline(model: str, rows: int, procs: int):
    """Reference CPU throughput from bounded samples: `procs` single-threaded
    processes (spawned) each time one sampled encoder layer + stem and one
    decoder step; per-window time = 24 layers x (1500/rows) x layer sample +
    stem scaled the same way. Returns (windows/s, tok/s, kind, cores, sample)."""
    import multiprocessing as mp
    from oracle import oracle as O
    from i_whisper_b200.checkpoint import DIMS
    kind = "reference" if os.path.exists(O.REF_PATH) else "port"
    lib_kind = "ref" if kind == "reference" else "port"
    dims = DIMS[model]
    ctx = mp.get_context("spawn")
    with ctx.Pool(procs) as pool:
        res = pool.map(_cpu_sample_worker, [(lib_kind, rows, 1000 + i, model) for i in range(procs)])
    t_layer = float(np.mean([r[0] for r in res]))
    t_stem = float(np.mean([r[1] for r in res]))
    t_dec = float(np.mean([r[2] for r in res]))
    t_clf = float(np.mean([r[3] for r in res]))
    scale = dims.n_audio_ctx / rows
    t_window = dims.n_audio_layer * t_layer * scale + t_stem * scale
    t_token = dims.n_text_layer * t_dec + t_clf
    sample = (f"{procs} processes x (1 encoder layer + conv stem on {rows}/{dims.n_audio_ctx} positions, "
              f"1 decoder layer step + classifier for 1 utterance); per-window time extrapolated x{scale:.1f} rows "
              f"x{dims.n_audio_layer} layers")
    return procs / t_window, procs / t_token, kind, procs, sample


# ---------------------------------------------------------------------------
# GPU arm
# ---------------------------------------------------------------------------
class ClockSampler:
    def __init__(self, dev_index: int):
        self.dev = dev_index
        self.rows = []
        self.proc = None
        self.thread = None

    def __enter__(self):
        q = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
             "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
             "clocks_event_reasons.sw_power_cap")
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={q}", "--format=csv,noheader,nounits",
                                          "-lms", "200", "-i", str(self.dev)], stdout=subprocess.PIPE,
                                         stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except Exception:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) >= 7:
                self.rows.append(parts)

    def __exit__(self, *a):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        sm = [float(r[0]) for r in self.rows if r[0].replace(".", "").isdigit()]
        mx = [float(r[1]) for r in self.rows if r[1].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in self.rows for i in range(4) if r[3 + i].lower() == "active"})
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(self.rows)}


def int8_mm_peak(torch):
    """Empirical dense INT8 tensor-core ceiling: torch._int_mm (cuBLASLt
    IMMA) on 8192^3, best of 10 (burst)."""
    a = torch.randint(-100, 100, (8192, 8192), dtype=torch.int8, device="cuda")
    b = torch.randint(-100, 100, (8192, 8192), dtype=torch.int8, device="cuda")
    for _ in range(3):
        torch._int_mm(a, b)
    best = 1e9
    for _ in range(10):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(); torch._int_mm(a, b); e1.record(); e1.synchronize()
        best = min(best, e0.elapsed_time(e1))
    del a, b
    return 2 * 8192 ** 3 / (best * 1e-3) / 1e12


# DRAM bytes per launch of the four encoder-layer GEMMs (QKV, out-proj,
# fc1, fc2) of whisper-medium measured with ncu at M = 48000 rows, and of
# the tensor-core attention at 64 windows (profiles/gemm_encoder_dram_traffic.md).
GEMM_TRAFFIC_M48000 = (149.0e6, 214.1e6, 199.6e6, 376.9e6)
ATTN_TRAFFIC_B64 = 375.2e6


def traffic_per_launch(kernel: str, windows: int, dims):
    """Measured DRAM traffic of one launch of the dominant kernel family at
    this batch (GEMM: the mean over the four layer shapes, scaled by rows;
    attention: scaled by windows); medium only, None otherwise."""
    if dims.n_audio_state != 1024:
        return None
    if kernel == "attention":
        return round(ATTN_TRAFFIC_B64 * windows / 64)
    if kernel == "gemm_i8":
        rows = windows * dims.n_audio_ctx
        return round(sum(GEMM_TRAFFIC_M48000) / 4 * rows / 48000)
    return None


def load_golden(model: str, sd):
    """The committed oracle digests for this model's calibrated checkpoint
    (tests/golden/calibrated_golden.json), or None when the weights are not
    the ones the digests were made with."""
    from i_whisper_b200.checkpoint import state_digest
    p = os.path.join(ROOT, "tests", "golden", "calibrated_golden.json")
    if not os.path.exists(p):
        return None
    g = json.load(open(p))
    key = {"medium": "medium_w2", "tiny": "tiny_config0", "small": "small_w1", "large": "large_w1"}.get(model)
    ck = g.get("checkpoints", {}).get(model)
    if key not in g or not ck or ck["state_digest"] != state_digest(sd):
        return None
    gold = dict(g[key])
    if isinstance(gold["encoder_sha256"], str):  # a one-window fixture
        gold["encoder_sha256"] = [gold["encoder_sha256"]]
    return gold


def check_parity(golden, xa, toks, seeds):
    """Windows of this rank's batch whose seeds have golden digests: encoder
    output bytes and the first greedy tokens against the oracle's."""
    import hashlib
    if golden is None:
        return {"ok": False, "why": "no golden digests for these weights"}
    sha = lambda a: hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()
    checked, bad = [], []
    for j, s in enumerate(golden["mel_seeds"]):
        if s not in seeds:
            continue
        b = seeds.index(s)
        enc_ok = sha(xa[b].cpu().numpy()) == golden["encoder_sha256"][j]
        tok_ok = True
        if toks is not None:
            # the common prefix: a run may decode fewer tokens than the golden holds
            n = min(len(golden["tokens"][j]), toks.shape[1])
            tok_ok = toks[b, :n].cpu().numpy().tolist() == golden["tokens"][j][:n]
        checked.append(b)
        if not (enc_ok and tok_ok):
            bad.append({"window": b, "encoder": enc_ok, "tokens": tok_ok})
    return {"ok": bool(checked) and not bad, "windows": checked, "mismatches": bad,
            "against": "oracle digests, tests/golden/calibrated_golden.json (encoder output, "
                       f"{golden['sample_len']} greedy tokens)"}


def measured_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        return json.load(open(p))
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "fallback": True}


def main():
    args = parse()
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))

    if args.impl == "reference":
        return reference_arm(args, rank, world)
    if args.config == 1:
        return micro_arm(args, rank, world)

    import torch
    import torch.distributed as dist
    from i_whisper_b200.checkpoint import DIMS, calibrated_name, load_calibrated, synthetic_state_dict
    from i_whisper_b200.model import KernelTimer, WhisperIntB200
    from i_whisper_b200.sharding import max_over_ranks, shard_bounds, window_seeds
    from i_whisper_b200.synthetic import synthetic_mel_batch

    # CPU baseline processes are spawned before this process touches the GPU
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline(args.model, args.cpu_rows, os.cpu_count() or 1)

    torch.cuda.set_device(local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=torch.device("cuda", local))

    def barrier():
        if world > 1:
            t = torch.ones(1, device="cuda")
            dist.all_reduce(t)
        torch.cuda.synchronize()

    B = args.batch
    try:
        dims, sd = load_calibrated(args.model)
        weights = "reference-calibrated checkpoint " + calibrated_name(args.model)
    except FileNotFoundError:
        dims = DIMS[args.model]
        sd = synthetic_state_dict(dims, seed=0)
        weights = "synthetic checkpoint (checkpoint.synthetic_state_dict, seed 0): calibrated one absent"
    golden = load_golden(args.model, sd)
    input_alpha = float(np.asarray(sd["encoder.input_alpha"]).reshape(-1)[0])
    model = WhisperIntB200(dims, sd)
    del sd
    start, stop = shard_bounds(B * world, world, rank)  # weak scaling: B utterances per rank
    seeds = list(args.seeds) if args.seeds else window_seeds(start, stop)
    mels32 = synthetic_mel_batch(dims.n_mels, sorted(set(seeds)), input_alpha)
    by_seed = dict(zip(sorted(set(seeds)), mels32))
    mel_np = np.stack([by_seed[s] for s in seeds])
    mel = torch.from_numpy(mel_np).cuda()
    enc_gops = enc_gop(dims)

    # ---- encoder, device-resident inputs ---------------------------------
    if args.phase == "decoder":
        args.steps, args.warmup = 1, 0
    # the encoder is replayed from a CUDA graph captured once for this batch
    # (the first warm-up call captures it)
    for _ in range(max(1, args.warmup)):
        model.encoder_graphed(mel)
    barrier()
    launches0 = model.replayed_launches
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    # A working set above L2 is timed over back-to-back steps; one that fits
    # in L2 (tiny) is timed one step at a time, each after a 256 MB write
    # that evicts L2, so no step reads what the previous one left there.
    resident = encoder_step_bytes(args.model, B) <= L2_BYTES
    flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda") if resident else None
    with ClockSampler(local) as clk:
        barrier()
        if resident:
            enc_ms = 0.0
            for _ in range(args.steps):
                flush.fill_(1)
                e0.record()
                model.encoder_graphed(mel)
                e1.record()
                e1.synchronize()
                enc_ms += e0.elapsed_time(e1)
        else:
            e0.record()
            for _ in range(args.steps):
                model.encoder_graphed(mel)
            e1.record()
            e1.synchronize()
            enc_ms = e0.elapsed_time(e1)
        barrier()
    launches = model.replayed_launches - launches0
    enc_ms = max_over_ranks(enc_ms, device="cuda")
    # the same steps again with a CUDA event pair around every launch (the
    # per-kernel rates and the roofline): kept out of the headline pass, whose
    # small configurations are bound by the host's launch rate
    timer = KernelTimer()
    model.timer = timer
    for _ in range(args.steps):
        model.encoder(mel)
    model.timer = None
    ksum = timer.summary()
    windows = B * world * args.steps
    value = windows / (enc_ms / 1e3)
    ms_per_step = enc_ms / args.steps

    # ---- encoder end to end through the public API (host buffers) ----------
    # Every step uploads its INT8 mel batch from pinned host memory and
    # downloads its INT8 features to pinned host memory; encode_batches
    # overlaps step i+1's upload and step i-1's download with step i.
    h_mel = torch.from_numpy(mel_np).pin_memory()
    h_outs = [torch.empty(B, dims.n_audio_ctx, dims.n_audio_state, dtype=torch.int8).pin_memory() for _ in range(2)]
    h_out = h_outs[0]
    model.encode_batches([h_mel, h_mel], h_outs)
    barrier()
    f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    f0.record()
    model.encode_batches([h_mel] * args.steps, [h_outs[i % 2] for i in range(args.steps)])
    f1.record()
    barrier()
    e2e_ms = max_over_ranks(f0.elapsed_time(f1), device="cuda")
    e2e_value = windows / (e2e_ms / 1e3)

    # ---- greedy decoder ------------------------------------------------------
    dec_tps = dec_e2e_tps = float("nan")
    dec_ms = float("nan")
    if args.phase == "encoder" or args.decode_tokens <= 0:
        args.decode_runs = 0
    xa = model.encoder(mel)
    rs_xa = model._enc_ws[B]["rs_xa"]
    if args.decode_runs > 0:
        model.decode(xa, rs_xa, args.decode_tokens, use_graph=True)  # warm-up + graph capture
        barrier()
        g0, g1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        g0.record()
        for _ in range(args.decode_runs):
            toks = model.decode(xa, rs_xa, args.decode_tokens, use_graph=True)
        g1.record()
        barrier()
        dec_ms = max_over_ranks(g0.elapsed_time(g1), device="cuda")
        dec_tokens = B * world * args.decode_tokens * args.decode_runs
        dec_tps = dec_tokens / (dec_ms / 1e3)
        h_tok = torch.empty(B, 3 + args.decode_tokens, dtype=torch.int64).pin_memory()
        g0.record()
        toks = model.decode(xa, rs_xa, args.decode_tokens, use_graph=True)
        h_tok.copy_(toks, non_blocking=True)
        g1.record()
        barrier()
        dec_e2e_ms = max_over_ranks(g0.elapsed_time(g1), device="cuda")
        dec_e2e_tps = B * world * args.decode_tokens / (dec_e2e_ms / 1e3)

    # ---- parity (outside the timed regions) -----------------------------------
    parity = check_parity(golden, xa, toks if args.decode_runs > 0 else None, seeds)
    ok = torch.tensor([1 if parity.get("ok") else 0], device="cuda")
    if world > 1:
        dist.all_reduce(ok, op=dist.ReduceOp.MIN)
    parity["all_ranks_ok"] = bool(ok.item())

    # ---- roofline of the dominant kernel ------------------------------------
    peaks = measured_peaks()
    int8_probe = int8_mm_peak(torch)
    int8_peak = 2.0 * peaks["bf16_tflops"]
    dom = max(ksum.items(), key=lambda kv: kv[1]["ms"])
    dname, dk = dom
    kernels = {k: {"launches": v["launches"], "ms": round(v["ms"], 3),
                   "share": round(v["ms"] / max(1e-9, sum(x["ms"] for x in ksum.values())), 4),
                   "tops": round(v["ops"] / (v["ms"] * 1e-3) / 1e12, 2) if v["ops"] else None}
               for k, v in ksum.items()}
    if dk["ops"]:
        achieved = dk["ops"] / dk["launches"] / (dk["ms"] / dk["launches"] * 1e-3) / 1e12
        roof = {"kernel": dname, "bound": "tensor", "achieved": round(achieved, 2), "peak": round(int8_peak, 1),
                "unit": "TFLOP/s", "frac": round(achieved / int8_peak, 4),
                "peak_source": ("2 x MEASURED_PEAKS.json bf16_tflops (dense INT8 = 2 x dense BF16 on B200; "
                                "the file has no INT8 entry)" + (" [fallback peaks]" if peaks.get("fallback") else "")),
                "frac_of_int_mm_probe": round(achieved / int8_probe, 4), "int_mm_probe_tops": round(int8_probe, 1),
                "frac_of_datasheet_4500": round(achieved / DATASHEET_INT8_TOPS, 4),
                "traffic": traffic_per_launch(dname, B, dims), "traffic_unit": "bytes per launch",
                "traffic_source": "ncu dram__bytes_read.sum + dram__bytes_write.sum of this kernel family "
                                  "(GEMM: four encoder shapes at M=48000, scaled by rows; attention: 64 "
                                  "windows, scaled by windows), profiles/gemm_encoder_dram_traffic.md",
                "algorithmic_ops_per_launch": dk["ops"] / dk["launches"]}
    else:
        achieved = dk["bytes"] / dk["launches"] / (dk["ms"] / dk["launches"] * 1e-3) / 1e9
        roof = {"kernel": dname, "bound": "hbm", "achieved": round(achieved, 1), "peak": peaks["hbm_gbs"],
                "unit": "GB/s", "frac": round(achieved / peaks["hbm_gbs"], 4), "traffic": None}
    enc_tops = enc_gops * B * args.steps / (ms_per_step * args.steps * 1e-3) / 1e3

    line = {
        "metric": metric_of(args.model), "value": round(value, 3), "unit": "windows/s", "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms_per_step, 3), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "int8", "data": f"synthetic (seeded sine+noise windows; {weights})",
        "config": arm_config(args, world),
        "pct_int8_tc_peak": {"encoder_tops": round(enc_tops, 1),
                             "of_2x_measured_bf16": round(enc_tops / int8_peak, 4),
                             "of_int_mm_probe": round(enc_tops / int8_probe, 4),
                             "of_datasheet_4500": round(enc_tops / DATASHEET_INT8_TOPS, 4)},
        "parity_checked": parity["all_ranks_ok"],
        "parity": parity,
        "decoder": ({"tok_per_s": round(dec_tps, 1), "e2e_tok_per_s": round(dec_e2e_tps, 1),
                     "tokens_per_utterance": args.decode_tokens, "utterances": B * world,
                     "ms_per_decode": round(dec_ms / max(1, args.decode_runs), 2)} if args.decode_runs > 0 else None),
        "e2e": {"value": round(e2e_value, 3), "unit": "windows/s", "h2d_bytes_per_step": int(h_mel.numel()),
                "d2h_bytes_per_step": int(h_out.numel())},
        "roofline": roof,
        "kernels": kernels,
        "gpu_launches": int(launches),
        "clocks": clk.summary(),
    }
    if cpu is not None:
        cw, ct, kind, cores, sample = cpu
        line["cpu_baseline"] = {"value": round(cw, 6), "unit": "windows/s", "cores": cores, "kind": kind,
                                "sample": sample, "decoder_tok_per_s": round(ct, 3)}
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


GEMM_SHAPES = [(1024, 1024), (1024, 4096), (4096, 1024), (1280, 5120)]


def micro_arm(args, rank, world):
    """BASELINE configs[1], the kernel microbench: every shape timed per
    launch with CUDA events on its stream, a 256 MB write flushing L2 between
    launches (most shapes fit in L2). One JSON line: ``value`` = the GEMMs'
    aggregate TOPS over the twelve shapes; ``kernels`` = each kernel's rate
    and roofline fraction. Rank 0 only (the shapes are single-GPU)."""
    import torch
    from i_whisper_b200 import microbench as MB, ops
    if rank != 0:
        return
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    cpu = None if args.no_cpu_baseline else cpu_kernel_baseline()
    peaks = measured_peaks()
    int8_peak = 2.0 * peaks["bf16_tflops"]
    flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
    reps = max(1, args.steps)
    launches = 0
    kernels, g_ops, g_ms = [], 0.0, 0.0
    with ClockSampler(local) as clk:
        for Bw in (1, 8, 32):
            for K, N in GEMM_SHAPES:
                r = MB.bench_gemm(1500 * Bw, K, N, "linear8", 0, reps, 0, flush=flush, warmup=args.warmup)
                g_ops += 2.0 * r["M"] * N * K * reps
                g_ms += r["ms"] * reps
                r["frac"] = round(r["tops"] / int8_peak, 4)
                kernels.append(r)
                launches += reps
        ln = MB.bench_layernorm(1500, 1024, reps, 0, flush=flush, warmup=args.warmup)
        # the same kernel at the encoder's size in configuration 3 (256 windows x 1500 rows)
        ln_enc = MB.bench_layernorm(1500 * 256, 1024, reps, 0, flush=flush, warmup=args.warmup)
        ln_enc["note"] = "the encoder's LayerNorm at 256 windows (configuration 3's batch)"
        kernels.append(ln_enc)
        launches += reps
        # requantisation of the calibrated whisper-medium checkpoint's first layer
        att = MB.bench_attention(1, 16, 1500, reps, 0, qk_m=68, qk_s=6, fb=14, std=30.0, flush=flush,
                                 warmup=args.warmup)
        att["frac"] = round(att["tops"] / int8_peak, 4)
        kernels += [ln, att]
        launches += 3 * reps  # LayerNorm, attention and its V^T transpose
    tops = g_ops / (g_ms * 1e-3) / 1e12
    # end to end through the public operator: host int8 x -> device -> linear8_cuda -> host
    M, K, N = 48000, 1024, 1024
    g = torch.Generator().manual_seed(0)
    hx = torch.randint(-127, 128, (M, K), dtype=torch.int8, generator=g).pin_memory()
    w = torch.randint(-127, 128, (N, K), dtype=torch.int8, generator=g).cuda()
    mult = torch.full((N,), 1 << 30, dtype=torch.uint32, device="cuda")
    shift = torch.full((N,), 20, dtype=torch.int8, device="cuda")
    hy = torch.empty(M, N, dtype=torch.int8).pin_memory()
    for _ in range(args.warmup):
        hy.copy_(ops.linear8_cuda(hx.cuda(non_blocking=True), w, None, None, mult, shift), non_blocking=True)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        hy.copy_(ops.linear8_cuda(hx.cuda(non_blocking=True), w, None, None, mult, shift), non_blocking=True)
    e1.record()
    e1.synchronize()
    e2e = 2.0 * M * N * K * reps / (e0.elapsed_time(e1) * 1e-3) / 1e12
    line = {"metric": "int8 kernel microbench: w8a8 GEMM TOPS over 12 shapes (+ LayerNorm GB/s, attention TOPS)",
            "value": round(tops, 1), "unit": "TOPS", "n_gpus": 1, "steps": reps, "warmup": args.warmup,
            "ms_per_step": round(g_ms / reps, 4), "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "int8", "data": "synthetic (seeded uniform INT8, per-channel frexp scales, N(0,30) Q/K/V)",
            "config": {"workload": CONFIGS[1]["workload"], "baseline_config": 1, "model": "kernels",
                       "global_batch": 1, "seq_len": 1500, "parallelism": "single GPU",
                       "l2": "flushed between launches (256 MB write)"},
            "roofline": {"kernel": "gemm_i8 (12 shapes)", "bound": "tensor", "achieved": round(tops, 1),
                         "peak": round(int8_peak, 1), "unit": "TFLOP/s", "frac": round(tops / int8_peak, 4),
                         "peak_source": "2 x MEASURED_PEAKS.json bf16_tflops" + (" [fallback]" if peaks.get("fallback") else ""),
                         "frac_of_datasheet_4500": round(tops / DATASHEET_INT8_TOPS, 4), "traffic": None},
            "kernels": kernels,
            "e2e": {"value": round(e2e, 1), "unit": "TOPS", "h2d_bytes_per_step": M * K, "d2h_bytes_per_step": M * N,
                    "note": "ops.linear8_cuda M=48000 K=N=1024 with the host input copied in and the output read back"},
            "gpu_launches": int(launches), "clocks": clk.summary()}
    if cpu is not None:
        line["cpu_baseline"] = cpu
    print(json.dumps(line), flush=True)


def cpu_kernel_baseline():
    """The reference's own scalar linear8 (oracle/_ref, or the port) on one
    host core over the smallest microbench GEMM (M=1500, K=N=1024)."""
    from oracle import oracle as O
    kind = "reference" if os.path.exists(O.REF_PATH) else "port"
    L = O.lib("ref" if kind == "reference" else "port")
    if kind == "port":
        L.set_threads(1)
    rng = np.random.default_rng(0)
    M, K, N = 1500, 1024, 1024
    x = rng.integers(-127, 128, (M, K), dtype=np.int8)
    w = rng.integers(-127, 128, (N, K), dtype=np.int8)
    m = np.full(N, 1 << 30, np.uint32)
    sh = np.full(N, 20, np.int8)
    t0 = time.perf_counter()
    L.linear8(x, w, None, None, m, sh)
    dt = time.perf_counter() - t0
    return {"value": round(2.0 * M * N * K / dt / 1e12, 6), "unit": "TOPS", "cores": 1, "kind": kind,
            "sample": "one linear8 of M=1500, K=N=1024 on one host core"}


L2_BYTES = 126e6


def encoder_step_bytes(model: str, batch: int) -> float:
    """Bytes one encoder step touches at least once: the INT8 weights of
    every block (Q/K/V, out-projection, fc1, fc2: 12 d^2 per layer) and, per
    position, the INT16 residual stream, the LayerNorm output, fused QKV, the
    attention output and fc1's output (11 d bytes)."""
    from i_whisper_b200.checkpoint import DIMS
    d = DIMS[model]
    return 12.0 * d.n_audio_state ** 2 * d.n_audio_layer + 11.0 * d.n_audio_state * batch * d.n_audio_ctx


def arm_config(args, world):
    """The workload both arms report (the reference arm times a bounded sample
    of it on the host cores, see its cpu_baseline.sample)."""
    cfg = CONFIGS[args.config]
    work = cfg["workload"].format(batch=args.batch, tokens=args.decode_tokens)
    if (args.model, args.batch, args.decode_tokens) != (cfg["model"], cfg["batch"], cfg["decode_tokens"]):
        work = (f"whisper-{args.model} integer encoder, {args.batch} windows per GPU; greedy decoder "
                f"{args.decode_tokens} tokens (overrides of BASELINE configs[{args.config}])")
    big = encoder_step_bytes(args.model, args.batch) > L2_BYTES
    return {"workload": work, "baseline_config": args.config,
            "model": f"whisper-{args.model}", "global_batch": args.batch * world, "seq_len": 1500,
            "parallelism": f"utterance-sharded x{world}",
            "l2": (f"working set per step ~{encoder_step_bytes(args.model, args.batch) / 1e9:.2g} GB "
                   "(inputs larger than L2)" if big else
                   "working set per step below L2 (126 MB): each step timed alone after a 256 MB write "
                   "that flushes L2")}


def reference_arm(args, rank, world):
    if rank != 0:
        return
    if args.config == 1:
        return reference_micro_arm(args, world)
    procs = os.cpu_count() or 1
    vals = []
    for _ in range(args.warmup):
        cpu_baseline(args.model, args.cpu_rows, procs)
    t_start = time.time()
    for _ in range(args.steps):
        vals.append(cpu_baseline(args.model, args.cpu_rows, procs))
    wall = time.time() - t_start
    cw = float(np.mean([v[0] for v in vals]))
    ct = float(np.mean([v[1] for v in vals]))
    kind, cores, sample = vals[0][2], vals[0][3], vals[0][4]
    line = {"impl": "reference", "metric": metric_of(args.model), "value": round(cw, 6), "unit": "windows/s",
            "n_gpus": world,
            # ms_per_step is the timed sample step on the host; the metric is
            # extrapolated from it to whole windows (cpu_baseline.sample)
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(wall * 1e3 / args.steps, 1),
            "ms_per_window_extrapolated": round(1e3 / cw, 1) if cw else None,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "int8",
            "data": "synthetic", "config": arm_config(args, world),
            "decoder": {"tok_per_s": round(ct, 4)},
            "cpu_baseline": {"value": round(cw, 6), "unit": "windows/s", "cores": cores, "kind": kind,
                             "sample": sample},
            "e2e": {"value": round(cw, 6), "unit": "windows/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "wall_s": round(wall, 1)}
    print(json.dumps(line), flush=True)


def reference_micro_arm(args, world):
    """The reference arm of the kernel microbench: the reference's scalar
    linear8 on one host core, one bounded sample per step."""
    for _ in range(args.warmup):
        cpu_kernel_baseline()
    t0 = time.time()
    vals = [cpu_kernel_baseline() for _ in range(args.steps)]
    wall = time.time() - t0
    v = float(np.mean([c["value"] for c in vals]))
    cb = dict(vals[0], value=round(v, 6))
    line = {"impl": "reference", "metric": "int8 kernel microbench: w8a8 GEMM TOPS over 12 shapes (+ LayerNorm GB/s, "
            "attention TOPS)", "value": round(v, 6), "unit": "TOPS", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(wall * 1e3 / max(1, args.steps), 1), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "int8", "data": "synthetic",
            "config": {"workload": CONFIGS[1]["workload"], "baseline_config": 1, "model": "kernels"},
            "cpu_baseline": cb, "e2e": {"value": round(v, 6), "unit": "TOPS", "h2d_bytes_per_step": 0,
                                        "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
