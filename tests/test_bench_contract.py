"""bench.py's reference arm and its JSON line, on the CPU.

The reference arm times the reference's own scalar C++ kernels (or the
oracle port where they were not built) on the host cores. This test runs it
on the tiny model with one small sample step and checks the keys and units
of the line it prints, and that a rank other than 0 prints nothing and
exits 0, as a torchrun launch of both arms requires."""
import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
ARGS = [sys.executable, "bench.py", "--impl", "reference", "--model", "tiny", "--steps", "1", "--warmup", "0",
        "--cpu-rows", "16"]


def _run(extra_env=None):
    env = dict(os.environ, **(extra_env or {}))
    return subprocess.run(ARGS, cwd=ROOT, env=env, capture_output=True, text=True, timeout=600)


def test_reference_arm_line():
    r = _run()
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [ln for ln in r.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1
    d = json.loads(lines[0])
    assert d["impl"] == "reference"
    for k in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better", "scaling",
              "vs_baseline", "dtype", "data", "config", "cpu_baseline", "e2e"):
        assert k in d, k
    assert d["value"] > 0 and d["unit"] == "windows/s" and d["higher_is_better"] is True
    assert d["steps"] == 1 and d["warmup"] == 0 and d["n_gpus"] == 1
    assert "whisper-tiny" in d["config"]["workload"]
    cb = d["cpu_baseline"]
    assert cb["value"] == d["value"] and cb["kind"] in ("reference", "port") and cb["cores"] >= 1 and cb["sample"]
    assert d["e2e"] == {"value": d["value"], "unit": "windows/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}
    # the timed sample step, not the extrapolated window time
    assert d["ms_per_step"] <= 1e3 * d["wall_s"] + 100
    assert d["ms_per_window_extrapolated"] > 0


def test_reference_arm_other_ranks_exit_quietly():
    r = _run({"RANK": "1", "WORLD_SIZE": "2", "LOCAL_RANK": "1"})
    assert r.returncode == 0, r.stderr[-2000:]
    assert r.stdout.strip() == ""


def test_encoder_work_formula_matches_the_published_table():
    """enc_gop (the roofline's algorithmic work per window) reproduces the
    per-size figures 36.9 / 344.2 / 1138.1 / 2273.8 GOP."""
    sys.path.insert(0, ROOT)
    import bench
    from i_whisper_b200.checkpoint import DIMS
    for name, gop in bench.ENC_GOP.items():
        assert round(bench.enc_gop(DIMS[name]), 1) == gop, name


def test_reference_arm_follows_the_config():
    """--config selects BASELINE configurations: 0 is whisper-tiny on one
    window, 1 the kernel microbench (the reference's linear8 in TOPS)."""
    r0 = subprocess.run([sys.executable, "bench.py", "--impl", "reference", "--config", "0", "--steps", "1",
                         "--warmup", "0", "--cpu-rows", "16"], cwd=ROOT, capture_output=True, text=True, timeout=600)
    assert r0.returncode == 0, r0.stderr[-2000:]
    d0 = json.loads([ln for ln in r0.stdout.splitlines() if ln.startswith("{")][0])
    assert d0["config"]["baseline_config"] == 0 and "whisper-tiny" in d0["config"]["workload"]
    assert "whisper-tiny" in d0["metric"]
    r1 = subprocess.run([sys.executable, "bench.py", "--impl", "reference", "--config", "1", "--steps", "1",
                         "--warmup", "0"], cwd=ROOT, capture_output=True, text=True, timeout=600)
    assert r1.returncode == 0, r1.stderr[-2000:]
    d1 = json.loads([ln for ln in r1.stdout.splitlines() if ln.startswith("{")][0])
    assert d1["unit"] == "TOPS" and d1["value"] > 0 and d1["config"]["baseline_config"] == 1
    assert d1["cpu_baseline"]["cores"] == 1 and d1["e2e"]["unit"] == "TOPS"


def test_parity_check_compares_the_decoded_prefix():
    """A run that decodes fewer tokens than the golden holds is checked on
    the tokens it has (and a wrong one among them still fails)."""
    import hashlib

    import numpy as np
    import torch

    sys.path.insert(0, ROOT)
    import bench

    xa = torch.arange(2 * 6, dtype=torch.int8).reshape(2, 2, 3)
    sha = [hashlib.sha256(xa[i].numpy().tobytes()).hexdigest() for i in range(2)]
    gold_toks = [[50258, 50259, 50359, 11, 12, 13, 14, 15], [50258, 50259, 50359, 21, 22, 23, 24, 25]]
    golden = {"mel_seeds": [0, 1], "encoder_sha256": sha, "tokens": gold_toks, "sample_len": 5}
    short = torch.tensor([t[:5] for t in gold_toks])
    r = bench.check_parity(golden, xa, short, [0, 1])
    assert r["ok"] and r["windows"] == [0, 1]
    full = torch.tensor(gold_toks)
    assert bench.check_parity(golden, xa, full, [0, 1])["ok"]
    bad = short.clone()
    bad[1, 4] = 99
    r = bench.check_parity(golden, xa, bad, [0, 1])
    assert not r["ok"] and r["mismatches"] == [{"window": 1, "encoder": True, "tokens": False}]
    assert np.array_equal(bad[0].numpy(), short[0].numpy())
