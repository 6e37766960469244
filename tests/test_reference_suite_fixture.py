"""The recorded calls of the reference's kernel test suite
(tests/golden/reference_suite_calls.*, replayed on the CUDA kernels by
test_gpu_reference_suite.py) checked on the CPU: no reference checkout is
needed, the C ABI is emulated over the oracle."""


def test_recorded_suite_calls_replay_on_the_emulator(monkeypatch):
    """The fixture the GPU replays (tests/golden/reference_suite_calls.*)
    reproduces on the CPU emulator: every recorded call gives the recorded
    output digests or exception class, and the record covers the suite."""
    from capi_emulator import install
    from reference_c_names import make_C
    from reference_replay import CALLS, replay
    assert len(CALLS) >= 1400 and len({c["test"] for c in CALLS}) >= 1390
    ops = {c["op"].replace("_simd", "_scalar") for c in CALLS}
    for op in ("linear8_scalar", "linear32_scalar", "layernorm32_scalar", "gelu_scalar", "qk_requant_rowmax_scalar",
               "shift_exp_scalar", "pv_norm_requant_scalar", "conv1d_scalar", "add_requant15_scalar",
               "classifier_scalar", "residual15_scalar"):
        assert op in ops, op
    install(monkeypatch.setattr)
    C = make_C()
    for c in CALLS:
        replay(c, C, "cpu")
