"""The exact folding of a Linear_int weight zero point into int8 weights
(model.fold_zero_point), on the CPU: sum_k x*(w - wz) == s * sum_k x*w' for
every channel, with w' in int8 and s = +-1, and None where a channel's
differences fit int8 neither way."""
import numpy as np

from i_whisper_b200.model import fold_zero_point


def test_fold_identity_and_signs():
    rng = np.random.default_rng(0)
    N, K = 64, 96
    w = rng.integers(-100, 101, (N, K)).astype(np.int8)
    wz = rng.integers(-27, 28, N).astype(np.int8)
    w[::5, 0], wz[::5] = 127, -1      # a difference of +128: folded negated
    w[2::5, 1], wz[2::5] = -128, 0    # -128 fits as it is
    wf, s = fold_zero_point(w, wz)
    assert wf.dtype == np.int8 and s.dtype == np.int8
    assert set(np.unique(s)) == {-1, 1} and (s[::5] == -1).all()
    x = rng.integers(-128, 128, (33, K)).astype(np.int64)
    acc = x @ w.astype(np.int64).T - np.outer(x.sum(1), wz.astype(np.int64))
    assert np.array_equal(acc, (x @ wf.astype(np.int64).T) * s.astype(np.int64))


def test_fold_refuses_unrepresentable_channels():
    w = np.array([[127, -128, 0]], np.int8)
    assert fold_zero_point(w, np.array([-2], np.int8)) is None   # differences 129 and -126
    assert fold_zero_point(w, np.array([2], np.int8)) is None    # 125 and -130
    w1, s1 = fold_zero_point(w, np.array([-1], np.int8))         # 128 and -127: negated
    assert s1.tolist() == [-1] and w1.tolist() == [[-128, 127, -1]]
    w0, s0 = fold_zero_point(w, np.zeros(1, np.int8))
    assert s0.tolist() == [1] and np.array_equal(w0, w)
