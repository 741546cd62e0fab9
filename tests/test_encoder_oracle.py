"""The encoder front end's oracle (log-mel, conv stem) pinned to the
reference's own tests (mel.rs:277-310, conv.rs:472-568; values in
tests/golden/), plus properties the reference code implies."""
import json
import os

import numpy as np
import pytest

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


@pytest.fixture(scope="module")
def ref_tests():
    with open(os.path.join(GOLDEN, "reference_unit_tests.json")) as f:
        return json.load(f)


def test_silence_has_constant_value(oracle, ref_tests):
    t = ref_tests["silence_has_constant_value"]  # mel.rs:277-294
    m = oracle.MelCtx(t["left_pad_samples"])
    assert m.left_pad_samples() == t["expect_left_pad"]
    assert m.feed(np.zeros(t["feed_zeros"], np.float32)) == t["expect_frames"]
    mel, n = m.data()
    assert n == t["expect_frames"] and mel.shape == (n, 128)
    assert np.max(np.abs(mel - t["expect_value"])) < t["tol"]


def test_finish_drops_last_frame(oracle, ref_tests):
    t = ref_tests["finish_drops_last_frame"]  # mel.rs:296-310
    m = oracle.MelCtx(0)
    m.feed(np.zeros(t["feed_zeros"], np.float32))
    m.finish(0)
    assert m.data()[1] == t["expect_frames_after_finish"]


def _offline_stem(oracle, t, mel):
    mb, dim, frames = t["mel_bins"], t["dim"], t["frames"]
    c0 = oracle.gelu(oracle.causal_conv1d_colmajor(mel.reshape(frames, mb).T.copy(), t["conv0_weight"],
                                                   t["conv0_bias"], mb, dim, frames, 3, 1).ravel())
    c0 = c0.reshape(dim, frames)
    c1 = oracle.gelu(oracle.causal_conv1d_colmajor(c0, t["conv1_weight"], t["conv1_bias"], dim, dim, frames, 3,
                                                   2).ravel()).reshape(dim, frames // 2)
    return c0, c1.T.copy()


def test_incremental_conv_matches_offline_even_length(oracle, ref_tests):
    t = ref_tests["incremental_conv_matches_offline_even_length"]  # conv.rs:472-568
    mel = np.array(t["mel"], np.float32)
    _, offline = _offline_stem(oracle, t, mel)
    st = oracle.ConvStemState(t["mel_bins"], t["dim"], t["conv0_weight"], t["conv0_bias"], t["conv1_weight"],
                              t["conv1_bias"])
    got, cur = [], 0
    for cs in t["chunks"]:
        got.append(st.process(mel[cur * t["mel_bins"]:(cur + cs) * t["mel_bins"]]))
        cur += cs
    got = np.concatenate(got)
    assert got.shape == offline.shape
    assert np.max(np.abs(got - offline)) < t["tol"]


def test_conv_out_len_and_causality(oracle):
    """conv.rs:35-37 output length; a causal conv's output at t ignores inputs after t."""
    for length in range(0, 9):
        for k, s in ((3, 1), (3, 2)):
            want = max(0, int(np.ceil((length - k + (k - s)) / s + 1))) if length else 0
            assert oracle.lib().vo_conv_out_len(length, k, s) == max(want, 0)
    rng = np.random.default_rng(0)
    x = rng.standard_normal((4, 10)).astype(np.float32)
    w = rng.standard_normal(5 * 4 * 3).astype(np.float32)
    y = oracle.causal_conv1d_colmajor(x, w, None, 4, 5, 10, 3, 1)
    x2 = x.copy()
    x2[:, 6:] = 0
    y2 = oracle.causal_conv1d_colmajor(x2, w, None, 4, 5, 10, 3, 1)
    assert np.array_equal(y[:, :6], y2[:, :6])


def test_mel_streaming_equals_one_shot(oracle):
    """Feeding in chunks gives the same frames as feeding all at once."""
    rng = np.random.default_rng(1)
    x = (0.1 * rng.standard_normal(16000)).astype(np.float32)
    a, b = oracle.MelCtx(320), oracle.MelCtx(320)
    a.feed(x)
    cur = 0
    for n in (1, 159, 160, 2000, 777):
        b.feed(x[cur:cur + n])
        cur += n
    b.feed(x[cur:])
    a.finish(1280)
    b.finish(1280)
    ma, na = a.data()
    mb, nb = b.data()
    assert na == nb and np.array_equal(ma, mb)
