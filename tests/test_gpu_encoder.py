"""GPU parity of the encoder front end: the log-mel spectrogram (MelCtx,
mel.rs:114-272) and the causal conv stem (ConvStemState, conv.rs:134-347)
against the oracle's restatement, on the reference's own tests (fixtures in
tests/golden/) and on the model's shapes (128 mel bins, encoder dim 1280)
with random audio fed in uneven chunks.

Tolerances: the DFT power and the mel band sums are formed in the
reference's order with separately rounded products and sums, so they match
exactly; log10f and tanhf may differ from the host libm in the last place,
so log-mel values are compared within 1e-5 and conv stem outputs within
1e-5 (the reference's own incremental-vs-offline test allows 1e-4)."""
import json
import os

import numpy as np
import pytest

from tests.vox_testlib import vox

pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")
MEL_TOL, CONV_TOL = 1e-5, 1e-5


@pytest.fixture(scope="module")
def V():
    return vox()


@pytest.fixture(scope="module")
def ref_tests():
    with open(os.path.join(GOLDEN, "reference_unit_tests.json")) as f:
        return json.load(f)


def test_silence_and_finish_reference_tests(V, ref_tests):
    t = ref_tests["silence_has_constant_value"]  # mel.rs:277-294
    m = V.MelCtx(t["left_pad_samples"])
    assert m.left_pad_samples() == t["expect_left_pad"]
    assert m.feed(np.zeros(t["feed_zeros"], np.float32)) == t["expect_frames"]
    mel, n = m.data()
    assert n == t["expect_frames"]
    assert np.max(np.abs(mel - t["expect_value"])) < t["tol"]
    t = ref_tests["finish_drops_last_frame"]  # mel.rs:296-310
    m = V.MelCtx(0)
    m.feed(np.zeros(t["feed_zeros"], np.float32))
    m.finish(0)
    assert m.frames() == t["expect_frames_after_finish"]


@pytest.mark.parametrize("left_pad,chunks,right_pad", [(0, [400, 1, 159, 3000, 12000, 777], 0),
                                                       (512, [16000, 24000], 1280 * 17 + 640),
                                                       (0, [100, 150], 0)])
def test_log_mel_matches_oracle(V, oracle, left_pad, chunks, right_pad):
    rng = np.random.default_rng(len(chunks) + left_pad)
    x = (0.2 * rng.standard_normal(sum(chunks))).astype(np.float32)
    a, b = V.MelCtx(left_pad), oracle.MelCtx(left_pad)
    cur = 0
    for n in chunks:
        na, nb = a.feed(x[cur:cur + n]), b.feed(x[cur:cur + n])
        assert na == nb
        cur += n
    a.finish(right_pad)
    b.finish(right_pad)
    ma, fa = a.data()
    mb, fb = b.data()
    assert fa == fb and ma.shape == mb.shape
    if fa:
        assert np.max(np.abs(ma - mb)) < MEL_TOL


def test_conv_stem_reference_test(V, oracle, ref_tests):
    t = ref_tests["incremental_conv_matches_offline_even_length"]  # conv.rs:472-568
    mel = np.array(t["mel"], np.float32)
    st = V.ConvStemState(t["mel_bins"], t["dim"], t["conv0_weight"], t["conv0_bias"], t["conv1_weight"],
                         t["conv1_bias"])
    ref = oracle.ConvStemState(t["mel_bins"], t["dim"], t["conv0_weight"], t["conv0_bias"], t["conv1_weight"],
                               t["conv1_bias"])
    cur, got, want = 0, [], []
    for cs in t["chunks"]:
        part = mel[cur * t["mel_bins"]:(cur + cs) * t["mel_bins"]]
        got.append(st.process(part))
        want.append(ref.process(part))
        assert got[-1].shape == want[-1].shape
        cur += cs
    got, want = np.concatenate(got), np.concatenate(want)
    assert np.max(np.abs(got - want)) < CONV_TOL
    # and against the offline stem, as the reference test checks
    mb, dim, frames = t["mel_bins"], t["dim"], t["frames"]
    c0 = oracle.gelu(oracle.causal_conv1d_colmajor(mel.reshape(frames, mb).T.copy(), t["conv0_weight"],
                                                   t["conv0_bias"], mb, dim, frames, 3, 1).ravel()).reshape(dim, frames)
    c1 = oracle.gelu(oracle.causal_conv1d_colmajor(c0, t["conv1_weight"], t["conv1_bias"], dim, dim, frames, 3,
                                                   2).ravel()).reshape(dim, frames // 2)
    assert np.max(np.abs(got - c1.T)) < t["tol"]


def test_conv_stem_model_shapes_uneven_chunks(V, oracle):
    """128 mel bins -> dim 1280, bf16-representable weights ~N(0, 0.02), chunks
    of 1, 2, odd and even sizes (the stride-2 residual carried across)."""
    mb, dim = 128, 1280
    w0 = oracle.bf16_to_f32(oracle.gen_normal_bf16(3, 7000, 0.02, dim * mb * 3))
    w1 = oracle.bf16_to_f32(oracle.gen_normal_bf16(3, 7001, 0.02, dim * dim * 3))
    b0 = oracle.gen_normal_f32(3, 7002, 0.02, dim)
    b1 = oracle.gen_normal_f32(3, 7003, 0.02, dim)
    rng = np.random.default_rng(7)
    chunks = [1, 2, 5, 8, 1, 1, 16, 3]
    mel = (rng.standard_normal((sum(chunks), mb)) * 0.5).astype(np.float32)
    st = V.ConvStemState(mb, dim, w0, b0, w1, b1)
    ref = oracle.ConvStemState(mb, dim, w0, b0, w1, b1)
    cur = 0
    for cs in chunks:
        g, w = st.process(mel[cur:cur + cs]), ref.process(mel[cur:cur + cs])
        assert g.shape == w.shape, (cur, g.shape, w.shape)
        if g.size:
            assert np.max(np.abs(g - w)) < CONV_TOL * max(1.0, float(np.max(np.abs(w))))
        cur += cs


@pytest.mark.parametrize("stride", [1, 2])
def test_causal_conv1d_op(V, oracle, stride):
    rng = np.random.default_rng(stride)
    cin, cout, length = 37, 300, 23
    x = rng.standard_normal((cin, length)).astype(np.float32)
    w = (0.1 * rng.standard_normal(cout * cin * 3)).astype(np.float32)
    b = rng.standard_normal(cout).astype(np.float32)
    got = V.causal_conv1d_gelu(x, w, b, cin, cout, length, stride, gelu=False)
    want = oracle.causal_conv1d_colmajor(x, w, b, cin, cout, length, 3, stride)
    assert np.array_equal(got, want)  # sums in the reference's order: bit-exact
    got = V.causal_conv1d_gelu(x, w, None, cin, cout, length, stride, gelu=True)
    want = oracle.gelu(oracle.causal_conv1d_colmajor(x, w, None, cin, cout, length, 3, stride).ravel())
    assert np.max(np.abs(got.ravel() - want)) < CONV_TOL * max(1.0, float(np.max(np.abs(want))))
