"""GPU parity of the op-level entry points against the oracle and the
reference's own unit-test vectors (tests/golden/reference_unit_tests.json)."""
import json
import os

import numpy as np
import pytest

from tests.vox_testlib import vox

pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


@pytest.fixture(scope="module")
def V():
    return vox()


@pytest.fixture(scope="module")
def ctx(V):
    c = V.DecoderConfig(dim=8, hidden_dim=16, n_heads=2, n_kv_heads=1, head_dim=4, sliding_window=4,
                        norm_eps=1e-5, rope_theta=1e4)
    with V.Context(c) as cx:
        yield cx


@pytest.fixture(scope="module")
def ref_tests():
    with open(os.path.join(GOLDEN, "reference_unit_tests.json")) as f:
        return json.load(f)


def test_linear_smoke_golden(V, ctx, ref_tests):
    t = ref_tests["linear_smoke"]  # ops.rs:139-151 (in_dim 3: f32 weights need in_dim % 4 == 0)
    # Pad in_dim to 4 with a zero column: the sums are unchanged.
    x = np.array(t["x"], np.float32).reshape(2, 3)
    w = np.array(t["w"], np.float32).reshape(2, 3)
    xp = np.concatenate([x, np.zeros((2, 1), np.float32)], 1)
    wp = np.concatenate([w, np.zeros((2, 1), np.float32)], 1)
    y = V.linear(ctx, xp, 2, 4, wp, 2, np.array(t["bias"], np.float32))
    assert np.max(np.abs(y - np.array(t["expected"], np.float32))) < t["tol"]


def test_linear_unsupported_in_dim_is_an_error(V, ctx):
    with pytest.raises(V.VoxError) as e:
        V.linear(ctx, np.zeros(3, np.float32), 1, 3, np.zeros(6, np.float32), 2)
    assert e.value.code == V.ERR_UNSUPPORTED


@pytest.mark.parametrize("n_rows,in_dim,out_dim,bf16,bias", [
    (1, 3072, 4096, True, False), (1, 4096, 3072, True, False), (1, 9216, 3072, True, False),
    (1, 3072, 18432, True, False), (3, 64, 37, True, True), (2, 3072, 300, False, True),
    (1, 8, 5, True, False), (1, 16384, 64, True, False), (1, 8192, 64, False, False),
])
def test_linear_matches_oracle(V, ctx, oracle, n_rows, in_dim, out_dim, bf16, bias):
    rng = np.random.default_rng(in_dim + out_dim)
    x = rng.standard_normal(n_rows * in_dim).astype(np.float32)
    b = rng.standard_normal(out_dim).astype(np.float32) if bias else None
    if bf16:
        w = oracle.gen_normal_bf16(3, in_dim, 0.02, in_dim * out_dim)
        ref = oracle.linear_bf16(x, n_rows, in_dim, w, out_dim, b)
    else:
        w = oracle.gen_normal_f32(3, in_dim, 0.02, in_dim * out_dim)
        ref = oracle.linear(x, n_rows, in_dim, w, out_dim, b)
    got = V.linear(ctx, x, n_rows, in_dim, w, out_dim, b)
    scale = np.sqrt(in_dim) * 0.02
    assert np.max(np.abs(got - ref)) < 2e-5 * scale + 1e-6


@pytest.mark.parametrize("n_rows,in_dim,out_dim,bias", [
    (1, 3072, 6144, False), (4, 3072, 6144, False), (8, 3072, 6144, True), (8, 4096, 3072, False),
    (3, 9216, 3072, False), (8, 3072, 18432, False), (5, 64, 37, True), (2, 128, 129, False),
    (8, 3072, 131072, False), (7, 640, 300, True),
])
def test_linear_batched_matches_oracle(V, ctx, oracle, n_rows, in_dim, out_dim, bias):
    """Tensor-core skinny GEMM (tcgen05, f32 accumulation, x as bf16 hi + lo)
    against the oracle's sequential f32 sums; tolerance 1e-4 of the output
    scale sqrt(in_dim) * 0.02."""
    rng = np.random.default_rng(in_dim * 7 + out_dim + n_rows)
    x = rng.standard_normal(n_rows * in_dim).astype(np.float32)
    b = rng.standard_normal(out_dim).astype(np.float32) if bias else None
    w = oracle.gen_normal_bf16(5, in_dim, 0.02, in_dim * out_dim)
    ref = oracle.linear_bf16(x, n_rows, in_dim, w, out_dim, b)
    got = V.linear_batched(ctx, x, n_rows, in_dim, w, out_dim, b)
    scale = np.sqrt(in_dim) * 0.02
    err = float(np.max(np.abs(got - ref)))
    assert err < 1e-4 * scale + 1e-6, f"max abs error {err:.3e} (scale {scale:.3f})"


def test_linear_batched_limits_are_errors(V, ctx):
    with pytest.raises(V.VoxError) as e:
        V.linear_batched(ctx, np.zeros(9 * 64, np.float32), 9, 64, np.zeros(64 * 4, np.uint16), 4)
    assert e.value.code == V.ERR_UNSUPPORTED
    with pytest.raises(V.VoxError) as e:
        V.linear_batched(ctx, np.zeros(32, np.float32), 1, 32, np.zeros(32 * 4, np.uint16), 4)
    assert e.value.code == V.ERR_UNSUPPORTED


def test_gqa_golden(V, ctx, ref_tests):
    t = ref_tests["gqa_matches_expanded_kv_reference"]  # ops.rs:154-237
    sh = V.AttentionShape(t["n_heads"], t["head_dim"], t["seq_len"], t["n_kv_heads"], t["sliding_window"])
    got = V.attention_gqa_step(ctx, t["q"], t["k"], t["v"], sh)
    assert np.max(np.abs(got - np.array(t["expected"], np.float32))) < t["tol"]


@pytest.mark.parametrize("nh,nkv,hd,seq,win", [
    (32, 8, 128, 1, 0), (32, 8, 128, 1536, 8192), (32, 8, 128, 8192, 8192), (32, 8, 128, 700, 300),
    (4, 2, 3, 5, 0), (8, 8, 64, 100, 0), (16, 2, 12, 77, 40), (32, 8, 128, 0, 0), (6, 3, 5, 33, 7),
])
def test_attention_matches_oracle(V, ctx, oracle, nh, nkv, hd, seq, win):
    rng = np.random.default_rng(seq + hd)
    q = rng.standard_normal(nh * hd).astype(np.float32)
    k = rng.standard_normal(seq * nkv * hd).astype(np.float32)
    v = rng.standard_normal(seq * nkv * hd).astype(np.float32)
    ref = oracle.attention_gqa_step(q, k, v, nh, hd, seq, nkv, win)
    got = V.attention_gqa_step(ctx, q, k, v, V.AttentionShape(nh, hd, seq, nkv, win))
    assert np.max(np.abs(got - ref)) < 1e-4


def test_rms_norm_golden_and_oracle(V, ctx, oracle, ref_tests):
    t = ref_tests["rms_norm_rows_smoke"]  # math.rs:95-104
    out = V.rms_norm_rows(ctx, t["input"], t["weight"], t["dim"], t["eps"])
    assert abs(out[0] - t["expected_first_row"][0]) < t["tol"]
    assert abs(out[1] - t["expected_first_row"][1]) < t["tol"]
    rng = np.random.default_rng(5)
    x = rng.standard_normal(3 * 3072 + 5).astype(np.float32)  # ragged tail stays untouched
    w = rng.standard_normal(3072).astype(np.float32)
    ref = oracle.rms_norm_rows(x, w, 3072, 1e-5)
    got = V.rms_norm_rows(ctx, x, w, 3072, 1e-5)
    assert np.max(np.abs(got - ref)) < 1e-5
    assert np.all(got[3 * 3072:] == 0)


def test_rope_golden_and_oracle(V, ctx, oracle, ref_tests):
    t = ref_tests["rope_preserves_pairwise_norm"]  # math.rs:107-133
    before = np.array(t["x"], np.float32)
    x = V.rope_interleaved_inplace(ctx, before, t["seq_len"], t["n_heads"], t["head_dim"], t["pos_offset"],
                                   t["theta"])
    for i0 in range(0, before.size, 2):
        n0 = before[i0] ** 2 + before[i0 + 1] ** 2
        n1 = x[i0] ** 2 + x[i0 + 1] ** 2
        assert abs(n0 - n1) < t["tol"]
    rng = np.random.default_rng(6)
    d = rng.standard_normal(5 * 32 * 128).astype(np.float32)
    ref = oracle.rope_interleaved(d, 5, 32, 128, 16380, 1e6)
    got = V.rope_interleaved_inplace(ctx, d, 5, 32, 128, 16380, 1e6)
    assert np.array_equal(got, ref)  # same table, unfused rotation: bit-exact


def test_silu_softmax_golden_and_oracle(V, ctx, oracle, ref_tests):
    t = ref_tests["silu_and_softmax_smoke"]  # math.rs:136-147
    v = V.silu_inplace(ctx, t["silu_input"])
    assert v[1] > v[0] and v[2] < v[0]
    s = V.softmax_inplace(ctx, t["softmax_input"])
    assert abs(float(np.sum(s)) - 1.0) < t["sum_tol"] and s[2] > s[1] > s[0]
    rng = np.random.default_rng(7)
    x = (rng.standard_normal(9216) * 4).astype(np.float32)
    assert np.max(np.abs(V.silu_inplace(ctx, x) - oracle.silu(x))) < 1e-5
    ref = oracle.softmax(x)
    # the GPU sums the 9216 exponentials as a tree, the reference left to right
    assert np.max(np.abs(V.softmax_inplace(ctx, x) - ref)) < 2e-5 * np.max(ref)


def test_add_inplace(V, ctx, oracle):
    rng = np.random.default_rng(8)
    a = rng.standard_normal(3072).astype(np.float32)
    b = rng.standard_normal(3072).astype(np.float32)
    assert np.array_equal(V.add_inplace(ctx, a, b), oracle.add_inplace(a, b))
