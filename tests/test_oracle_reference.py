"""Pins the CPU oracle to the reference crate's own hot-path unit tests.

Each test re-runs one reference test (cited) on the oracle, with the inputs
and expected answers stored in tests/golden/reference_unit_tests.json.
"""
import json
import os

import numpy as np
import pytest

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


@pytest.fixture(scope="module")
def ref_tests():
    with open(os.path.join(GOLDEN, "reference_unit_tests.json")) as f:
        return json.load(f)


def test_linear_smoke(oracle, ref_tests):
    t = ref_tests["linear_smoke"]  # ops.rs:139-151
    y = oracle.linear(t["x"], t["n_rows"], t["in_dim"], t["w"], t["out_dim"], t["bias"])
    assert np.max(np.abs(y - np.array(t["expected"], np.float32))) < t["tol"]


def test_gqa_matches_expanded_kv_reference(oracle, ref_tests):
    t = ref_tests["gqa_matches_expanded_kv_reference"]  # ops.rs:154-237
    got = oracle.attention_gqa_step(t["q"], t["k"], t["v"], t["n_heads"], t["head_dim"],
                                    t["seq_len"], t["n_kv_heads"], t["sliding_window"])
    assert np.max(np.abs(got - np.array(t["expected"], np.float32))) < t["tol"]


def test_rms_norm_rows_smoke(oracle, ref_tests):
    t = ref_tests["rms_norm_rows_smoke"]  # math.rs:95-104
    out = oracle.rms_norm_rows(t["input"], t["weight"], t["dim"], t["eps"])
    assert abs(out[0] - t["expected_first_row"][0]) < t["tol"]
    assert abs(out[1] - t["expected_first_row"][1]) < t["tol"]


def test_rope_preserves_pairwise_norm(oracle, ref_tests):
    t = ref_tests["rope_preserves_pairwise_norm"]  # math.rs:107-133
    before = np.array(t["x"], np.float32)
    x = oracle.rope_interleaved(before, t["seq_len"], t["n_heads"], t["head_dim"],
                                t["pos_offset"], t["theta"])
    for i0 in range(0, before.size, 2):
        n0 = before[i0] * before[i0] + before[i0 + 1] * before[i0 + 1]
        n1 = x[i0] * x[i0] + x[i0 + 1] * x[i0 + 1]
        assert abs(n0 - n1) < t["tol"]


def test_silu_and_softmax_smoke(oracle, ref_tests):
    t = ref_tests["silu_and_softmax_smoke"]  # math.rs:136-147
    v = oracle.silu(t["silu_input"])
    assert v[1] > v[0] and v[2] < v[0]
    s = oracle.softmax(t["softmax_input"])
    assert abs(float(np.sum(s)) - 1.0) < t["sum_tol"]
    assert s[2] > s[1] > s[0]


def test_compacts_when_exceeding_window(oracle, ref_tests):
    t = ref_tests["compacts_when_exceeding_window"]  # kv.rs:109-136
    kv = oracle.RollingKvCache(t["n_layers"], t["n_kv_heads"], t["head_dim"], t["window"])
    for a in t["appends"]:
        kv.append_layer(0, a["k"], a["v"], a["n"])
        assert kv.layer_len_tokens(0) == a["expect_len"]
        assert kv.layer_pos_offset(0) == a["expect_pos_offset"]
    k, v = kv.layer_tensors(0)
    stride = t["n_kv_heads"] * t["head_dim"]
    assert k.size == 4 * stride and v.size == 4 * stride
    assert k[0] == t["expect_k_first"] and v[0] == t["expect_v_first"]
    assert k[3 * stride] == t["expect_k_last"] and v[3 * stride] == t["expect_v_last"]


def test_layers_are_isolated(oracle, ref_tests):
    t = ref_tests["layers_are_isolated"]  # kv.rs:139-151
    kv = oracle.RollingKvCache(t["n_layers"], t["n_kv_heads"], t["head_dim"], t["window"])
    for a in t["appends"]:
        kv.append_layer(a["layer"], a["k"], a["v"], a["n"])
    for layer in range(2):
        assert kv.layer_len_tokens(layer) == t["expect_len"][layer]
        assert kv.layer_tensors(layer)[0].tolist() == t["expect_k"][layer]


def test_decoder_step_grows_and_compacts_cache(oracle, ref_tests):
    t = ref_tests["decoder_step_grows_and_compacts_cache"]  # decoder.rs:185-214
    c = t["config"]
    cfg = oracle.config(**c)
    w = {k: np.array(v, np.float32) for k, v in t["weights"].items()}
    lw = oracle.LayerWeights(w["attention_norm"], w["ffn_norm"],
                             **{n: w[n] for n in oracle.LayerWeights.NAMES})
    cache = oracle.RollingKvCache(1, c["n_kv_heads"], c["head_dim"], c["sliding_window"])
    from tests.golden.make_golden import decoder_test_hidden
    for pos in range(t["steps"]):
        out = oracle.decoder_layer_forward_step(cfg, 0, lw, cache,
                                                decoder_test_hidden(pos, c["dim"]), pos)
        assert out.shape == (c["dim"],) and np.all(np.isfinite(out))
    assert cache.layer_len_tokens(0) == t["expect_len"]
    assert cache.layer_pos_offset(0) == t["expect_pos_offset"]


def test_regression_fixture_matches_oracle(oracle, ref_tests):
    """oracle_regression.json is bit-identical to a fresh oracle run."""
    from tests.golden import make_golden
    with open(os.path.join(GOLDEN, "oracle_regression.json")) as f:
        reg = json.load(f)
    fresh = make_golden.oracle_regression(ref_tests)
    assert fresh["decoder_step_outputs"] == reg["decoder_step_outputs"]
    assert fresh["decoder_step_k"] == reg["decoder_step_k"]
