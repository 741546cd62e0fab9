"""GPU parity of the decoder layer step (decoder.rs:88-155) and the device
KV ring (kv.rs) against the oracle: outputs within tolerance, ring
bookkeeping bit-exact."""
import json
import os

import numpy as np
import pytest

from tests.golden.make_golden import decoder_test_hidden
from tests.vox_testlib import FULL, config_dict, oracle_layer, vox

pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


@pytest.fixture(scope="module")
def V():
    return vox()


@pytest.fixture(scope="module")
def ref_tests():
    with open(os.path.join(GOLDEN, "reference_unit_tests.json")) as f:
        return json.load(f)


@pytest.fixture(scope="module")
def regression():
    with open(os.path.join(GOLDEN, "oracle_regression.json")) as f:
        return json.load(f)


def rel_err(got, ref):
    return float(np.max(np.abs(got - ref)) / max(np.max(np.abs(ref)), 1e-30))


@pytest.mark.parametrize("weight_dtype", [1, 0])
def test_reference_decoder_step(V, oracle, ref_tests, regression, weight_dtype):
    """decoder.rs:185-214 on the GPU: LCG weights, 6 steps, window 4."""
    t = ref_tests["decoder_step_grows_and_compacts_cache"]
    c = t["config"]
    cfg = V.DecoderConfig(**c)
    w = {k: np.array(v, np.float32) for k, v in t["weights"].items()}
    with V.Context(cfg, weight_dtype=weight_dtype) as ctx:
        ctx.upload_layer(0, w)
        cache = V.RollingKvCache(ctx, 1, c["n_kv_heads"], c["head_dim"], c["sliding_window"])
        if weight_dtype == 1:
            expected = [np.array(o, np.float32) for o in regression["decoder_step_outputs"]]
        else:  # bf16 context rounds the matrices: compare with the oracle on rounded weights
            wr = {k: (oracle.bf16_to_f32(oracle.f32_to_bf16(v)) if k not in ("attention_norm", "ffn_norm")
                      else v) for k, v in w.items()}
            lw = oracle.LayerWeights(wr["attention_norm"], wr["ffn_norm"],
                                     **{n: wr[n] for n in oracle.LayerWeights.NAMES})
            oc = oracle.RollingKvCache(1, c["n_kv_heads"], c["head_dim"], c["sliding_window"])
            ocfg = oracle.config(**c)
            expected = [oracle.decoder_layer_forward_step(ocfg, 0, lw, oc, decoder_test_hidden(p, c["dim"]), p)
                        for p in range(t["steps"])]
        for pos in range(t["steps"]):
            out = V.decoder_layer_forward_step(ctx, 0, cache, decoder_test_hidden(pos, c["dim"]), pos)
            assert out.shape == (c["dim"],) and np.all(np.isfinite(out))
            assert np.max(np.abs(out - expected[pos])) < 1e-5
        assert cache.layer_len_tokens(0) == t["expect_len"]
        assert cache.layer_pos_offset(0) == t["expect_pos_offset"]
        ln, start, off = cache.device_state(0)
        assert (ln, off) == (t["expect_len"], t["expect_pos_offset"])
        if weight_dtype == 1:
            k, v = cache.layer_tensors(0)
            assert np.max(np.abs(k - np.array(regression["decoder_step_k"], np.float32))) < 1e-5
            assert np.max(np.abs(v - np.array(regression["decoder_step_v"], np.float32))) < 1e-5


def test_decoder_step_errors(V):
    c = config_dict(dim=8, hidden_dim=16, n_heads=2, n_kv_heads=1, head_dim=4, sliding_window=4)
    with V.Context(V.DecoderConfig(**c)) as ctx:
        cache = V.RollingKvCache(ctx, 1, 1, 4, 4)
        with pytest.raises(V.VoxError) as e:   # weights never uploaded (decoder.rs:97)
            V.decoder_layer_forward_step(ctx, 0, cache, np.zeros(8, np.float32), 0)
        assert e.value.code == V.ERR_NOT_READY
        ctx.init_random(1)
        with pytest.raises(V.VoxError) as e:   # decoder.rs:98
            V.decoder_layer_forward_step(ctx, 0, cache, np.zeros(7, np.float32), 0)
        assert e.value.code == V.ERR_SHAPE and e.value.message == "hidden size mismatch"
        wrong = V.RollingKvCache(ctx, 1, 2, 4, 4)
        with pytest.raises(V.VoxError):
            V.decoder_layer_forward_step(ctx, 0, wrong, np.zeros(8, np.float32), 0)


def run_layer_parity(V, oracle, c, steps, window, capacity=None, check_every=1, seed=0):
    """Single layer, fresh N(0,1) hidden every step (config 0's input)."""
    cfg = V.DecoderConfig(**c)
    lw = oracle_layer(oracle, c, 0, seed=seed)
    ocfg = oracle.config(**c)
    oc = oracle.RollingKvCache(1, c["n_kv_heads"], c["head_dim"], window)
    worst = 0.0
    with V.Context(cfg, n_layers=1) as ctx:
        ctx.init_random(seed)
        cache = V.RollingKvCache(ctx, 1, c["n_kv_heads"], c["head_dim"], window, capacity)
        for pos in range(steps):
            hidden = oracle.gen_normal_f32(seed, 2000000 + pos, 1.0, c["dim"])
            got = V.decoder_layer_forward_step(ctx, 0, cache, hidden, pos)
            ref = oracle.decoder_layer_forward_step(ocfg, 0, lw, oc, hidden, pos)
            worst = max(worst, rel_err(got, ref))
            assert cache.layer_len_tokens(0) == oc.layer_len_tokens(0)
            assert cache.layer_pos_offset(0) == oc.layer_pos_offset(0)
            if pos % check_every == 0 or pos == steps - 1:
                ln, start, off = cache.device_state(0)
                assert ln == oc.layer_len_tokens(0) and off == oc.layer_pos_offset(0)
                assert start == oc.layer_pos_offset(0) % (capacity or window)
        k, v = cache.layer_tensors(0)
        rk, rv = oc.layer_tensors(0)
        assert k.shape == rk.shape
        assert rel_err(k, rk) < 1e-5 and rel_err(v, rv) < 1e-5
    return worst


def test_config0_layer_256_steps(V, oracle):
    """Full layer shapes (dim 3072, 32/8 heads, hd 128, hidden 9216, theta 1e6),
    256 steps from an empty cache, window 8192."""
    worst = run_layer_parity(V, oracle, FULL, 256, 8192, check_every=32)
    assert worst < 1e-4, worst


def test_full_shape_layer_eviction(V, oracle):
    """Same shapes with a 24-token window: eviction starts at step 25 and the
    ring start wraps; indices stay bit-exact, outputs within tolerance."""
    worst = run_layer_parity(V, oracle, FULL, 70, 24)
    assert worst < 1e-4, worst


def test_kv_reference_tests_on_device(V, ref_tests):
    c = config_dict(dim=8, hidden_dim=16, n_heads=2, n_kv_heads=1, head_dim=4, sliding_window=4)
    with V.Context(V.DecoderConfig(**c)) as ctx:
        t = ref_tests["compacts_when_exceeding_window"]  # kv.rs:109-136
        kv = V.RollingKvCache(ctx, t["n_layers"], t["n_kv_heads"], t["head_dim"], t["window"])
        for a in t["appends"]:
            kv.append_layer(0, a["k"], a["v"], a["n"])
            assert kv.layer_len_tokens(0) == a["expect_len"]
            assert kv.layer_pos_offset(0) == a["expect_pos_offset"]
        k, v = kv.layer_tensors(0)
        stride = t["n_kv_heads"] * t["head_dim"]
        assert k.size == 4 * stride
        assert k[0] == t["expect_k_first"] and v[0] == t["expect_v_first"]
        assert k[3 * stride] == t["expect_k_last"] and v[3 * stride] == t["expect_v_last"]

        t = ref_tests["layers_are_isolated"]  # kv.rs:139-151
        kv = V.RollingKvCache(ctx, t["n_layers"], t["n_kv_heads"], t["head_dim"], t["window"])
        for a in t["appends"]:
            kv.append_layer(a["layer"], a["k"], a["v"], a["n"])
        for layer in range(2):
            assert kv.layer_len_tokens(layer) == t["expect_len"][layer]
            assert kv.layer_tensors(layer)[0].tolist() == t["expect_k"][layer]


def test_kv_append_sequences_match_oracle(V, oracle):
    """Random append sizes, including appends larger than the window (which
    the reference keeps whole, kv.rs:64-74) into a ring with spare capacity."""
    c = config_dict(dim=8, hidden_dim=16, n_heads=2, n_kv_heads=1, head_dim=4, sliding_window=4)
    rng = np.random.default_rng(11)
    with V.Context(V.DecoderConfig(**c)) as ctx:
        for window in (1, 3, 5):
            cap = window + 6
            kv = V.RollingKvCache(ctx, 2, 2, 3, window, capacity=cap)
            ok = oracle.RollingKvCache(2, 2, 3, window)
            counter = 0
            for step in range(50):
                layer = int(rng.integers(0, 2))
                n = int(rng.integers(0, window + 7)) if step % 9 == 0 else int(rng.integers(0, 3))
                k = np.arange(counter, counter + n * 6, dtype=np.float32)
                counter += n * 6
                kv.append_layer(layer, k, -k, n)
                ok.append_layer(layer, k, -k, n)
                for l in range(2):
                    assert kv.layer_len_tokens(l) == ok.layer_len_tokens(l)
                    assert kv.layer_pos_offset(l) == ok.layer_pos_offset(l)
                    gk, gv = kv.layer_tensors(l)
                    rk, rv = ok.layer_tensors(l)
                    assert np.array_equal(gk, rk) and np.array_equal(gv, rv)
            with pytest.raises(V.VoxError) as e:
                kv.append_layer(0, np.zeros((cap + 1) * 6), np.zeros((cap + 1) * 6), cap + 1)
            assert e.value.code == V.ERR_UNSUPPORTED
