"""CPU checks of the oracle beyond the reference's own tests: config
validation order, window-eviction index arithmetic, masking, the composed
token loop, threading invariance, and the seeded data generator."""
import numpy as np
import pytest


def cfg_of(o, **kw):
    base = dict(dim=8, hidden_dim=16, n_heads=2, n_kv_heads=1, head_dim=4,
                sliding_window=4, norm_eps=1e-5, rope_theta=1e4)
    base.update(kw)
    return o.config(**base)


@pytest.mark.parametrize("field,value,code", [
    ("dim", 0, 1), ("hidden_dim", 0, 2), ("n_heads", 0, 3), ("n_kv_heads", 0, 4),
    ("head_dim", 0, 5), ("n_kv_heads", 3, 6), ("head_dim", 2, 7), ("sliding_window", 0, 8),
])
def test_config_validate_codes(oracle, field, value, code):
    # decoder.rs:22-41, checked in source order
    assert oracle.config_validate(cfg_of(oracle, **{field: value})) == code
    assert oracle.config_validate(cfg_of(oracle)) == 0


def expected_state(appends, window):
    """Closed form of kv.rs:48-88 bookkeeping, step by step."""
    length, off = 0, 0
    for n in appends:
        if n == 0:
            continue
        drop = max(0, length + n - window)
        if drop:
            keep = max(0, length - drop)
            length = keep
            off += drop
        length += n
    return length, off


@pytest.mark.parametrize("window", [1, 3, 8])
def test_kv_eviction_indices(oracle, window):
    rng = np.random.default_rng(window)
    stride = 3
    kv = oracle.RollingKvCache(1, 1, stride, window)
    appended = []  # every token ever appended, as its first k element
    hist = []
    for step in range(60):
        n = int(rng.integers(0, 4)) if step % 7 else int(rng.integers(window, window + 3))
        k = np.arange(len(appended), len(appended) + n, dtype=np.float32).repeat(stride)
        kv.append_layer(0, k, -k, n)
        appended.extend(range(len(appended), len(appended) + n))
        hist.append(n)
        length, off = expected_state(hist, window)
        assert kv.layer_len_tokens(0) == length
        assert kv.layer_pos_offset(0) == off
        kk, vv = kv.layer_tensors(0)
        # contents are always the most recent `length` tokens, in order
        assert kk[::stride].tolist() == [float(a) for a in appended[len(appended) - length:]]
        assert np.array_equal(vv, -kk)


def test_attention_window_masks_oldest(oracle):
    rng = np.random.default_rng(0)
    nh, nkv, hd, seq, win = 4, 2, 8, 9, 5
    q = rng.standard_normal(nh * hd).astype(np.float32)
    k = rng.standard_normal(seq * nkv * hd).astype(np.float32)
    v = rng.standard_normal(seq * nkv * hd).astype(np.float32)
    full = oracle.attention_gqa_step(q, k, v, nh, hd, seq, nkv, win)
    tail = oracle.attention_gqa_step(q, k[(seq - win) * nkv * hd:], v[(seq - win) * nkv * hd:],
                                     nh, hd, win, nkv, 0)
    assert np.max(np.abs(full - tail)) < 1e-6


def test_linear_threads_bit_identical(oracle):
    rng = np.random.default_rng(1)
    x = rng.standard_normal(300).astype(np.float32)
    w = rng.standard_normal(300 * 257).astype(np.float32)
    oracle.set_threads(1)
    a = oracle.linear(x, 1, 300, w, 257)
    oracle.set_threads(4)
    b = oracle.linear(x, 1, 300, w, 257)
    assert np.array_equal(a, b)
    ref = (w.reshape(257, 300).astype(np.float64) @ x.astype(np.float64))
    assert np.max(np.abs(a - ref)) < 1e-3


def test_linear_bf16_equals_widened_f32(oracle):
    rng = np.random.default_rng(2)
    x = rng.standard_normal(64).astype(np.float32)
    wb = oracle.gen_normal_bf16(0, 77, 0.02, 64 * 33)
    a = oracle.linear_bf16(x, 1, 64, wb, 33)
    b = oracle.linear(x, 1, 64, oracle.bf16_to_f32(wb), 33)
    assert np.array_equal(a, b)


def test_generator_deterministic_and_normal(oracle):
    a = oracle.gen_normal_f32(0, 5, 1.0, 200000)
    b = oracle.gen_normal_f32(0, 5, 1.0, 1000, first=500)
    assert np.array_equal(a[500:1500], b)
    assert abs(float(a.mean())) < 0.01 and abs(float(a.std()) - 1.0) < 0.01
    c = oracle.gen_normal_f32(1, 5, 1.0, 1000)
    assert not np.array_equal(a[:1000], c)
    bits = oracle.gen_normal_bf16(0, 5, 0.02, 1000)
    assert np.array_equal(bits, oracle.f32_to_bf16(a[:1000] * np.float32(0.02)))
    ids = oracle.gen_uniform_ids(0, 9, 131072, 100000)
    assert ids.min() >= 0 and ids.max() < 131072
    assert abs(float(ids.mean()) / 131072 - 0.5) < 0.01


def make_mini_model(o, seed=0, n_layers=2, vocab=64, **kw):
    cfg = cfg_of(o, **kw)
    layers = []
    dims = dict(wq=(cfg.n_heads * cfg.head_dim, cfg.dim), wk=(cfg.n_kv_heads * cfg.head_dim, cfg.dim),
                wv=(cfg.n_kv_heads * cfg.head_dim, cfg.dim), wo=(cfg.dim, cfg.n_heads * cfg.head_dim),
                w1=(cfg.hidden_dim, cfg.dim), w2=(cfg.dim, cfg.hidden_dim), w3=(cfg.hidden_dim, cfg.dim))
    for l in range(n_layers):
        mats = {n: o.gen_normal_bf16(seed, 16 * l + i + 1, 0.2, r * c)
                for i, (n, (r, c)) in enumerate(dims.items())}
        layers.append(o.LayerWeights(np.ones(cfg.dim, np.float32), np.ones(cfg.dim, np.float32), **mats))
    emb = o.gen_normal_bf16(seed, 1000, 0.5, vocab * cfg.dim)
    head = o.gen_normal_bf16(seed, 1001, 0.5, vocab * cfg.dim)
    return cfg, o.Model(cfg, layers, emb, np.ones(cfg.dim, np.float32), head, vocab)


def test_model_step_composes_layer_steps(oracle):
    cfg, m = make_mini_model(oracle)
    cache = oracle.RollingKvCache(2, cfg.n_kv_heads, cfg.head_dim, cfg.sliding_window)
    cache2 = oracle.RollingKvCache(2, cfg.n_kv_heads, cfg.head_dim, cfg.sliding_window)
    toks = [3, 17, 5, 60, 2, 9]
    for pos, t in enumerate(toks):
        logits, am = m.step(cache, t, pos)
        x = oracle.bf16_to_f32(m.embed[t * cfg.dim:(t + 1) * cfg.dim])
        for l in range(2):
            x = oracle.decoder_layer_forward_step(cfg, l, m.layers[l], cache2, x, pos)
        xn = oracle.rms_norm_rows(x, m.final_norm, cfg.dim, cfg.norm_eps)
        ref = oracle.linear_bf16(xn, 1, cfg.dim, m.lm_head, 64)
        assert np.array_equal(logits, ref)
        assert am == int(np.argmax(ref))
    assert cache.layer_len_tokens(1) == 4 and cache.layer_pos_offset(1) == 2


def test_kv_index_simulation_matches_oracle_cache(oracle):
    """The index-only restatement of kv.rs:48-88 used by the 16384-step device
    test agrees with the oracle's kv.rs port on random append sequences."""
    from tests.vox_testlib import kv_index_after_append
    rng = np.random.default_rng(5)
    W = 7
    oc = oracle.RollingKvCache(1, 1, 2, W)
    s = (0, 0, 0)
    for _ in range(300):
        n = int(rng.integers(0, 10))
        oc.append_layer(0, np.zeros(n * 2, np.float32), np.zeros(n * 2, np.float32), n)
        s = kv_index_after_append(*s, n, W, 64)
        assert (s[0], s[2]) == (oc.layer_len_tokens(0), oc.layer_pos_offset(0))
    # single-token appends over 3 windows: the ring start is pos_offset mod window
    s = (0, 0, 0)
    for i in range(3 * W):
        s = kv_index_after_append(*s, 1, W, W)
        assert s == (min(i + 1, W), max(0, i + 1 - W) % W, max(0, i + 1 - W))
