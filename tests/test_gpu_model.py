"""GPU parity of the composed token loop (embed -> layers -> final RMSNorm ->
LM head -> argmax) against the oracle, plus the seeded weight generator."""
import numpy as np
import pytest

from tests.vox_testlib import (EMBED_ID, FULL, HEAD_ID, MATS, assert_logits_close, config_dict,
                               mat_shapes, oracle_model, top2_margin, vox)

pytestmark = pytest.mark.gpu

MINI = config_dict(dim=64, hidden_dim=128, n_heads=4, n_kv_heads=2, head_dim=16, sliding_window=8,
                   rope_theta=1e4)


@pytest.fixture(scope="module")
def V():
    return vox()


def make_ctx(V, c, n_layers, vocab, seed=0, weight_dtype=0, step_mode=0):
    ctx = V.Context(V.DecoderConfig(**c), n_layers=n_layers, vocab=vocab, weight_dtype=weight_dtype,
                    step_mode=step_mode)
    ctx.init_random(seed, 0.02)
    return ctx


def test_generator_bit_exact(V, oracle):
    """vox_ctx_init_random writes the oracle generator's bytes."""
    vocab = 512
    with make_ctx(V, MINI, 2, vocab, seed=7) as ctx:
        shapes = mat_shapes(MINI)
        for layer in range(2):
            for i, n in enumerate(MATS):
                r, k = shapes[n]
                ref = oracle.gen_normal_bf16(7, 16 * layer + i + 1, 0.02, r * k)
                assert np.array_equal(ctx.download_matrix(layer, n), ref), (layer, n)
        assert np.array_equal(ctx.download_matrix(0, "embed"),
                              oracle.gen_normal_bf16(7, EMBED_ID, 0.02, vocab * MINI["dim"]))
        assert np.array_equal(ctx.download_matrix(0, "lm_head"),
                              oracle.gen_normal_bf16(7, HEAD_ID, 0.02, vocab * MINI["dim"]))
    with make_ctx(V, MINI, 1, 0, seed=3, weight_dtype=1) as ctx:
        ref = oracle.gen_normal_f32(3, 5, 0.02, 128 * 64)
        assert np.array_equal(ctx.download_matrix(0, "w1"), ref)


def test_generator_full_layer_bit_exact(V, oracle):
    with make_ctx(V, FULL, 1, 0, seed=0) as ctx:
        for i, n in enumerate(MATS):
            r, k = mat_shapes(FULL)[n]
            ref = oracle.gen_normal_bf16(0, i + 1, 0.02, r * k)
            assert np.array_equal(ctx.download_matrix(0, n), ref), n


def teacher_forced(V, oracle, c, n_layers, vocab, n_steps, window=None, seed=0, prefill=0, step_mode=0):
    """Run n_steps teacher-forced steps on both sides; returns (max diff, margins)."""
    if window is not None:
        c = dict(c, sliding_window=window)
    ids = oracle.gen_uniform_ids(seed, 3000000, vocab, n_steps)
    m = oracle_model(oracle, c, n_layers, vocab, seed)
    oc = oracle.RollingKvCache(n_layers, c["n_kv_heads"], c["head_dim"], c["sliding_window"])
    worst, margins = 0.0, []
    with make_ctx(V, c, n_layers, vocab, seed, step_mode=step_mode) as ctx:
        kv = V.RollingKvCache(ctx, n_layers, c["n_kv_heads"], c["head_dim"], c["sliding_window"])
        if prefill:
            ctx.model_prefill(kv, ids[:prefill], 0)
            for p in range(prefill):
                m.step(oc, int(ids[p]), p, want_logits=False)
        for p in range(prefill, n_steps):
            tok, logits = ctx.model_step(kv, int(ids[p]), p, want_logits=True)
            ref_logits, ref_tok = m.step(oc, int(ids[p]), p)
            worst = max(worst, assert_logits_close(logits, ref_logits, f"step {p}"))
            margins.append(top2_margin(ref_logits))
            assert tok == ref_tok, f"step {p}: argmax {tok} != oracle {ref_tok} (margin {margins[-1]:.3e})"
            assert tok == int(np.argmax(logits))
        for l in range(n_layers):
            assert kv.layer_len_tokens(l) == oc.layer_len_tokens(l)
            assert kv.layer_pos_offset(l) == oc.layer_pos_offset(l)
            ln, start, off = kv.device_state(l)
            assert (ln, off) == (oc.layer_len_tokens(l), oc.layer_pos_offset(l))
    return worst, margins


# step_mode 1 (the chain of per-layer kernels, the default); 2 selects the
# multi-stream persistent GEMM chain and leaves single-stream steps unchanged.
MODES = [1, 2]


@pytest.mark.parametrize("step_mode", MODES)
def test_mini_model_with_eviction(V, oracle, step_mode):
    worst, _ = teacher_forced(V, oracle, MINI, 3, 1000, 40, prefill=5, step_mode=step_mode)
    assert worst < 1e-4


@pytest.mark.parametrize("step_mode", MODES)
def test_full_width_two_layers(V, oracle, step_mode):
    """dim 3072 / hidden 9216 / 32:8 heads / vocab 131072, 2 layers."""
    worst, margins = teacher_forced(V, oracle, FULL, 2, 131072, 24, prefill=8, step_mode=step_mode)
    assert worst < 1e-3


@pytest.mark.parametrize("step_mode", MODES)
def test_full_width_eviction(V, oracle, step_mode):
    """Full shapes with a 16-token window: 40 steps, eviction from step 17."""
    worst, _ = teacher_forced(V, oracle, FULL, 2, 131072, 40, window=16, prefill=10, step_mode=step_mode)
    assert worst < 1e-3


def test_argmax_identical_256_teacher_forced_steps(V, oracle):
    """256 teacher-forced steps, full-width 4-layer model, full vocabulary:
    greedy argmax identical at every step."""
    worst, margins = teacher_forced(V, oracle, FULL, 4, 131072, 256)
    assert worst < 1e-3


def test_full_26_layer_token_loop(V, oracle):
    """The full 26-layer decoder with embedding and untied LM head."""
    worst, _ = teacher_forced(V, oracle, FULL, 26, 131072, 6, prefill=2)
    assert worst < 1e-3


@pytest.mark.parametrize("step_mode", MODES)
def test_generate_matches_stepwise_greedy(V, step_mode):
    with make_ctx(V, MINI, 2, 1000, seed=2, step_mode=step_mode) as ctx:
        kv1 = V.RollingKvCache(ctx, 2, 2, 16, 8)
        kv2 = V.RollingKvCache(ctx, 2, 2, 16, 8)
        ctx.model_prefill(kv1, [1, 2, 3], 0)
        ctx.model_prefill(kv2, [1, 2, 3], 0)
        gen = ctx.model_generate(kv1, 4, 3, 30)
        tok, toks = 4, []
        for i in range(30):
            tok, _ = ctx.model_step(kv2, tok, 3 + i)
            toks.append(tok)
        assert gen.tolist() == toks
        assert kv1.layer_len_tokens(1) == kv2.layer_len_tokens(1) == 8
        assert kv1.layer_pos_offset(0) == 33 - 8


def test_model_step_range_errors(V):
    with make_ctx(V, MINI, 1, 100) as ctx:
        kv = V.RollingKvCache(ctx, 1, 2, 16, 8)
        with pytest.raises(V.VoxError) as e:
            ctx.model_step(kv, 100, 0)
        assert e.value.code == V.ERR_RANGE
        with pytest.raises(V.VoxError) as e:
            ctx.model_step(kv, 0, 1 << 20)
        assert e.value.code == V.ERR_RANGE


@pytest.mark.parametrize("step_mode", MODES)
def test_full_window_rolling_eviction(V, oracle, step_mode):
    """Rolling-window stress at the full window: the cache holds 8190 of 8192
    tokens (filled from the generator on both sides), then teacher-forced
    steps run through the first evictions; logits, argmax and the ring state
    (len, pos_offset, physical start) are checked after every step."""
    c, n_layers, vocab, fill, n_steps = FULL, 4, 8192, 8190, 6
    m = oracle_model(oracle, c, n_layers, vocab, 0)
    oc = oracle.RollingKvCache(n_layers, c["n_kv_heads"], c["head_dim"], c["sliding_window"])
    n = fill * c["n_kv_heads"] * c["head_dim"]
    for l in range(n_layers):
        k = oracle.bf16_to_f32(oracle.gen_normal_bf16(0, 5000000 + 2 * l, 1.0, n))
        v = oracle.bf16_to_f32(oracle.gen_normal_bf16(0, 5000000 + 2 * l + 1, 1.0, n))
        oc.layer_set(l, k, v, fill, 0)
    ids = oracle.gen_uniform_ids(0, 3000003, vocab, n_steps)
    with make_ctx(V, c, n_layers, vocab, 0, step_mode=step_mode) as ctx:
        kv = V.RollingKvCache(ctx, n_layers, c["n_kv_heads"], c["head_dim"], c["sliding_window"])
        kv.fill_random(fill, 0, 5000000, 1.0)
        for i in range(n_steps):
            pos = fill + i
            tok, logits = ctx.model_step(kv, int(ids[i]), pos, want_logits=True)
            ref_logits, ref_tok = m.step(oc, int(ids[i]), pos)
            assert_logits_close(logits, ref_logits, f"step {i}")
            assert tok == ref_tok, f"step {i}: {tok} != {ref_tok} (margin {top2_margin(ref_logits):.3e})"
            want_len, want_off = oc.layer_len_tokens(0), oc.layer_pos_offset(0)
            assert (kv.layer_len_tokens(0), kv.layer_pos_offset(0)) == (want_len, want_off)
            ln, start, off = kv.device_state(n_layers - 1)
            # the ring starts at slot 0 and drops `off` tokens in all: start = off mod window
            assert (ln, off, start) == (want_len, want_off, want_off % c["sliding_window"])
        assert oc.layer_pos_offset(0) == fill + n_steps - c["sliding_window"] > 0


@pytest.mark.parametrize("fill", [3581, 5000])
def test_attention_kernel_switch(V, oracle, fill):
    """Single-stream steps run attention as one thread-block cluster per kv
    head up to 3584 live tokens (kAttnClusterMaxTokens) and as the split-K
    kernel above it: teacher-forced steps across the switch (3582 -> 3587
    tokens) and above it, against the oracle; generate and step agree."""
    c, n_layers, vocab, n_steps = FULL, 2, 8192, 6
    m = oracle_model(oracle, c, n_layers, vocab, 0)
    oc = oracle.RollingKvCache(n_layers, c["n_kv_heads"], c["head_dim"], c["sliding_window"])
    n = fill * c["n_kv_heads"] * c["head_dim"]
    for l in range(n_layers):
        k = oracle.bf16_to_f32(oracle.gen_normal_bf16(0, 5000000 + 2 * l, 1.0, n))
        v = oracle.bf16_to_f32(oracle.gen_normal_bf16(0, 5000000 + 2 * l + 1, 1.0, n))
        oc.layer_set(l, k, v, fill, 0)
    ids = oracle.gen_uniform_ids(0, 3000004, vocab, n_steps)
    with make_ctx(V, c, n_layers, vocab, 0) as ctx:
        kv = V.RollingKvCache(ctx, n_layers, c["n_kv_heads"], c["head_dim"], c["sliding_window"])
        kv.fill_random(fill, 0, 5000000, 1.0)
        for i in range(n_steps):
            pos = fill + i
            tok, logits = ctx.model_step(kv, int(ids[i]), pos, want_logits=True)
            ref_logits, ref_tok = m.step(oc, int(ids[i]), pos)
            assert_logits_close(logits, ref_logits, f"step {i}")
            assert tok == ref_tok, f"step {i}: {tok} != {ref_tok} (margin {top2_margin(ref_logits):.3e})"
        # greedy generate across the switch equals step-by-step greedy
        kv2 = V.RollingKvCache(ctx, n_layers, c["n_kv_heads"], c["head_dim"], c["sliding_window"])
        kv3 = V.RollingKvCache(ctx, n_layers, c["n_kv_heads"], c["head_dim"], c["sliding_window"])
        kv2.fill_random(fill, 0, 5000000, 1.0)
        kv3.fill_random(fill, 0, 5000000, 1.0)
        gen = ctx.model_generate(kv2, int(ids[0]), fill, n_steps)
        tok, toks = int(ids[0]), []
        for i in range(n_steps):
            tok, _ = ctx.model_step(kv3, tok, fill + i)
            toks.append(tok)
        assert gen.tolist() == toks
