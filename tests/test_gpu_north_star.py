"""The parity contract of the decoder token loop at the benchmark's own sizes.

1. The full 26-layer decoder (dim 3072, 32/8 heads, head_dim 128, SwiGLU
   9216, untied 131072 x 3072 LM head, window 8192), 256 teacher-forced steps
   from an empty cache: logits within max-abs 2e-2 / relative 1e-2 and the
   greedy argmax identical to the oracle's at EVERY step.  The top-1/top-2
   margin of every step is recorded and the smallest one is reported.
2. The same model decoding greedily on the device (`vox_model_generate`)
   after a prompt prefill, token by token against the oracle's own greedy
   continuation.
3. The rolling-window stress (16384 steps, window 8192, eviction from step
   8193 on) on a narrow model: the device ring state of every layer after
   EVERY step against an index-only restatement of kv.rs:48-88, and logits /
   argmax against the oracle at checkpoints past the first eviction.

The oracle composes the token loop from the reference's layer step
(decoder.rs:88-155): embed row -> layer steps -> final RMSNorm -> LM head ->
argmax, lowest index on ties.
"""
import numpy as np
import pytest

from tests.vox_testlib import (FULL, assert_logits_close, config_dict, kv_index_after_append, oracle_model,
                               top2_margin, vox)

pytestmark = pytest.mark.gpu

N_LAYERS, VOCAB = 26, 131072


@pytest.fixture(scope="module")
def V():
    return vox()


@pytest.fixture(scope="module")
def full_model(V, oracle):
    """The 26-layer decoder on both sides: the oracle's bf16 weights made on
    the host by the generator the device uses (the bytes are identical)."""
    m = oracle_model(oracle, FULL, N_LAYERS, VOCAB, seed=0)
    ctx = V.Context(V.DecoderConfig(**FULL), n_layers=N_LAYERS, vocab=VOCAB)
    ctx.init_random(0, 0.02)
    yield m, ctx
    ctx.close()


def _report(name, text):
    """One line per parity run for the test log (pytest -s shows it)."""
    print(f"[{name}] {text}")


def test_26_layers_256_teacher_forced_steps(V, oracle, full_model):
    m, ctx = full_model
    n_steps = 256
    ids = oracle.gen_uniform_ids(0, 3000010, VOCAB, n_steps)
    oc = oracle.RollingKvCache(N_LAYERS, FULL["n_kv_heads"], FULL["head_dim"], FULL["sliding_window"])
    kv = V.RollingKvCache(ctx, N_LAYERS, FULL["n_kv_heads"], FULL["head_dim"], FULL["sliding_window"])
    worst, margins = 0.0, []
    try:
        for p in range(n_steps):
            tok, logits = ctx.model_step(kv, int(ids[p]), p, want_logits=True)
            ref_logits, ref_tok = m.step(oc, int(ids[p]), p)
            worst = max(worst, assert_logits_close(logits, ref_logits, f"step {p}"))
            margins.append(top2_margin(ref_logits))
            assert tok == ref_tok, f"step {p}: argmax {tok} != oracle {ref_tok} (margin {margins[-1]:.3e})"
        for l in range(N_LAYERS):
            assert kv.layer_len_tokens(l) == oc.layer_len_tokens(l) == n_steps
            assert kv.layer_pos_offset(l) == oc.layer_pos_offset(l) == 0
    finally:
        kv.close()
    mg = np.asarray(margins)
    _report("26x256", f"max |dlogit| {worst:.3e}; top-2 margin min {mg.min():.3e} median {np.median(mg):.3e}; "
                      f"steps with margin < 10x max error: {int(np.sum(mg < 10 * worst))}")
    assert worst < 2e-3


def test_26_layers_greedy_continuation(V, oracle, full_model):
    """Prompt of 32 ids prefilled (positions 0..30), then 64 greedy steps on
    the device from the last prompt id at position 31, token by token against
    the oracle's greedy continuation."""
    m, ctx = full_model
    n_prompt, n_gen = 32, 64
    prompt = oracle.gen_uniform_ids(0, 3000011, VOCAB, n_prompt)
    oc = oracle.RollingKvCache(N_LAYERS, FULL["n_kv_heads"], FULL["head_dim"], FULL["sliding_window"])
    kv = V.RollingKvCache(ctx, N_LAYERS, FULL["n_kv_heads"], FULL["head_dim"], FULL["sliding_window"])
    try:
        ctx.model_prefill(kv, prompt[:n_prompt - 1], 0)
        gen = ctx.model_generate(kv, int(prompt[-1]), n_prompt - 1, n_gen).tolist()
        for p in range(n_prompt - 1):
            m.step(oc, int(prompt[p]), p, want_logits=False)
        tok, ref, margins = int(prompt[-1]), [], []
        for i in range(n_gen):
            logits, tok = m.step(oc, tok, n_prompt - 1 + i)
            ref.append(tok)
            margins.append(top2_margin(logits))
        for i in range(n_gen):
            assert gen[i] == ref[i], (f"greedy step {i}: device {gen[i]} != oracle {ref[i]} "
                                      f"(oracle top-2 margin {margins[i]:.3e})")
        for l in range(N_LAYERS):
            assert kv.layer_len_tokens(l) == oc.layer_len_tokens(l) == n_prompt - 1 + n_gen
    finally:
        kv.close()
    _report("26-greedy", f"{n_gen} greedy tokens identical; top-2 margin min {min(margins):.3e}")


# ---- rolling-window stress (16384 steps, window 8192) -------------------------------

ROLL = config_dict(dim=128, hidden_dim=256, n_heads=4, n_kv_heads=1, head_dim=32, sliding_window=8192,
                   rope_theta=1e6)


def test_rolling_window_16384_steps(V, oracle):
    c, n_layers, vocab, n_steps = ROLL, 2, 4096, 16384
    W = c["sliding_window"]
    checkpoints = {8191, 8192, 8193, 12000, n_steps - 1}   # step indices (0-based)
    ids = oracle.gen_uniform_ids(0, 3000012, vocab, n_steps)
    m = oracle_model(oracle, c, n_layers, vocab, seed=0)
    oc = oracle.RollingKvCache(n_layers, c["n_kv_heads"], c["head_dim"], W)
    sim = [(0, 0, 0)] * n_layers
    with V.Context(V.DecoderConfig(**c), n_layers=n_layers, vocab=vocab, max_positions=n_steps + 8) as ctx:
        ctx.init_random(0, 0.02)
        kv = V.RollingKvCache(ctx, n_layers, c["n_kv_heads"], c["head_dim"], W)
        checked = 0
        for p in range(n_steps):
            want = p in checkpoints
            tok, logits = ctx.model_step(kv, int(ids[p]), p, want_logits=want)
            if want:
                ref_logits, ref_tok = m.step(oc, int(ids[p]), p)
                assert_logits_close(logits, ref_logits, f"rolling step {p}")
                assert tok == ref_tok, f"rolling step {p}: {tok} != {ref_tok} (margin {top2_margin(ref_logits):.3e})"
                checked += 1
            else:
                m.step(oc, int(ids[p]), p, want_logits=False)
            for l in range(n_layers):
                sim[l] = kv_index_after_append(*sim[l], 1, W, W)
                ln, start, off = kv.device_state(l)
                assert (ln, start, off) == sim[l], f"step {p} layer {l}: device {(ln, start, off)} != {sim[l]}"
                assert (kv.layer_len_tokens(l), kv.layer_pos_offset(l)) == (sim[l][0], sim[l][2])
        assert checked == len(checkpoints)
        for l in range(n_layers):
            assert oc.layer_len_tokens(l) == W and oc.layer_pos_offset(l) == n_steps - W
            # ring contents in logical order against the oracle's compacted cache
            kd, vd = kv.layer_tensors(l)
            ko, vo = oc.layer_tensors(l)
            assert kd.shape == ko.shape and vd.shape == vo.shape
            assert float(np.abs(kd - ko).max()) < 1e-4 and float(np.abs(vd - vo).max()) < 1e-4
        kv.close()

