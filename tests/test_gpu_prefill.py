"""Batched (tensor-core) prefill against the oracle's token loop.

`vox_model_prefill` runs passes of up to 512 prompt tokens through each layer
at once (dense tcgen05 GEMMs over the pass, causal attention over the cache
plus the pass, keys and values appended at the slots single-token appends
use).  The cache it leaves must be the one n single-token steps of the
reference leave (decoder.rs:88-155 per token, kv.rs:48-88 per append): ring
state bit-exact, keys and values within float tolerance (written below), and
the steps that follow within the logit tolerance with identical argmax.

The oracle side composes the reference's layer step per token: x =
widen(embed[token]) (plus the adapter row for the streaming input), then
decoder_layer_forward_step for every layer; the logits of a prefill are never
computed, as in the reference's prompt loop.
"""
import numpy as np
import pytest

from tests.vox_testlib import (FULL, assert_logits_close, config_dict, kv_index_after_append, oracle_model,
                               top2_margin, vox)

pytestmark = pytest.mark.gpu

# keys / values after a prefill against the oracle's: the pass's linears read
# bf16 hi + lo parts of the f32 activations (about 16 mantissa bits) and sum in
# a different order, so per-element differences stay near 1e-5 of values of
# order 1 at full width; the bound leaves an order of magnitude.
KV_ATOL, KV_RTOL = 2e-3, 2e-3


@pytest.fixture(scope="module")
def V():
    return vox()


def widen(bits):
    return (np.asarray(bits, np.uint16).astype(np.uint32) << 16).view(np.float32)


def oracle_prefill(oracle, m, oc, ids, pos0, adapter=None):
    """n single-token layer steps of the reference (no LM head)."""
    dim = m.cfg.dim
    for i, tok in enumerate(ids):
        x = widen(m.embed[int(tok) * dim:(int(tok) + 1) * dim])
        if adapter is not None:
            x = (adapter[pos0 + i] + x).astype(np.float32)
        for l, lw in enumerate(m.layers):
            x = oracle.decoder_layer_forward_step(m.cfg, l, lw, oc, x, pos0 + i)


def compare_caches(kv, oc, n_layers, what):
    worst = 0.0
    for l in range(n_layers):
        assert kv.layer_len_tokens(l) == oc.layer_len_tokens(l), f"{what} layer {l}: length"
        assert kv.layer_pos_offset(l) == oc.layer_pos_offset(l), f"{what} layer {l}: pos_offset"
        k, v = kv.layer_tensors(l)
        rk, rv = oc.layer_tensors(l)
        for got, ref, name in ((k, rk, "keys"), (v, rv, "values")):
            np.testing.assert_allclose(got, ref, atol=KV_ATOL, rtol=KV_RTOL, err_msg=f"{what} layer {l} {name}")
            if got.size:
                worst = max(worst, float(np.max(np.abs(got.astype(np.float64) - ref))))
    return worst


def check_ring_states(kv, n_layers, n_appended, window, cap, start_state=(0, 0, 0)):
    ln, st, off = start_state
    for _ in range(n_appended):
        ln, st, off = kv_index_after_append(ln, st, off, 1, window, cap)
    for l in range(n_layers):
        assert kv.device_state(l) == (ln, st, off), f"layer {l}: device ring state"
    return ln, st, off


def run_case(V, oracle, c, n_layers, vocab, prompt, steps_after, window=None, calls=None, seed=0):
    """Prefill `prompt` (in the given call sizes) on the device and token by
    token on the oracle, compare the caches, then `steps_after` teacher-forced
    steps with logits.  Returns (max |dkv|, max |dlogit|)."""
    cache_window = window or c["sliding_window"]
    ids = oracle.gen_uniform_ids(seed, 3000100, vocab, prompt + steps_after)
    m = oracle_model(oracle, c, n_layers, vocab, seed)
    oc = oracle.RollingKvCache(n_layers, c["n_kv_heads"], c["head_dim"], cache_window)
    worst_logit = 0.0
    with V.Context(V.DecoderConfig(**c), n_layers=n_layers, vocab=vocab,
                   max_positions=prompt + steps_after + 8) as ctx:
        ctx.init_random(seed, 0.02)
        kv = V.RollingKvCache(ctx, n_layers, c["n_kv_heads"], c["head_dim"], cache_window)
        pos = 0
        for n in calls or [prompt]:
            ctx.model_prefill(kv, ids[pos:pos + n], pos)
            pos += n
        assert pos == prompt
        oracle_prefill(oracle, m, oc, ids[:prompt], 0)
        check_ring_states(kv, n_layers, prompt, cache_window, cache_window)
        worst_kv = compare_caches(kv, oc, n_layers, "after prefill")
        for p in range(prompt, prompt + steps_after):
            tok, logits = ctx.model_step(kv, int(ids[p]), p, want_logits=True)
            ref_logits, ref_tok = m.step(oc, int(ids[p]), p)
            worst_logit = max(worst_logit, assert_logits_close(logits, ref_logits, f"step {p}"))
            assert tok == ref_tok, f"step {p}: {tok} != {ref_tok} (margin {top2_margin(ref_logits):.3e})"
        if steps_after:
            compare_caches(kv, oc, n_layers, "after the steps")
        kv.close()
    print(f"[prefill {prompt} tokens, {n_layers} layers] max |dkv| {worst_kv:.3e}, max |dlogit| {worst_logit:.3e}")
    return worst_kv, worst_logit


def test_full_width_prefill_two_layers(V, oracle):
    """dim 3072 / hidden 9216 / 32:8 heads / head_dim 128, vocab 131072: a
    300-token prompt in one pass, then 6 teacher-forced steps."""
    run_case(V, oracle, FULL, 2, 131072, 300, 6)


NARROW = config_dict(dim=256, hidden_dim=512, n_heads=8, n_kv_heads=2, head_dim=32, sliding_window=4096,
                     rope_theta=1e6)


def test_prefill_two_passes_and_a_second_call(V, oracle):
    """700 tokens in one call (passes of 512 and 188), then 50 more at
    position 700 on the filled cache."""
    run_case(V, oracle, NARROW, 3, 4096, 750, 8, calls=[700, 50])


def test_prefill_evicts_inside_a_pass(V, oracle):
    """Cache window 64 < pass of 300 tokens: the first 236 tokens of the pass
    are evicted by later ones; each token still attends over its own last 64."""
    c = dict(NARROW, sliding_window=64)
    run_case(V, oracle, c, 2, 4096, 300, 12)


def test_prefill_attention_window_below_cache_window(V, oracle):
    """Attention window 48 (the config's) inside a 128-token cache window."""
    c = dict(NARROW, sliding_window=48)
    run_case(V, oracle, c, 2, 4096, 200, 8, window=128)


@pytest.mark.parametrize("heads,head_dim,dim", [((2, 2), 64, 128), ((4, 1), 64, 256), ((3, 3), 64, 192),
                                               ((2, 1), 256, 512), ((4, 4), 32, 128)])
def test_prefill_head_shapes(V, oracle, heads, head_dim, dim):
    nh, nkv = heads
    c = config_dict(dim=dim, hidden_dim=2 * dim, n_heads=nh, n_kv_heads=nkv, head_dim=head_dim,
                    sliding_window=1024, rope_theta=1e4)
    run_case(V, oracle, c, 2, 1024, 77, 4)


def test_prefill_short_prompts_and_one_token(V, oracle):
    """Prompts of 1 (a token step), 2, 17 and 129 tokens in successive calls."""
    run_case(V, oracle, NARROW, 2, 4096, 149, 4, calls=[1, 2, 17, 129])


# 4 q heads per kv head at head_dim 128 take the tensor-core attention
# (32-token blocks, 64-key tiles); the narrow width keeps the oracle fast.
NARROW_G4 = config_dict(dim=512, hidden_dim=1024, n_heads=4, n_kv_heads=1, head_dim=128, sliding_window=4096,
                        rope_theta=1e6)


@pytest.mark.parametrize("window,cache_window,prompt,calls", [
    (4096, None, 750, [700, 50]),      # two passes, then a call on the filled cache
    (64, None, 300, None),             # evictions inside the pass
    (48, 128, 200, None),              # attention window below the cache window
    (4096, None, 149, [1, 2, 17, 129]),  # ragged blocks of 2, 17 and 129 tokens
])
def test_prefill_tensor_core_attention(V, oracle, window, cache_window, prompt, calls):
    c = dict(NARROW_G4, sliding_window=window)
    run_case(V, oracle, c, 2, 4096, prompt, 6, window=cache_window, calls=calls)


@pytest.mark.parametrize("width", ["g4_hd128", "g4_hd32"])
@pytest.mark.parametrize("window,cache_window,prompt,calls", [
    (64, None, 237, [100, 100, 37]),  # each later call reads a ring whose live keys wrap past its end
    (48, 128, 240, [150, 90]),        # wrapped 128-slot ring, attention window 48 inside it
])
def test_prefill_reads_a_wrapped_ring(V, oracle, width, window, cache_window, prompt, calls):
    """Calls after the first read the cache before the pass from a ring whose
    start is not slot 0 (start0 + j runs past the capacity): the tensor-core
    attention (4 q heads per kv head, head_dim 128) and the CUDA-core one."""
    base = NARROW_G4 if width == "g4_hd128" else NARROW
    run_case(V, oracle, dict(base, sliding_window=window), 2, 4096, prompt, 6, window=cache_window, calls=calls)


def test_prefill_matches_token_steps(V):
    """The batched prefill and vox_model_prefill_steps leave the same ring
    state and caches within tolerance (26 layers at full width)."""
    with V.Context(V.DecoderConfig(**FULL), n_layers=26, vocab=131072) as ctx:
        ctx.init_random(0, 0.02)
        ids = np.random.default_rng(1).integers(0, 131072, 96).astype(np.int32)
        a = V.RollingKvCache(ctx, 26, FULL["n_kv_heads"], FULL["head_dim"], FULL["sliding_window"])
        b = V.RollingKvCache(ctx, 26, FULL["n_kv_heads"], FULL["head_dim"], FULL["sliding_window"])
        ctx.model_prefill(a, ids, 0)
        ctx.model_prefill_steps(b, ids, 0)
        worst = 0.0
        for l in range(26):
            assert a.device_state(l) == b.device_state(l)
            ka, va = a.layer_tensors(l)
            kb, vb = b.layer_tensors(l)
            np.testing.assert_allclose(ka, kb, atol=KV_ATOL, rtol=KV_RTOL, err_msg=f"layer {l} keys")
            np.testing.assert_allclose(va, vb, atol=KV_ATOL, rtol=KV_RTOL, err_msg=f"layer {l} values")
            worst = max(worst, float(np.max(np.abs(ka - kb))), float(np.max(np.abs(va - vb))))
        ta = ctx.model_generate(a, int(ids[-1]), 96, 16).tolist()
        tb = ctx.model_generate(b, int(ids[-1]), 96, 16).tolist()
        assert ta == tb
        print(f"[prefill vs token steps, 26 layers] max |dkv| {worst:.3e}")
        a.close()
        b.close()


def test_prefill_range_errors(V):
    c = NARROW
    with V.Context(V.DecoderConfig(**c), n_layers=1, vocab=100, max_positions=64) as ctx:
        ctx.init_random(0, 0.02)
        kv = V.RollingKvCache(ctx, 1, c["n_kv_heads"], c["head_dim"], c["sliding_window"])
        with pytest.raises(V.VoxError):
            ctx.model_prefill(kv, [1, 2, 100], 0)   # token outside the vocabulary
        with pytest.raises(V.VoxError):
            ctx.model_prefill(kv, list(range(10)), 60)  # positions past max_positions
        assert kv.layer_len_tokens(0) == 0
        ctx.model_prefill(kv, list(range(10)), 0)
        assert kv.device_state(0) == (10, 0, 0)
        kv.close()
