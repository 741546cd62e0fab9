"""GPU parity of the multi-stream step (tensor-core GEMMs, one weight read for
all streams) against the oracle: per-stream logits, greedy tokens and ring
bookkeeping, with caches prefilled from the shared generator."""
import numpy as np
import pytest

from tests.vox_testlib import FULL, assert_logits_close, config_dict, oracle_model, top2_margin, vox

pytestmark = pytest.mark.gpu

KV_ID = 5000000  # generator tensor id of the random cache contents


@pytest.fixture(scope="module")
def V():
    return vox()


def make_ctx(V, c, n_layers, vocab, seed=0, step_mode=0):
    ctx = V.Context(V.DecoderConfig(**c), n_layers=n_layers, vocab=vocab, step_mode=step_mode)
    ctx.init_random(seed, 0.02)
    return ctx


def oracle_cache(oracle, c, n_layers, n_tokens, seed, tensor_id):
    """The oracle cache holding what vox_kv_fill_random writes."""
    oc = oracle.RollingKvCache(n_layers, c["n_kv_heads"], c["head_dim"], c["sliding_window"])
    n = n_tokens * c["n_kv_heads"] * c["head_dim"]
    for l in range(n_layers):
        k = oracle.bf16_to_f32(oracle.gen_normal_bf16(seed, tensor_id + 2 * l, 1.0, n))
        v = oracle.bf16_to_f32(oracle.gen_normal_bf16(seed, tensor_id + 2 * l + 1, 1.0, n))
        oc.layer_set(l, k, v, n_tokens, 0)
    return oc


def run_batch(V, oracle, c, n_layers, vocab, lens, n_steps, seed=0, greedy=False, step_mode=0):
    """Teacher-forced (or greedy) steps of len(lens) streams on both sides."""
    B = len(lens)
    m = oracle_model(oracle, c, n_layers, vocab, seed)
    ids = oracle.gen_uniform_ids(seed, 3000001, vocab, B * n_steps).reshape(n_steps, B)
    worst = 0.0
    with make_ctx(V, c, n_layers, vocab, seed, step_mode) as ctx:
        kv = V.RollingKvCache(ctx, n_layers, c["n_kv_heads"], c["head_dim"], c["sliding_window"], n_streams=B)
        ocs = []
        for s, n in enumerate(lens):
            kv.stream(s).fill_random(n, seed, KV_ID + 100 * s, 1.0)
            ocs.append(oracle_cache(oracle, c, n_layers, n, seed, KV_ID + 100 * s))
        pos = list(lens)
        if greedy:
            got = ctx.model_generate_batch(kv, ids[0], pos, n_steps)
            toks = [int(t) for t in ids[0]]
            for i in range(n_steps):
                for s in range(B):
                    ref_logits, ref_tok = m.step(ocs[s], toks[s], pos[s] + i)
                    assert got[i, s] == ref_tok, (
                        f"step {i} stream {s}: {got[i, s]} != {ref_tok} (margin {top2_margin(ref_logits):.3e})")
                    toks[s] = ref_tok
        else:
            for i in range(n_steps):
                nxt, logits = ctx.model_step_batch(kv, ids[i], [p + i for p in pos], want_logits=True)
                for s in range(B):
                    ref_logits, ref_tok = m.step(ocs[s], int(ids[i, s]), pos[s] + i)
                    worst = max(worst, assert_logits_close(logits[s], ref_logits, f"step {i} stream {s}"))
                    assert nxt[s] == ref_tok, (
                        f"step {i} stream {s}: {nxt[s]} != {ref_tok} (margin {top2_margin(ref_logits):.3e})")
        for s in range(B):
            view = kv.stream(s)
            for l in range(n_layers):
                want = (ocs[s].layer_len_tokens(l), ocs[s].layer_pos_offset(l))
                assert (view.layer_len_tokens(l), view.layer_pos_offset(l)) == want, (s, l)
                ln, start, off = view.device_state(l)
                assert (ln, off) == want, (s, l)
        # New ring entries (k after RoPE, v) against the oracle's cache.
        view = kv.stream(B - 1)
        k, v = view.layer_tensors(n_layers - 1)
        rk, rv = ocs[B - 1].layer_tensors(n_layers - 1)
        assert k.shape == rk.shape
        assert np.max(np.abs(k - rk)) < 1e-3 and np.max(np.abs(v - rv)) < 1e-3
    return worst


@pytest.mark.parametrize("step_mode", [0, 2])
def test_batch_step_three_streams(V, oracle, step_mode):
    """Both ways of launching the GEMMs: one launch per GEMM (default) and one
    persistent chain per layer (VOX_STEP_PERSISTENT)."""
    run_batch(V, oracle, FULL, 3, 8192, [5, 37, 200], 3, step_mode=step_mode)


def test_batch_step_eviction(V, oracle):
    """Window 48: streams prefilled to 46 and 48 tokens evict during the steps
    (kv.rs:48-88), with bit-exact len/pos_offset per stream."""
    c = dict(FULL, sliding_window=48)
    run_batch(V, oracle, c, 2, 4096, [46, 48, 1, 30], 4)
    run_batch(V, oracle, c, 2, 4096, [47, 2], 3, step_mode=2)


def test_batch_small_shapes_and_one_stream(V, oracle):
    c = config_dict(dim=128, hidden_dim=192, n_heads=4, n_kv_heads=2, head_dim=32, sliding_window=64,
                    rope_theta=1e4)
    run_batch(V, oracle, c, 3, 1000, [0, 7], 3)
    run_batch(V, oracle, c, 3, 1000, [9], 2)


def test_batch_greedy_generate(V, oracle):
    run_batch(V, oracle, FULL, 2, 8192, [17, 64, 3, 128, 250, 1, 90, 33], 4, greedy=True)


def test_batch_eight_streams_full_width(V, oracle):
    """The multi-stream workload's layer shapes, vocab 131072 and 8 streams
    with contexts drawn from [256, 4096), on 4 layers."""
    lens = [256 + int(x) for x in oracle.gen_uniform_ids(0, 3000002, 4096 - 256, 8)]
    run_batch(V, oracle, FULL, 4, 131072, lens, 2)


def test_batch_errors(V):
    c = config_dict(dim=128, hidden_dim=192, n_heads=4, n_kv_heads=2, head_dim=32, sliding_window=64)
    with make_ctx(V, c, 2, 500) as ctx:
        kv = V.RollingKvCache(ctx, 2, 2, 32, 64, n_streams=3)
        with pytest.raises(V.VoxError) as e:
            ctx.model_step(kv, 1, 0)  # a multi-stream cache is not a single-stream cache
        assert e.value.code == V.ERR_INVALID_ARG
        with pytest.raises(V.VoxError) as e:
            kv.layer_len_tokens(0)
        assert e.value.code == V.ERR_INVALID_ARG
        view = kv.stream(1)
        with pytest.raises(V.VoxError) as e:
            ctx.model_step_batch(view, [1], [0])  # the batched step takes the whole cache
        assert e.value.code == V.ERR_INVALID_ARG
        with pytest.raises(V.VoxError) as e:
            ctx.model_step_batch(kv, [1, 500, 2], [0, 0, 0])
        assert e.value.code == V.ERR_RANGE
        # a view is an ordinary single-stream cache
        ctx.model_step(view, 3, 0)
        assert view.layer_len_tokens(0) == 1 and kv.stream(0).layer_len_tokens(0) == 0
        with pytest.raises(V.VoxError):
            V.RollingKvCache(ctx, 2, 2, 32, 64, n_streams=9)


def test_batch_greedy_26_layers_subset_of_streams(V, oracle):
    """The multi-stream workload of the benchmark on the full 26-layer model:
    8 streams with caches prefilled to the bench's contexts (uniform in
    [256, 4096) from seed 1000), 64 greedy steps decoded together on the
    device; streams 0 and 5 checked token by token against the oracle's own
    greedy continuation (a subset, as the oracle costs about 0.2 s per token)."""
    c, n_layers, vocab, n_steps = FULL, 26, 131072, 64
    rng = np.random.default_rng(1000)
    lens = [int(x) for x in rng.integers(256, 4096, 8)]
    first = [int(t) for t in rng.integers(0, vocab, 8)]
    m = oracle_model(oracle, c, n_layers, vocab, 0)
    with make_ctx(V, c, n_layers, vocab, 0) as ctx:
        kv = V.RollingKvCache(ctx, n_layers, c["n_kv_heads"], c["head_dim"], c["sliding_window"], n_streams=8)
        for s, n in enumerate(lens):
            kv.stream(s).fill_random(n, 0, KV_ID + 100 * s, 1.0)
        got = ctx.model_generate_batch(kv, first, lens, n_steps)
        kv.close()
    for s in (0, 5):
        oc = oracle_cache(oracle, c, n_layers, lens[s], 0, KV_ID + 100 * s)
        tok, margins = first[s], []
        for i in range(n_steps):
            logits, tok = m.step(oc, tok, lens[s] + i)
            margins.append(top2_margin(logits))
            assert got[i, s] == tok, f"stream {s} step {i}: {got[i, s]} != {tok} (margin {margins[-1]:.3e})"
