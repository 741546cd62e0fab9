"""GPU parity of the streaming decode driver (vox_pipeline_*): adapter rows
pushed in chunks, decode gated by PipelineState (pipeline.rs:28-90), the
first decode prefilling the [BOS] + [STREAMING_PAD]* prompt with
adapter[p] + tok_embed(prompt[p]) and every later position feeding
adapter[p] + tok_embed(previous token) (docs/plans/2026-02-11-voxtral-rust-design.md:40-46),
against the oracle's composition of the same schedule over the reference's
layer step."""
import numpy as np
import pytest

from tests.vox_testlib import FULL, config_dict, oracle_model, vox

pytestmark = pytest.mark.gpu

MINI = config_dict(dim=64, hidden_dim=128, n_heads=4, n_kv_heads=2, head_dim=16, sliding_window=24,
                   rope_theta=1e4)


@pytest.fixture(scope="module")
def V():
    return vox()


def run_pipeline(V, oracle, c, n_layers, vocab, chunks, prompt_cfg, capacity=4096, seed=0):
    """Push adapter rows in `chunks`, decode after each push, compare every
    decoded token with the oracle's streaming schedule; returns the tokens."""
    total = sum(chunks)
    adapter = oracle.gen_normal_f32(seed, 4000000, 0.02, total * c["dim"]).reshape(total, c["dim"])
    m = oracle_model(oracle, c, n_layers, vocab, seed)
    oc = oracle.RollingKvCache(n_layers, c["n_kv_heads"], c["head_dim"], c["sliding_window"])
    pc = V.PipelineConfig(1, 3, 1280, V.StreamPromptConfig(*prompt_cfg))
    got = []
    with V.Context(V.DecoderConfig(**c), n_layers=n_layers, vocab=vocab) as ctx:
        ctx.init_random(seed, 0.02)
        kv = V.RollingKvCache(ctx, n_layers, c["n_kv_heads"], c["head_dim"], c["sliding_window"])
        with V.PipelineState(pc, ctx, kv, adapter_capacity=capacity) as st:
            prompt = st.prompt_ids()
            pushed = 0
            for n in chunks:
                st.push_adapter_tokens(adapter[pushed:pushed + n])
                pushed += n
                want_n = st.decodable_now()
                toks = st.decode()
                assert len(toks) == want_n
                ref = m.stream_decode(oc, prompt, adapter, len(toks), generated=got)
                assert toks.tolist() == ref, (pushed, toks.tolist(), ref)
                got.extend(ref)
                assert st.decodable_now() == 0
            assert st.generated_tokens() == len(got) == V.decodable_token_budget(total, len(prompt))
            for l in range(n_layers):
                assert kv.layer_len_tokens(l) == oc.layer_len_tokens(l)
                assert kv.layer_pos_offset(l) == oc.layer_pos_offset(l)
        kv.close()
    return got


def test_streaming_pipeline_mini_model_with_eviction(V, oracle):
    """Prompt of 1 + 4 + 2 ids, window 24: pushes of 3, 5, 1, 9, 30 positions;
    decoding starts at the 7th position and runs past the window."""
    toks = run_pipeline(V, oracle, MINI, 3, 1000, [3, 5, 1, 9, 30], (4, 2, 10))
    assert len(toks) == 48 - 7 + 1


def test_streaming_pipeline_full_width(V, oracle):
    """dim 3072 / 32:8 heads / vocab 131072, 2 layers, the default prompt
    (1 + 32 + 6 ids) and 80-ms-chunk-like pushes."""
    toks = run_pipeline(V, oracle, FULL, 2, 131072, [20, 19, 10, 7, 8], (32, 6, 10))
    assert len(toks) == 64 - 39 + 1


def test_streaming_pipeline_ring_wraps(V, oracle):
    """A 12-position adapter ring (prompt of 7): pushes wrap it several times."""
    run_pipeline(V, oracle, MINI, 2, 500, [7, 5, 4, 12, 3, 11], (4, 2, 10), capacity=12)


def test_streaming_pipeline_errors(V):
    with V.Context(V.DecoderConfig(**MINI), n_layers=1, vocab=100) as ctx:
        ctx.init_random(0, 0.02)
        kv = V.RollingKvCache(ctx, 1, 2, 16, 24)
        pc = V.PipelineConfig(1, 3, 1280, V.StreamPromptConfig(4, 2, 10))
        with pytest.raises(V.VoxError) as e:   # capacity below the prompt length
            V.PipelineState(pc, ctx, kv, adapter_capacity=6)
        assert e.value.code == V.ERR_INVALID_ARG
        with pytest.raises(V.VoxError) as e:   # prompt ids outside the vocabulary
            V.PipelineState(V.PipelineConfig(1, 300, 1280, V.StreamPromptConfig(4, 2, 10)), ctx, kv)
        assert e.value.code == V.ERR_RANGE
        with V.PipelineState(pc, ctx, kv, adapter_capacity=8) as st:
            rows = np.zeros((8, 64), np.float32)
            st.push_adapter_tokens(rows)
            with pytest.raises(V.VoxError) as e:   # would overwrite positions not yet decoded
                st.push_adapter_tokens(rows[:1])
            assert e.value.code == V.ERR_RANGE
            with pytest.raises(V.VoxError) as e:   # a decoding pipeline marks its own tokens
                st.mark_decoded(1)
            assert e.value.code == V.ERR_INVALID_ARG
            assert len(st.decode()) == 2
            st.push_adapter_tokens(rows[:7])        # positions 0..7 are enqueued: room for 7 more
        kv.close()
