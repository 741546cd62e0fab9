"""The streaming schedule (stream.rs, pipeline.rs) on the host: the reference's
own unit tests (inputs and expected values in tests/golden/) run against the
oracle port and against the library's C ABI (a pipeline without a context is
the reference's planner), and the two agree on random push/decode sequences.
No GPU is needed."""
import json
import os

import numpy as np
import pytest

from tests.vox_testlib import vox

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


@pytest.fixture(scope="module")
def ref_tests():
    with open(os.path.join(GOLDEN, "reference_unit_tests.json")) as f:
        return json.load(f)


@pytest.fixture(scope="module")
def V():
    return vox()


def _oracle_side(oracle):
    return dict(cfg=lambda p: oracle.stream_prompt_config(**p), prompt=oracle.stream_build_prompt_ids,
                ready=oracle.stream_decode_ready, budget=oracle.stream_decodable_token_budget,
                pad=oracle.stream_finish_zero_padding_samples,
                state=lambda t, cfg: oracle.PipelineState(t["bos_id"], t["streaming_pad_id"],
                                                          t["samples_per_token"], cfg))


def _library_side(V):
    def state(t, cfg):
        return V.PipelineState(V.PipelineConfig(t["bos_id"], t["streaming_pad_id"], t["samples_per_token"], cfg))
    return dict(cfg=lambda p: V.StreamPromptConfig(**p), prompt=V.build_prompt_ids, ready=V.decode_ready,
                budget=V.decodable_token_budget, pad=V.finish_zero_padding_samples, state=state)


@pytest.fixture(params=["oracle", "library"])
def side(request, oracle, V):
    return _oracle_side(oracle) if request.param == "oracle" else _library_side(V)


def test_prompt_and_budget_formulas_match_reference_schedule(side, ref_tests):
    t = ref_tests["prompt_and_budget_formulas_match_reference_schedule"]  # stream.rs:78-91
    cfg = side["cfg"](t["prompt"])
    prompt = side["prompt"](t["bos_id"], t["streaming_pad_id"], cfg)
    assert len(prompt) == t["expect_prompt_len"]
    assert prompt[0] == t["expect_first"] and all(i == t["expect_rest"] for i in prompt[1:])
    L = len(prompt)
    for rel, ready, budget in t["budget_cases"]:
        if ready is not None:
            assert side["ready"](L + rel, L) == ready
        assert side["budget"](L + rel, L) == budget


def test_finish_padding_matches_alignment_plus_right_budget(side, ref_tests):
    t = ref_tests["finish_padding_matches_alignment_plus_right_budget"]  # stream.rs:93-102
    cfg = side["cfg"](dict(left_pad_tokens=32, delay_tokens=6, eos_extra_tokens=10))
    assert side["pad"](t["consumed"], t["samples_per_token"], cfg) == t["expect"]


def test_planner_tracks_budget_across_chunks(side, ref_tests):
    t = ref_tests["planner_tracks_budget_across_chunks"]  # pipeline.rs:99-130
    st = side["state"](t, side["cfg"](dict(left_pad_tokens=32, delay_tokens=6, eos_extra_tokens=10)))
    prompt = st.prompt_ids() if callable(st.prompt_ids) else st.prompt_ids
    assert len(prompt) == t["expect_prompt_len"]
    for op, arg, want in t["ops"]:
        if op == "push":
            st.push_adapter_tokens(arg)
        elif op == "mark_decoded":
            st.mark_decoded(arg)
        else:
            assert getattr(st, op)() == want, op


def test_planner_finish_padding_formula(side, ref_tests):
    t = ref_tests["planner_finish_padding_formula"]  # pipeline.rs:132-144
    st = side["state"](t, side["cfg"](dict(left_pad_tokens=32, delay_tokens=6, eos_extra_tokens=10)))
    assert st.finish_padding_samples(t["consumed"]) == t["expect"]
    assert st.is_finished() == t["expect_finished"]


def test_library_planner_matches_oracle_on_random_sequences(oracle, V):
    rng = np.random.default_rng(11)
    for trial in range(20):
        lp, dl, ex = (int(x) for x in rng.integers(0, 40, 3))
        spt = int(rng.integers(1, 3000))
        ocfg = oracle.stream_prompt_config(lp, dl, ex)
        lcfg = V.StreamPromptConfig(lp, dl, ex)
        assert V.build_prompt_ids(7, 9, lcfg) == oracle.stream_build_prompt_ids(7, 9, ocfg)
        assert lcfg.right_pad_tokens() == oracle.stream_right_pad_tokens(ocfg)
        a = oracle.PipelineState(7, 9, spt, ocfg)
        b = V.PipelineState(V.PipelineConfig(7, 9, spt, lcfg))
        for _ in range(50):
            if rng.random() < 0.5:
                n = int(rng.integers(0, 30))
                a.push_adapter_tokens(n)
                b.push_adapter_tokens(n)
            else:
                n = int(rng.integers(0, a.decodable_now() + 1))
                a.mark_decoded(n)
                b.mark_decoded(n)
            assert (a.adapter_tokens_total(), a.generated_tokens(), a.decodable_now()) == \
                   (b.adapter_tokens_total(), b.generated_tokens(), b.decodable_now())
        consumed = int(rng.integers(0, 100000))
        assert a.finish_padding_samples(consumed) == b.finish_padding_samples(consumed)


def test_library_planner_errors(V):
    st = V.PipelineState(V.PipelineConfig(1, 32, 1280, V.StreamPromptConfig()))
    st.push_adapter_tokens(39)
    with pytest.raises(V.VoxError) as e:
        st.mark_decoded(2)  # pipeline.rs:74 debug_assert: n <= decodable_now
    assert e.value.code == V.ERR_INVALID_ARG
    with pytest.raises(V.VoxError) as e:
        st.decode()          # a planner has no device to decode on
    assert e.value.code == V.ERR_NOT_READY
    assert V.finish_zero_padding_samples(100, 0, V.StreamPromptConfig()) == 0
