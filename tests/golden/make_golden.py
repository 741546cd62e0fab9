"""Writes the golden fixtures under tests/golden/.

reference_unit_tests.json holds the inputs and expected answers of the
reference crate's own hot-path unit tests, transcribed from its source
(the reference is Rust and cannot be compiled here, so its tests are read as
text and re-run against the oracle and the CUDA library):

  ops.rs:139-151   linear_smoke
  ops.rs:154-237   gqa_matches_expanded_kv_reference (LCG seed 123)
  math.rs:95-104   rms_norm_rows_smoke
  math.rs:107-133  rope_preserves_pairwise_norm
  math.rs:136-147  silu_and_softmax_smoke
  kv.rs:109-136    compacts_when_exceeding_window
  kv.rs:139-151    layers_are_isolated
  decoder.rs:185-214 decoder_step_grows_and_compacts_cache (LCG seed 7, x0.05)
  stream.rs:78-91   prompt_and_budget_formulas_match_reference_schedule
  stream.rs:93-102  finish_padding_matches_alignment_plus_right_budget
  pipeline.rs:99-130  planner_tracks_budget_across_chunks
  pipeline.rs:132-144 planner_finish_padding_formula
  weights.rs:141-193  loads_f32_and_bf16_tensors
  tokenizer.rs:219-257 tokenizer_decodes_basic_tokens
  tokenizer.rs:259-286 default_prompt_has_expected_length
  mel.rs:277-294   silence_has_constant_value
  mel.rs:296-310   finish_drops_last_frame
  conv.rs:472-568  incremental_conv_matches_offline_even_length (LCG seed 1 x0.01, mel seed 123)

The 32-bit LCG below is the one the reference tests use
(seed = seed*1664525 + 1013904223; value = (seed>>8)/2^24*2-1, in f32).

oracle_regression.json holds oracle outputs for those same inputs (the
decoder test's per-step hidden states), used as fixed regression vectors.

Run:  python tests/golden/make_golden.py
"""
from __future__ import annotations

import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

F = np.float32


def lcg_values(seed: int, n: int, scale=None):
    """ops.rs:160-164 / decoder.rs:163-167."""
    out = np.empty(n, np.float32)
    s = seed
    for i in range(n):
        s = (s * 1664525 + 1013904223) & 0xFFFFFFFF
        v = F(s >> 8) / F(1 << 24) * F(2.0) - F(1.0)
        if scale is not None:
            v = F(v * F(scale))
        out[i] = v
    return out, s


def gqa_expanded_reference(q, k, v, n_heads, n_kv_heads, head_dim, seq_len):
    """The test's own expanded-KV restatement, ops.rs:194-228 (f32 scalar ops)."""
    repeat = n_heads // n_kv_heads
    out = np.zeros(n_heads * head_dim, np.float32)
    scale = F(1.0) / np.sqrt(F(head_dim), dtype=np.float32)
    for h in range(n_heads):
        kv_h = h // repeat
        qh = q[h * head_dim:(h + 1) * head_dim]
        scores = np.zeros(seq_len, np.float32)
        for t in range(seq_len):
            kb = (t * n_kv_heads + kv_h) * head_dim
            dot = F(0.0)
            for i in range(head_dim):
                dot = F(dot + F(qh[i] * k[kb + i]))
            scores[t] = F(dot * scale)
        m = F(-np.inf)
        for s_ in scores:
            m = max(m, s_)
        ssum = F(0.0)
        for t in range(seq_len):
            scores[t] = np.exp(F(scores[t] - m), dtype=np.float32)
            ssum = F(ssum + scores[t])
        for t in range(seq_len):
            scores[t] = F(scores[t] / ssum)
        for t in range(seq_len):
            vb = (t * n_kv_heads + kv_h) * head_dim
            for i in range(head_dim):
                out[h * head_dim + i] = F(out[h * head_dim + i] + F(scores[t] * v[vb + i]))
    return out


def decoder_fake_weights(cfg):
    """decoder.rs:162-182: one LCG stream (seed 7, scale 0.05) in field order."""
    dim, hid = cfg["dim"], cfg["hidden_dim"]
    q_dim = cfg["n_heads"] * cfg["head_dim"]
    kv_dim = cfg["n_kv_heads"] * cfg["head_dim"]
    sizes = [("attention_norm", dim), ("wq", q_dim * dim), ("wk", kv_dim * dim),
             ("wv", kv_dim * dim), ("wo", dim * q_dim), ("ffn_norm", dim),
             ("w1", hid * dim), ("w2", dim * hid), ("w3", hid * dim)]
    total = sum(n for _, n in sizes)
    vals, _ = lcg_values(7, total, 0.05)
    out, o = {}, 0
    for name, n in sizes:
        out[name] = vals[o:o + n]
        o += n
    return out


def reference_unit_tests():
    tests = {}
    # ops.rs:139-151
    tests["linear_smoke"] = {
        "cite": "crates/voxtral/src/ops.rs:139-151",
        "x": [1.0, 2.0, 3.0, -1.0, 0.0, 1.0], "n_rows": 2, "in_dim": 3,
        "w": [1.0, 0.0, -1.0, 2.0, 1.0, 0.0], "out_dim": 2, "bias": [0.5, -1.0],
        "expected": [-1.5, 3.0, -1.5, -3.0], "tol": 1e-6,
    }
    # ops.rs:154-237
    n_heads, n_kv, hd, seq = 4, 2, 3, 5
    vals, _ = lcg_values(123, n_heads * hd + 2 * seq * n_kv * hd)
    q = vals[:n_heads * hd]
    k = vals[n_heads * hd:n_heads * hd + seq * n_kv * hd]
    v = vals[n_heads * hd + seq * n_kv * hd:]
    tests["gqa_matches_expanded_kv_reference"] = {
        "cite": "crates/voxtral/src/ops.rs:154-237",
        "n_heads": n_heads, "n_kv_heads": n_kv, "head_dim": hd, "seq_len": seq,
        "sliding_window": 0, "q": q.tolist(), "k": k.tolist(), "v": v.tolist(),
        "expected": gqa_expanded_reference(q, k, v, n_heads, n_kv, hd, seq).tolist(),
        "tol": 1e-5,
    }
    # math.rs:95-104
    tests["rms_norm_rows_smoke"] = {
        "cite": "crates/voxtral/src/math.rs:95-104",
        "input": [3.0, 4.0, 0.0, 1.0], "weight": [1.0, 1.0], "dim": 2, "eps": 1e-5,
        "expected_first_row": [0.8485, 1.1314], "tol": 1e-3,
    }
    # math.rs:107-133
    x = (np.arange(3 * 2 * 4, dtype=np.float32) * F(0.01) + F(0.1)).astype(np.float32)
    tests["rope_preserves_pairwise_norm"] = {
        "cite": "crates/voxtral/src/math.rs:107-133",
        "x": x.tolist(), "seq_len": 3, "n_heads": 2, "head_dim": 4, "pos_offset": 7,
        "theta": 10000.0, "tol": 1e-4,
    }
    # math.rs:136-147
    tests["silu_and_softmax_smoke"] = {
        "cite": "crates/voxtral/src/math.rs:136-147",
        "silu_input": [0.0, 1.0, -1.0], "softmax_input": [1.0, 2.0, 3.0], "sum_tol": 1e-5,
    }
    # kv.rs:109-136
    tests["compacts_when_exceeding_window"] = {
        "cite": "crates/voxtral/src/kv.rs:109-136",
        "n_layers": 1, "n_kv_heads": 2, "head_dim": 2, "window": 4,
        "appends": [
            {"k": list(range(0, 12)), "v": list(range(100, 112)), "n": 3,
             "expect_len": 3, "expect_pos_offset": 0},
            {"k": list(range(1000, 1012)), "v": list(range(2000, 2012)), "n": 3,
             "expect_len": 4, "expect_pos_offset": 2},
        ],
        # First kept token = absolute token 2 of the first append; last = token 2 of the second.
        "expect_k_first": 8.0, "expect_v_first": 108.0,
        "expect_k_last": 1008.0, "expect_v_last": 2008.0,
    }
    # kv.rs:139-151
    tests["layers_are_isolated"] = {
        "cite": "crates/voxtral/src/kv.rs:139-151",
        "n_layers": 2, "n_kv_heads": 1, "head_dim": 2, "window": 3,
        "appends": [
            {"layer": 0, "k": [1.0, 2.0], "v": [3.0, 4.0], "n": 1},
            {"layer": 1, "k": [10.0, 20.0, 30.0, 40.0], "v": [50.0, 60.0, 70.0, 80.0], "n": 2},
        ],
        "expect_len": [1, 2], "expect_k": [[1.0, 2.0], [10.0, 20.0, 30.0, 40.0]],
    }
    # decoder.rs:185-214
    cfg = {"dim": 8, "hidden_dim": 16, "n_heads": 2, "n_kv_heads": 1, "head_dim": 4,
           "sliding_window": 4, "norm_eps": 1e-5, "rope_theta": 10000.0}
    w = decoder_fake_weights(cfg)
    tests["decoder_step_grows_and_compacts_cache"] = {
        "cite": "crates/voxtral/src/decoder.rs:185-214",
        "config": cfg, "weights": {k_: v_.tolist() for k_, v_ in w.items()},
        "steps": 6, "hidden_rule": "hidden[i] = pos*0.1 + i*0.01 (f32), rewritten before every step",
        "expect_len": 4, "expect_pos_offset": 2,
    }
    # stream.rs:78-91 (default StreamPromptConfig: left pad 32, delay 6, eos extra 10)
    tests["prompt_and_budget_formulas_match_reference_schedule"] = {
        "cite": "crates/voxtral/src/stream.rs:78-91",
        "bos_id": 1, "streaming_pad_id": 32, "prompt": {"left_pad_tokens": 32, "delay_tokens": 6,
                                                        "eos_extra_tokens": 10},
        "expect_prompt_len": 1 + 32 + 6, "expect_first": 1, "expect_rest": 32,
        # (total adapter tokens relative to the prompt length, decode_ready, budget)
        "budget_cases": [[-1, False, 0], [0, True, 1], [9, None, 10]],
    }
    # stream.rs:93-102
    tests["finish_padding_matches_alignment_plus_right_budget"] = {
        "cite": "crates/voxtral/src/stream.rs:93-102",
        "consumed": 3 * 1280 + 640, "samples_per_token": 1280, "expect": 640 + 17 * 1280,
    }
    # pipeline.rs:99-130: a sequence of (op, argument, expected) on one PipelineState
    tests["planner_tracks_budget_across_chunks"] = {
        "cite": "crates/voxtral/src/pipeline.rs:99-130",
        "bos_id": 1, "streaming_pad_id": 32, "samples_per_token": 1280,
        "expect_prompt_len": 39,
        "ops": [["decodable_now", None, 0], ["push", 20, None], ["decodable_now", None, 0],
                ["push", 19, None], ["adapter_tokens_total", None, 39], ["decodable_now", None, 1],
                ["mark_decoded", 1, None], ["generated_tokens", None, 1], ["decodable_now", None, 0],
                ["push", 10, None], ["decodable_now", None, 10], ["mark_decoded", 7, None],
                ["decodable_now", None, 3]],
    }
    # pipeline.rs:132-144
    tests["planner_finish_padding_formula"] = {
        "cite": "crates/voxtral/src/pipeline.rs:132-144",
        "bos_id": 1, "streaming_pad_id": 32, "samples_per_token": 1280,
        "consumed": 3 * 1280 + 640, "expect": 640 + 17 * 1280, "expect_finished": True,
    }
    # weights.rs:141-193: an F32 [2, 2] tensor "a" and a BF16 [2] tensor "b"
    tests["loads_f32_and_bf16_tensors"] = {
        "cite": "crates/voxtral/src/weights.rs:141-193",
        "a": {"dtype": "F32", "shape": [2, 2], "values": [1.0, 2.5, -3.0, 4.25]},
        "b": {"dtype": "BF16", "shape": [2], "words": [0x3F80, 0xC000], "expect": [1.0, -2.0], "tol": 1e-6},
    }
    # tokenizer.rs:219-257: 16-id vocabulary, 4 specials, ranks 0..2 = "A", "B", "C"
    audio = {"sampling_rate": 16000, "frame_rate": 12.5, "transcription_delay_ms": 480,
             "streaming_n_left_pad_tokens": 32}
    tests["tokenizer_decodes_basic_tokens"] = {
        "cite": "crates/voxtral/src/tokenizer.rs:219-257",
        "json": json.dumps({
            "config": {"default_vocab_size": 16, "default_num_special_tokens": 4},
            "special_tokens": [{"rank": 0, "token_str": "<unk>", "is_control": True},
                               {"rank": 1, "token_str": "<s>", "is_control": True},
                               {"rank": 2, "token_str": "</s>", "is_control": True},
                               {"rank": 3, "token_str": "[STREAMING_PAD]", "is_control": True}],
            "vocab": [{"rank": 0, "token_bytes": "QQ=="}, {"rank": 1, "token_bytes": "Qg=="},
                      {"rank": 2, "token_bytes": "Qw=="}],
            "audio": audio}),
        "expect": {"default_vocab_size": 16, "special_token_count": 4, "bos_id": 1, "eos_id": 2,
                   "streaming_pad_id": 3, "transcription_delay_tokens": 6},
        "decode_ids": [1, 4, 5, 6, 2], "decode_expect": "ABC",
    }
    # tokenizer.rs:259-286: rank 0 missing, empty vocabulary
    tests["default_prompt_has_expected_length"] = {
        "cite": "crates/voxtral/src/tokenizer.rs:259-286",
        "json": json.dumps({
            "config": {"default_vocab_size": 8, "default_num_special_tokens": 4},
            "special_tokens": [{"rank": 1, "token_str": "<s>", "is_control": True},
                               {"rank": 2, "token_str": "</s>", "is_control": True},
                               {"rank": 3, "token_str": "[STREAMING_PAD]", "is_control": True}],
            "vocab": [], "audio": audio}),
        "expect_len": 1 + 32 + 6, "expect_first": 1, "expect_rest": 3,
    }
    # mel.rs:277-294 and :296-310 (MelCtx with no extra left padding)
    tests["silence_has_constant_value"] = {
        "cite": "crates/voxtral/src/mel.rs:277-294",
        "left_pad_samples": 0, "expect_left_pad": 200, "feed_zeros": 400, "expect_frames": 2,
        "expect_value": -0.625, "tol": 1e-6,
    }
    fed = 1600
    tests["finish_drops_last_frame"] = {
        "cite": "crates/voxtral/src/mel.rs:296-310",
        "feed_zeros": fed, "expect_frames_after_finish": ((200 + fed + 200 - 400) // 160 + 1) - 1,
    }
    # conv.rs:472-568: ConvStemWeights::fake (conv.rs:92-131) draws conv0_weight,
    # conv0_bias, conv1_weight, conv1_bias in that order from one LCG (seed 1), x0.01
    mel_bins, dim, frames = 8, 16, 40
    st = 1
    w0, st = lcg_values(st, dim * mel_bins * 3, 0.01)
    b0, st = lcg_values(st, dim, 0.01)
    w1, st = lcg_values(st, dim * dim * 3, 0.01)
    b1, st = lcg_values(st, dim, 0.01)
    mel, _ = lcg_values(123, frames * mel_bins)
    tests["incremental_conv_matches_offline_even_length"] = {
        "cite": "crates/voxtral/src/conv.rs:472-568",
        "mel_bins": mel_bins, "dim": dim, "frames": frames, "chunks": [7, 3, 11, 5, 14],
        "conv0_weight": w0.tolist(), "conv0_bias": b0.tolist(), "conv1_weight": w1.tolist(),
        "conv1_bias": b1.tolist(), "mel": mel.tolist(), "conv0_bit_exact": True, "tol": 1e-4,
    }
    return tests


def decoder_test_hidden(pos, dim):
    """decoder.rs:200-203: hidden[i] = (pos as f32)*0.1 + (i as f32)*0.01."""
    return np.array([F(F(pos) * F(0.1)) + F(F(i) * F(0.01)) for i in range(dim)], np.float32)


def oracle_regression(tests):
    from oracle import oracle as o
    o.build()
    t = tests["decoder_step_grows_and_compacts_cache"]
    c = t["config"]
    cfg = o.config(**c)
    w = {k: np.array(v, np.float32) for k, v in t["weights"].items()}
    lw = o.LayerWeights(w["attention_norm"], w["ffn_norm"],
                        **{n: w[n] for n in o.LayerWeights.NAMES})
    cache = o.RollingKvCache(1, c["n_kv_heads"], c["head_dim"], c["sliding_window"])
    outs = []
    # decoder.rs:199-209: the loop overwrites hidden from the pos rule every step, so
    # the fed-back output is replaced before use.
    for pos in range(t["steps"]):
        hidden = decoder_test_hidden(pos, c["dim"])
        out = o.decoder_layer_forward_step(cfg, 0, lw, cache, hidden, pos)
        outs.append(out.tolist())
    k, v = cache.layer_tensors(0)
    return {
        "decoder_step_outputs": outs,
        "decoder_step_len": cache.layer_len_tokens(0),
        "decoder_step_pos_offset": cache.layer_pos_offset(0),
        "decoder_step_k": k.tolist(), "decoder_step_v": v.tolist(),
    }


def main():
    tests = reference_unit_tests()
    with open(os.path.join(HERE, "reference_unit_tests.json"), "w") as f:
        json.dump(tests, f, indent=1)
    reg = oracle_regression(tests)
    with open(os.path.join(HERE, "oracle_regression.json"), "w") as f:
        json.dump(reg, f, indent=1)
    print("wrote reference_unit_tests.json and oracle_regression.json")


if __name__ == "__main__":
    main()
