"""Tekken decode (tokenizer.rs) on the host: the reference's two tokenizer
tests (fixtures in tests/golden/) through the library's C ABI and the
oracle's Python restatement, the two agreeing on random vocabularies
(invalid UTF-8 included), and the parse errors."""
import base64
import json
import os

import numpy as np
import pytest

from oracle.tekken import Tekken
from tests.vox_testlib import vox

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


@pytest.fixture(scope="module")
def V():
    return vox()


@pytest.fixture(scope="module")
def ref_tests():
    with open(os.path.join(GOLDEN, "reference_unit_tests.json")) as f:
        return json.load(f)


def test_tokenizer_decodes_basic_tokens(V, ref_tests):
    t = ref_tests["tokenizer_decodes_basic_tokens"]  # tokenizer.rs:219-257
    for tok in (V.TekkenTokenizer.from_json_str(t["json"]), Tekken(t["json"])):
        if isinstance(tok, Tekken):
            assert tok.vsize == 16 and tok.nspecial == 4
            assert tok.special_id("<s>") == 1 and tok.special_id("</s>") == 2
        else:
            for k, v in t["expect"].items():
                assert getattr(tok, k)() == v, k
        assert tok.transcription_delay_tokens() == t["expect"]["transcription_delay_tokens"]
        assert tok.decode_to_utf8_lossy(t["decode_ids"]) == t["decode_expect"]


def test_default_prompt_has_expected_length(V, ref_tests, tmp_path):
    t = ref_tests["default_prompt_has_expected_length"]  # tokenizer.rs:259-286
    path = tmp_path / "tekken.json"
    path.write_text(t["json"])
    for tok in (V.TekkenTokenizer.from_path(str(path)), Tekken(t["json"])):
        prompt = tok.default_prompt_ids()
        assert len(prompt) == t["expect_len"]
        assert prompt[0] == t["expect_first"] and all(i == t["expect_rest"] for i in prompt[1:])
    lib_tok = V.TekkenTokenizer.from_path(str(path))
    assert lib_tok.decode_token_bytes(0) is None        # the missing rank 0 is a control token
    assert lib_tok.decode_token_bytes(5) is None        # vocab id without bytes
    assert lib_tok.decode_token_bytes(8) is None        # beyond default_vocab_size


def _random_vocab(rng, n_special, n_vocab, vsize):
    specials = [{"rank": r, "token_str": f"<sp{r}>é", "is_control": bool(rng.random() < 0.5)}
                for r in range(n_special + 2) if rng.random() < 0.8]          # ranks past the count are skipped
    vocab = []
    for r in range(n_vocab):
        n = int(rng.integers(0, 5))
        b = bytes(int(x) for x in rng.integers(0, 256, n))                    # arbitrary bytes, often invalid UTF-8
        vocab.append({"rank": r, "token_bytes": base64.b64encode(b).decode(), "extra": "ignored"})
    audio = {"sampling_rate": 16000, "frame_rate": float(rng.choice([12.5, 10.0, 7.3])),
             "transcription_delay_ms": int(rng.integers(0, 2000)), "streaming_n_left_pad_tokens": 32}
    return json.dumps({"config": {"default_vocab_size": vsize, "default_num_special_tokens": n_special},
                       "special_tokens": specials, "vocab": vocab, "audio": audio})


def test_random_vocabularies_match_oracle(V):
    rng = np.random.default_rng(9)
    for trial in range(25):
        ns, nv = int(rng.integers(0, 6)), int(rng.integers(0, 40))
        vsize = int(rng.integers(1, ns + nv + 5))
        text = _random_vocab(rng, ns, nv, vsize)
        a, b = V.TekkenTokenizer.from_json_str(text), Tekken(text)
        assert a.transcription_delay_tokens() == b.transcription_delay_tokens()
        assert a.default_prompt_ids() == b.default_prompt_ids()
        for i in range(vsize + 3):
            assert a.decode_token_bytes(i) == b.decode_token_bytes(i), (trial, i)
            assert a.special_id(f"<sp{i}>é") == b.special_id(f"<sp{i}>é")
        for _ in range(10):
            ids = [int(x) for x in rng.integers(0, vsize + 3, int(rng.integers(0, 12)))]
            assert a.decode_to_utf8_lossy(ids) == b.decode_to_utf8_lossy(ids), (trial, ids)


def test_utf8_lossy_maximal_subparts(V):
    """Byte sequences with the replacement counts String::from_utf8_lossy gives."""
    cases = [b"\xf0\x9f\x98", b"\xe0\x80\x80", b"\xed\xa0\x80", b"\xc0\xaf", b"a\xffb", b"\xf4\x90\x80\x80",
             b"\xe2\x82\xac\xe2\x82", "héllo \U0001F600".encode()]
    for raw in cases:
        text = json.dumps({"config": {"default_vocab_size": 2, "default_num_special_tokens": 1},
                           "special_tokens": [], "vocab": [{"rank": 0, "token_bytes": base64.b64encode(raw).decode()}]})
        tok = V.TekkenTokenizer.from_json_str(text)
        assert tok.decode_to_utf8_lossy([1]) == raw.decode("utf-8", errors="replace"), raw


@pytest.mark.parametrize("text,msg", [
    ("{", "parse tekken.json"),
    ('{"config": {"default_vocab_size": 0, "default_num_special_tokens": 0}, "special_tokens": [], "vocab": []}',
     "default_vocab_size must be > 0"),
    ('{"config": {"default_vocab_size": 4, "default_num_special_tokens": 0}, "special_tokens": [],'
     ' "vocab": [{"rank": 0, "token_bytes": "QQ="}]}', "decode base64 for vocab rank 0"),
    ('{"config": {"default_vocab_size": 4, "default_num_special_tokens": 0}, "special_tokens": [],'
     ' "vocab": [{"rank": 0, "token_bytes": "QR=="}]}', "decode base64 for vocab rank 0"),
    ('{"config": {"default_vocab_size": 4.5, "default_num_special_tokens": 0}, "special_tokens": [], "vocab": []}',
     "default_vocab_size"),
    ('{"config": {"default_vocab_size": 4, "default_num_special_tokens": 0}, "vocab": []}', "special_tokens"),
])
def test_parse_errors(V, text, msg):
    with pytest.raises(V.VoxError) as e:
        V.TekkenTokenizer.from_json_str(text)
    assert e.value.code == V.ERR_FORMAT and msg in e.value.message
    with pytest.raises(Exception):
        Tekken(text)
