"""Restatement of the Tekken decode path (crates/voxtral/src/tokenizer.rs:72-213)
in Python (TEST INFRASTRUCTURE ONLY).  json, base64 with validation and
Python's UTF-8 'replace' error handler (maximal invalid subparts become
U+FFFD, the rule of String::from_utf8_lossy) stand in for serde_json, the
base64 0.22 STANDARD engine and the Rust standard library."""
from __future__ import annotations

import base64
import binascii
import json
import math
import struct


def _b64_standard(s: str) -> bytes:
    """Standard alphabet, canonical padding, no trailing bits (base64 0.22 STANDARD)."""
    if len(s) % 4:
        raise ValueError("invalid length")
    try:
        out = base64.b64decode(s, validate=True)
    except binascii.Error as e:
        raise ValueError(str(e))
    if base64.b64encode(out).decode() != s:   # rejects non-canonical trailing bits
        raise ValueError("non-canonical encoding")
    return out


def _usize(v):
    if isinstance(v, bool) or not isinstance(v, int) or v < 0:
        raise ValueError("expected usize")
    return v


def _f32(x: float) -> float:
    return struct.unpack("<f", struct.pack("<f", x))[0]


class Tekken:
    def __init__(self, text: str):
        f = json.loads(text)                                        # tokenizer.rs:73
        cfg = f["config"]
        vsize = _usize(cfg["default_vocab_size"])
        nspecial = _usize(cfg["default_num_special_tokens"])
        specials = [(_usize(e["rank"]), str(e["token_str"]), bool(e["is_control"])) for e in f["special_tokens"]]
        vocab = [(_usize(e["rank"]), str(e["token_bytes"])) for e in f["vocab"]]
        audio = f.get("audio")
        if vsize == 0:                                              # tokenizer.rs:74-77
            raise ValueError("default_vocab_size must be > 0")
        slots = [None] * nspecial
        self.lookup = {}
        for rank, text_, ctl in specials:                           # tokenizer.rs:79-90
            if rank >= nspecial:
                continue
            self.lookup[text_] = rank
            slots[rank] = (text_, ctl)
        self.specials = [s if s else (f"<missing-special-{r}>", True) for r, s in enumerate(slots)]
        self.tokens = [None] * vsize
        for rank, b64 in vocab:                                     # tokenizer.rs:102-113
            tid = nspecial + rank
            if tid >= vsize:
                continue
            self.tokens[tid] = _b64_standard(b64)
        self.vsize, self.nspecial = vsize, nspecial
        self.audio = None if audio is None else dict(
            sampling_rate=_usize(audio["sampling_rate"]), frame_rate=_f32(float(audio["frame_rate"])),
            transcription_delay_ms=_usize(audio["transcription_delay_ms"]),
            streaming_n_left_pad_tokens=_usize(audio["streaming_n_left_pad_tokens"]))

    def special_id(self, text):
        return self.lookup.get(text)

    def transcription_delay_tokens(self):
        if self.audio is None:
            return None
        seconds = _f32(_f32(float(self.audio["transcription_delay_ms"])) / 1000.0)
        prod = _f32(seconds * self.audio["frame_rate"])
        r = math.floor(abs(prod) + 0.5) * (1 if prod >= 0 else -1)   # f32::round: half away from zero
        return max(0, int(r))

    def default_prompt_ids(self):
        bos, pad = self.special_id("<s>"), self.special_id("[STREAMING_PAD]")
        if bos is None or pad is None or self.audio is None:
            return None
        n = self.audio["streaming_n_left_pad_tokens"] + self.transcription_delay_tokens()
        return [bos] + [pad] * n

    def decode_token_bytes(self, tid):
        if tid >= self.vsize:
            return None
        if tid < self.nspecial:
            text_, ctl = self.specials[tid]
            return None if ctl else text_.encode()
        return self.tokens[tid]

    def decode_to_utf8_lossy(self, ids):
        raw = b"".join(b for b in (self.decode_token_bytes(i) for i in ids) if b is not None)
        return raw.decode("utf-8", errors="replace")
