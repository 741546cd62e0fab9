"""ctypes front end for the CPU oracle (oracle/vox_oracle.c).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and the
CPU-baseline leg of bench.py, never by the product package.  Each wrapper
names the reference function (crates/voxtral/src/...) it restates.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "_build", "libvoxoracle.so")

_lib = None

F32P = C.POINTER(C.c_float)
U16P = C.POINTER(C.c_uint16)
I32P = C.POINTER(C.c_int32)
SZ = C.c_size_t


class VoConfig(C.Structure):
    """DecoderConfig (crates/voxtral/src/decoder.rs:10-19)."""

    _fields_ = [
        ("dim", SZ), ("hidden_dim", SZ), ("n_heads", SZ), ("n_kv_heads", SZ),
        ("head_dim", SZ), ("sliding_window", SZ), ("norm_eps", C.c_float),
        ("rope_theta", C.c_float),
    ]


class VoLayerWeights(C.Structure):
    _fields_ = [
        ("bf16", C.c_int), ("attention_norm", F32P), ("ffn_norm", F32P),
        ("wq", F32P), ("wk", F32P), ("wv", F32P), ("wo", F32P),
        ("w1", F32P), ("w2", F32P), ("w3", F32P),
        ("wq_h", U16P), ("wk_h", U16P), ("wv_h", U16P), ("wo_h", U16P),
        ("w1_h", U16P), ("w2_h", U16P), ("w3_h", U16P),
    ]


class VoModel(C.Structure):
    _fields_ = [
        ("cfg", VoConfig), ("n_layers", SZ), ("vocab", SZ),
        ("layers", C.POINTER(VoLayerWeights)), ("embed", U16P),
        ("final_norm", F32P), ("lm_head", U16P),
    ]


class VoStreamPromptConfig(C.Structure):
    """StreamPromptConfig (stream.rs:4-9)."""

    _fields_ = [("left_pad_tokens", SZ), ("delay_tokens", SZ), ("eos_extra_tokens", SZ)]


class VoPipeline(C.Structure):
    _fields_ = [("bos_id", C.c_uint32), ("streaming_pad_id", C.c_uint32), ("samples_per_token", SZ),
                ("prompt", VoStreamPromptConfig), ("prompt_len", SZ), ("adapter_tokens_total", SZ),
                ("generated_tokens", SZ), ("finished", C.c_int)]


def build():
    """Compile the oracle with its Makefile (gcc, -ffp-contract=off)."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        L = C.CDLL(_LIB_PATH)
        L.vo_config_validate.argtypes = [C.POINTER(VoConfig)]
        L.vo_silu_inplace.argtypes = [F32P, SZ]
        L.vo_rms_norm_rows.argtypes = [F32P, F32P, F32P, SZ, SZ, C.c_float]
        L.vo_rope_interleaved_inplace.argtypes = [F32P, SZ, SZ, SZ, SZ, C.c_float]
        L.vo_softmax_inplace.argtypes = [F32P, SZ]
        L.vo_linear.argtypes = [F32P, SZ, SZ, F32P, SZ, F32P, F32P]
        L.vo_linear_bf16.argtypes = [F32P, SZ, SZ, U16P, SZ, F32P, F32P]
        L.vo_add_inplace.argtypes = [F32P, F32P, SZ]
        L.vo_attention_gqa_step.argtypes = [F32P, F32P, F32P, SZ, SZ, SZ, SZ, SZ, F32P]
        L.vo_kv_new.argtypes = [SZ, SZ, SZ, SZ]
        L.vo_kv_new.restype = C.c_void_p
        L.vo_kv_free.argtypes = [C.c_void_p]
        L.vo_kv_clone.argtypes = [C.c_void_p]
        L.vo_kv_clone.restype = C.c_void_p
        L.vo_kv_append_layer.argtypes = [C.c_void_p, SZ, F32P, F32P, SZ]
        L.vo_kv_layer_len_tokens.argtypes = [C.c_void_p, SZ]
        L.vo_kv_layer_len_tokens.restype = SZ
        L.vo_kv_layer_pos_offset.argtypes = [C.c_void_p, SZ]
        L.vo_kv_layer_pos_offset.restype = SZ
        L.vo_kv_layer_keys.argtypes = [C.c_void_p, SZ]
        L.vo_kv_layer_keys.restype = F32P
        L.vo_kv_layer_values.argtypes = [C.c_void_p, SZ]
        L.vo_kv_layer_values.restype = F32P
        L.vo_kv_layer_set.argtypes = [C.c_void_p, SZ, F32P, F32P, SZ, SZ]
        L.vo_decoder_layer_forward_step.argtypes = [
            C.POINTER(VoConfig), SZ, C.POINTER(VoLayerWeights), C.c_void_p, F32P, SZ, SZ, F32P]
        L.vo_model_step.argtypes = [C.POINTER(VoModel), C.c_void_p, C.c_int32, SZ, F32P, I32P]
        L.vo_model_step_adapter.argtypes = [C.POINTER(VoModel), C.c_void_p, C.c_int32, F32P, SZ, F32P, I32P]
        L.vo_stream_right_pad_tokens.argtypes = [C.POINTER(VoStreamPromptConfig)]
        L.vo_stream_right_pad_tokens.restype = SZ
        L.vo_stream_build_prompt_ids.argtypes = [C.c_uint32, C.c_uint32, C.POINTER(VoStreamPromptConfig),
                                                 C.POINTER(C.c_uint32), SZ]
        L.vo_stream_build_prompt_ids.restype = SZ
        L.vo_stream_decode_ready.argtypes = [SZ, SZ]
        L.vo_stream_decodable_token_budget.argtypes = [SZ, SZ]
        L.vo_stream_decodable_token_budget.restype = SZ
        L.vo_stream_finish_zero_padding_samples.argtypes = [SZ, SZ, C.POINTER(VoStreamPromptConfig)]
        L.vo_stream_finish_zero_padding_samples.restype = SZ
        L.vo_pipeline_init.argtypes = [C.POINTER(VoPipeline), C.c_uint32, C.c_uint32, SZ,
                                       C.POINTER(VoStreamPromptConfig)]
        L.vo_pipeline_push_adapter_tokens.argtypes = [C.POINTER(VoPipeline), SZ]
        L.vo_pipeline_decodable_now.argtypes = [C.POINTER(VoPipeline)]
        L.vo_pipeline_decodable_now.restype = SZ
        L.vo_pipeline_mark_decoded.argtypes = [C.POINTER(VoPipeline), SZ]
        L.vo_pipeline_finish_padding_samples.argtypes = [C.POINTER(VoPipeline), SZ]
        L.vo_pipeline_finish_padding_samples.restype = SZ
        L.vo_gen_normal_f32.argtypes = [C.c_uint64, C.c_uint64, C.c_float, C.c_uint64, SZ, F32P]
        L.vo_gen_normal_bf16.argtypes = [C.c_uint64, C.c_uint64, C.c_float, C.c_uint64, SZ, U16P]
        L.vo_gen_uniform_ids.argtypes = [C.c_uint64, C.c_uint64, C.c_uint32, C.c_uint64, SZ, I32P]
        L.vo_f32_to_bf16_rne.argtypes = [C.c_float]
        L.vo_f32_to_bf16_rne.restype = C.c_uint16
        L.vo_set_threads.argtypes = [C.c_int]
        L.vo_mel_build_filters.argtypes = [F32P]
        L.vo_mel_build_dft.argtypes = [F32P, F32P]
        L.vo_mel_build_window.argtypes = [F32P]
        L.vo_mel_new.argtypes = [SZ]
        L.vo_mel_new.restype = C.c_void_p
        L.vo_mel_free.argtypes = [C.c_void_p]
        L.vo_mel_left_pad_samples.argtypes = [C.c_void_p]
        L.vo_mel_left_pad_samples.restype = SZ
        L.vo_mel_feed.argtypes = [C.c_void_p, F32P, SZ]
        L.vo_mel_feed.restype = SZ
        L.vo_mel_finish.argtypes = [C.c_void_p, SZ]
        L.vo_mel_frames.argtypes = [C.c_void_p]
        L.vo_mel_frames.restype = SZ
        L.vo_mel_data.argtypes = [C.c_void_p]
        L.vo_mel_data.restype = F32P
        L.vo_gelu_inplace.argtypes = [F32P, SZ]
        L.vo_conv_out_len.argtypes = [SZ, SZ, SZ]
        L.vo_conv_out_len.restype = SZ
        L.vo_causal_conv1d_colmajor.argtypes = [F32P, F32P, F32P, F32P, SZ, SZ, SZ, SZ, SZ]
        L.vo_conv_stem_new.argtypes = [SZ, SZ]
        L.vo_conv_stem_new.restype = C.c_void_p
        L.vo_conv_stem_free.argtypes = [C.c_void_p]
        L.vo_conv_stem_process.argtypes = [C.c_void_p, F32P, F32P, F32P, F32P, F32P, SZ, F32P]
        L.vo_conv_stem_process.restype = SZ
        _lib = L
    return _lib


def set_threads(n: int) -> None:
    lib().vo_set_threads(int(n))


def _f32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


def _p(a, t=F32P):
    return a.ctypes.data_as(t)


def config(**kw) -> VoConfig:
    return VoConfig(**kw)


# ---- math.rs ---------------------------------------------------------------

def silu(x):
    """math.rs:4-9"""
    y = _f32(x).copy()
    lib().vo_silu_inplace(_p(y), y.size)
    return y


def rms_norm_rows(x, w, dim, eps):
    """math.rs:11-27"""
    x = _f32(x)
    w = _f32(w)
    out = np.zeros_like(x)
    lib().vo_rms_norm_rows(_p(out), _p(x), _p(w), x.size, dim, eps)
    return out


def rope_interleaved(x, seq_len, n_heads, head_dim, pos_offset, theta):
    """math.rs:30-65"""
    y = _f32(x).copy()
    lib().vo_rope_interleaved_inplace(_p(y), seq_len, n_heads, head_dim, pos_offset, theta)
    return y


def softmax(x):
    """math.rs:67-88"""
    y = _f32(x).copy()
    lib().vo_softmax_inplace(_p(y), y.size)
    return y


# ---- ops.rs ----------------------------------------------------------------

def linear(x, n_rows, in_dim, w, out_dim, bias=None):
    """ops.rs:11-39 (f32 weights)"""
    x = _f32(x)
    w = _f32(w)
    out = np.zeros(n_rows * out_dim, np.float32)
    b = _f32(bias) if bias is not None else None
    lib().vo_linear(_p(x), n_rows, in_dim, _p(w), out_dim, _p(b) if b is not None else None, _p(out))
    return out


def linear_bf16(x, n_rows, in_dim, w_bits, out_dim, bias=None):
    """ops.rs:11-39 with bf16 weights widened exactly (weights.rs:77-81)."""
    x = _f32(x)
    w = np.ascontiguousarray(w_bits, dtype=np.uint16)
    out = np.zeros(n_rows * out_dim, np.float32)
    b = _f32(bias) if bias is not None else None
    lib().vo_linear_bf16(_p(x), n_rows, in_dim, _p(w, U16P), out_dim,
                         _p(b) if b is not None else None, _p(out))
    return out


def add_inplace(dst, src):
    """ops.rs:41-46 (returns the updated copy)"""
    d = _f32(dst).copy()
    s = _f32(src)
    lib().vo_add_inplace(_p(d), _p(s), d.size)
    return d


def attention_gqa_step(q, k, v, n_heads, head_dim, seq_len, n_kv_heads, sliding_window):
    """ops.rs:66-132"""
    q, k, v = _f32(q), _f32(k), _f32(v)
    out = np.zeros(n_heads * head_dim, np.float32)
    lib().vo_attention_gqa_step(_p(q), _p(k), _p(v), n_heads, head_dim, seq_len,
                                n_kv_heads, sliding_window, _p(out))
    return out


# ---- kv.rs -----------------------------------------------------------------

class RollingKvCache:
    """kv.rs:22-101"""

    def __init__(self, n_layers, n_kv_heads, head_dim, sliding_window, _handle=None):
        self.n_layers, self.n_kv_heads, self.head_dim = n_layers, n_kv_heads, head_dim
        self.sliding_window = sliding_window
        self.h = _handle or lib().vo_kv_new(n_layers, n_kv_heads, head_dim, sliding_window)

    def __del__(self):
        if getattr(self, "h", None) and _lib is not None:
            _lib.vo_kv_free(self.h)
            self.h = None

    def clone(self):
        return RollingKvCache(self.n_layers, self.n_kv_heads, self.head_dim,
                              self.sliding_window, lib().vo_kv_clone(self.h))

    def append_layer(self, layer, k_new, v_new, n_new):
        k, v = _f32(k_new), _f32(v_new)
        lib().vo_kv_append_layer(self.h, layer, _p(k), _p(v), n_new)

    def layer_len_tokens(self, layer):
        return lib().vo_kv_layer_len_tokens(self.h, layer)

    def layer_pos_offset(self, layer):
        return lib().vo_kv_layer_pos_offset(self.h, layer)

    def layer_tensors(self, layer):
        n = self.layer_len_tokens(layer) * self.n_kv_heads * self.head_dim
        if n == 0:
            return np.zeros(0, np.float32), np.zeros(0, np.float32)
        k = np.ctypeslib.as_array(lib().vo_kv_layer_keys(self.h, layer), shape=(n,)).copy()
        v = np.ctypeslib.as_array(lib().vo_kv_layer_values(self.h, layer), shape=(n,)).copy()
        return k, v

    def layer_set(self, layer, keys, values, len_tokens, pos_offset):
        k, v = _f32(keys), _f32(values)
        lib().vo_kv_layer_set(self.h, layer, _p(k), _p(v), len_tokens, pos_offset)


# ---- decoder.rs ------------------------------------------------------------

class LayerWeights:
    """DecoderLayerWeights (decoder.rs:45-55).  Matrices are f32 arrays, or
    bf16 bit patterns (uint16) that the oracle widens exactly."""

    NAMES = ("wq", "wk", "wv", "wo", "w1", "w2", "w3")

    def __init__(self, attention_norm, ffn_norm, **mats):
        self.attention_norm = _f32(attention_norm)
        self.ffn_norm = _f32(ffn_norm)
        first = mats["wq"]
        self.bf16 = first.dtype == np.uint16
        self.mats = {}
        for n in self.NAMES:
            a = mats[n]
            self.mats[n] = (np.ascontiguousarray(a, dtype=np.uint16) if self.bf16 else _f32(a))
        self.c = VoLayerWeights()
        self.c.bf16 = 1 if self.bf16 else 0
        self.c.attention_norm = _p(self.attention_norm)
        self.c.ffn_norm = _p(self.ffn_norm)
        for n in self.NAMES:
            if self.bf16:
                setattr(self.c, n + "_h", _p(self.mats[n], U16P))
            else:
                setattr(self.c, n, _p(self.mats[n]))


def config_validate(cfg: VoConfig) -> int:
    """decoder.rs:22-41; returns 0 or the VO_ERR_* code of the first failed check."""
    return lib().vo_config_validate(C.byref(cfg))


def decoder_layer_forward_step(cfg, layer_idx, weights: LayerWeights, cache: RollingKvCache,
                               hidden, pos):
    """decoder.rs:88-155.  Raises ValueError on the reference's Err cases."""
    h = _f32(hidden)
    out = np.zeros(cfg.dim, np.float32)
    rc = lib().vo_decoder_layer_forward_step(C.byref(cfg), layer_idx, C.byref(weights.c),
                                             cache.h, _p(h), h.size, pos, _p(out))
    if rc:
        raise ValueError(f"oracle decoder step failed with code {rc}")
    return out


class Model:
    """Composed token loop: embed -> layers -> final norm -> LM head -> argmax."""

    def __init__(self, cfg, layers, embed_bits, final_norm, lm_head_bits, vocab):
        self.cfg, self.layers = cfg, layers
        self.embed = np.ascontiguousarray(embed_bits, dtype=np.uint16)
        self.final_norm = _f32(final_norm)
        self.lm_head = np.ascontiguousarray(lm_head_bits, dtype=np.uint16)
        self._arr = (VoLayerWeights * len(layers))(*[l.c for l in layers])
        self.c = VoModel(cfg, len(layers), vocab, self._arr, _p(self.embed, U16P),
                         _p(self.final_norm), _p(self.lm_head, U16P))
        self.vocab = vocab

    def step(self, cache, token, pos, want_logits=True):
        logits = np.zeros(self.vocab, np.float32) if want_logits else None
        am = C.c_int32(-1)
        rc = lib().vo_model_step(C.byref(self.c), cache.h, int(token), int(pos),
                                 _p(logits) if want_logits else None, C.byref(am))
        if rc:
            raise ValueError(f"oracle model step failed with code {rc}")
        return logits, am.value


    def step_adapter(self, cache, token, adapter_row, pos, want_logits=True):
        """Streaming input: x = adapter_row + tok_embed(token)."""
        logits = np.zeros(self.vocab, np.float32) if want_logits else None
        am = C.c_int32(-1)
        row = _f32(adapter_row)
        rc = lib().vo_model_step_adapter(C.byref(self.c), cache.h, int(token), _p(row), int(pos),
                                         _p(logits) if want_logits else None, C.byref(am))
        if rc:
            raise ValueError(f"oracle adapter step failed with code {rc}")
        return logits, am.value

    def stream_decode(self, cache, prompt_ids, adapter, n_tokens, generated=(), want_logits=False):
        """The streaming schedule of docs/plans/2026-02-11-voxtral-rust-design.md:40-46
        composed over the layer step.  With L = len(prompt_ids) and no token
        generated yet: positions 0..L-2 are prefilled with adapter[p] +
        tok_embed(prompt[p]); position L-1 takes adapter[L-1] +
        tok_embed(prompt[L-1]) and yields the first token; every later
        position p takes adapter[p] + tok_embed(previous token).  `generated`
        lists tokens produced by earlier calls on the same cache.  Returns the
        next n_tokens greedy tokens (and their logits if asked)."""
        L = len(prompt_ids)
        adapter = np.asarray(adapter, np.float32)
        done = len(generated)
        out, lg = [], []
        if done == 0 and n_tokens > 0:
            for p in range(L - 1):
                self.step_adapter(cache, int(prompt_ids[p]), adapter[p], p, want_logits=False)
        prev = int(prompt_ids[L - 1]) if done == 0 else int(generated[-1])
        for i in range(n_tokens):
            pos = L - 1 + done + i
            logits, prev = self.step_adapter(cache, prev, adapter[pos], pos, want_logits=want_logits)
            out.append(prev)
            lg.append(logits)
        return (out, lg) if want_logits else out


# ---- streaming schedule (stream.rs, pipeline.rs) -------------------------------

def stream_prompt_config(left_pad_tokens=32, delay_tokens=6, eos_extra_tokens=10):
    """StreamPromptConfig; the defaults are StreamPromptConfig::default (stream.rs:11-19)."""
    return VoStreamPromptConfig(left_pad_tokens, delay_tokens, eos_extra_tokens)


def stream_right_pad_tokens(cfg):
    return lib().vo_stream_right_pad_tokens(C.byref(cfg))


def stream_build_prompt_ids(bos_id, pad_id, cfg):
    n = lib().vo_stream_build_prompt_ids(bos_id, pad_id, C.byref(cfg), None, 0)
    out = (C.c_uint32 * max(n, 1))()
    lib().vo_stream_build_prompt_ids(bos_id, pad_id, C.byref(cfg), out, n)
    return [int(out[i]) for i in range(n)]


def stream_decode_ready(total, prompt_len):
    return bool(lib().vo_stream_decode_ready(total, prompt_len))


def stream_decodable_token_budget(total, prompt_len):
    return lib().vo_stream_decodable_token_budget(total, prompt_len)


def stream_finish_zero_padding_samples(consumed, samples_per_token, cfg):
    return lib().vo_stream_finish_zero_padding_samples(consumed, samples_per_token, C.byref(cfg))


class PipelineState:
    """PipelineState (pipeline.rs:28-90), planner only."""

    def __init__(self, bos_id, streaming_pad_id, samples_per_token, prompt_cfg):
        self.c = VoPipeline()
        lib().vo_pipeline_init(C.byref(self.c), bos_id, streaming_pad_id, samples_per_token, C.byref(prompt_cfg))
        self.prompt_ids = stream_build_prompt_ids(bos_id, streaming_pad_id, prompt_cfg)

    def adapter_tokens_total(self):
        return self.c.adapter_tokens_total

    def generated_tokens(self):
        return self.c.generated_tokens

    def push_adapter_tokens(self, n):
        lib().vo_pipeline_push_adapter_tokens(C.byref(self.c), n)

    def decodable_now(self):
        return lib().vo_pipeline_decodable_now(C.byref(self.c))

    def mark_decoded(self, n):
        if lib().vo_pipeline_mark_decoded(C.byref(self.c), n):
            raise ValueError("mark_decoded beyond decodable_now")

    def finish_padding_samples(self, consumed):
        return lib().vo_pipeline_finish_padding_samples(C.byref(self.c), consumed)

    def is_finished(self):
        return bool(self.c.finished)


# ---- encoder front end (mel.rs, conv.rs) ---------------------------------------

MEL_BINS, N_FREQ, N_FFT = 128, 201, 400


def mel_tables():
    """(filters [128, 201], dft cos [201, 400], dft sin [201, 400], Hann [400]) (mel.rs:42-106)."""
    f = np.zeros(MEL_BINS * N_FREQ, np.float32)
    c = np.zeros(N_FREQ * N_FFT, np.float32)
    s_ = np.zeros(N_FREQ * N_FFT, np.float32)
    w = np.zeros(N_FFT, np.float32)
    lib().vo_mel_build_filters(_p(f))
    lib().vo_mel_build_dft(_p(c), _p(s_))
    lib().vo_mel_build_window(_p(w))
    return f.reshape(MEL_BINS, N_FREQ), c.reshape(N_FREQ, N_FFT), s_.reshape(N_FREQ, N_FFT), w


class MelCtx:
    """MelCtx (mel.rs:114-272): incremental log-mel frames [frames, 128]."""

    def __init__(self, left_pad_samples=0):
        self.h = lib().vo_mel_new(left_pad_samples)

    def __del__(self):
        if getattr(self, "h", None):
            lib().vo_mel_free(self.h)
            self.h = None

    def left_pad_samples(self):
        return lib().vo_mel_left_pad_samples(self.h)

    def feed(self, x):
        x = _f32(x)
        return lib().vo_mel_feed(self.h, _p(x), x.size)

    def finish(self, right_pad_samples=0):
        lib().vo_mel_finish(self.h, right_pad_samples)

    def frames(self):
        return lib().vo_mel_frames(self.h)

    def data(self, first=0, n=None):
        """(frames [first, first + n) as [n, 128], total frame count)."""
        total = lib().vo_mel_frames(self.h)
        n = total - first if n is None else n
        if total == 0 or n <= 0:
            return np.zeros((0, MEL_BINS), np.float32), total
        p = lib().vo_mel_data(self.h)
        a = np.ctypeslib.as_array(p, shape=(total * MEL_BINS,)).reshape(total, MEL_BINS)
        return a[first:first + n].copy(), total


def gelu(x):
    """gelu_inplace (conv.rs:11-19) on a copy."""
    y = _f32(x).copy()
    lib().vo_gelu_inplace(_p(y), y.size)
    return y


def causal_conv1d_colmajor(x, w, b, cin, cout, length, kernel, stride):
    """causal_conv1d_colmajor (conv.rs:28-73): x [cin, length] -> [cout, out_len]."""
    n = lib().vo_conv_out_len(length, kernel, stride)
    out = np.zeros(cout * n, np.float32)
    xx, ww = _f32(x), _f32(w)
    bb = _f32(b) if b is not None else None
    lib().vo_causal_conv1d_colmajor(_p(out), _p(xx), _p(ww), _p(bb) if bb is not None else None,
                                    cin, cout, length, kernel, stride)
    return out.reshape(cout, n)


class ConvStemState:
    """ConvStemState (conv.rs:134-347): mel frames [n, mel_bins] -> positions [m, dim]."""

    def __init__(self, mel_bins, dim, w0, b0, w1, b1):
        self.h = lib().vo_conv_stem_new(mel_bins, dim)
        self.mel_bins, self.dim = mel_bins, dim
        self.w = [_f32(w0), _f32(b0), _f32(w1), _f32(b1)]

    def __del__(self):
        if getattr(self, "h", None):
            lib().vo_conv_stem_free(self.h)
            self.h = None

    def process(self, mel_new):
        mel_new = _f32(mel_new)
        n = mel_new.size // self.mel_bins
        out = np.zeros((n // 2 + 2) * self.dim, np.float32)
        m = lib().vo_conv_stem_process(self.h, *[_p(a) for a in self.w], _p(mel_new), n, _p(out))
        return out[:m * self.dim].reshape(m, self.dim)


# ---- seeded synthetic data ---------------------------------------------------

def gen_normal_f32(seed, tensor_id, std, n, first=0):
    out = np.empty(n, np.float32)
    lib().vo_gen_normal_f32(seed, tensor_id, std, first, n, _p(out))
    return out


def gen_normal_bf16(seed, tensor_id, std, n, first=0):
    out = np.empty(n, np.uint16)
    lib().vo_gen_normal_bf16(seed, tensor_id, std, first, n, _p(out, U16P))
    return out


def gen_uniform_ids(seed, tensor_id, bound, n, first=0):
    out = np.empty(n, np.int32)
    lib().vo_gen_uniform_ids(seed, tensor_id, bound, first, n, _p(out, I32P))
    return out


def bf16_to_f32(bits):
    return (np.asarray(bits, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16(x):
    x = _f32(x)
    u = x.view(np.uint32).astype(np.uint64)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    nan = np.isnan(x)
    r[nan] = 0x7FC0
    return r
