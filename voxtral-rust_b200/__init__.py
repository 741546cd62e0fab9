"""voxtral-rust_b200 -- B200 (sm_100a) decoder token loop of voxtral-rust.

Python front end over the C ABI in include/vox_decoder.h (libvoxb200.so).
Names and argument meanings follow the reference crate
(crates/voxtral/src/{decoder,kv,ops,math}.rs) so that code written against
it reads the same.  Every compute call runs CUDA kernels; there is no CPU
fallback: if the shared library is missing the import fails.

The directory name is not a Python identifier; import it with
``importlib.import_module("voxtral-rust_b200")``.
"""
from __future__ import annotations

import ctypes as C
import os
import weakref

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libvoxb200.so")
HEADER_PATH = os.path.join(os.path.dirname(_HERE), "include", "vox_decoder.h")

F32P = C.POINTER(C.c_float)
U16P = C.POINTER(C.c_uint16)
I32P = C.POINTER(C.c_int32)
SZ = C.c_size_t
VP = C.c_void_p

OK, ERR_INVALID_ARG, ERR_CONFIG, ERR_SHAPE, ERR_UNSUPPORTED, ERR_CUDA, ERR_OOM, ERR_NOT_READY, \
    ERR_DEVICE_TIMEOUT, ERR_RANGE, ERR_IO, ERR_FORMAT = range(12)
WEIGHTS_BF16, WEIGHTS_F32 = 0, 1


class VoxError(RuntimeError):
    def __init__(self, code: int, message: str):
        super().__init__(f"[{code}] {message}")
        self.code = code
        self.message = message


class DecoderConfig(C.Structure):
    """DecoderConfig (decoder.rs:10-19)."""

    _fields_ = [("dim", SZ), ("hidden_dim", SZ), ("n_heads", SZ), ("n_kv_heads", SZ),
                ("head_dim", SZ), ("sliding_window", SZ), ("norm_eps", C.c_float),
                ("rope_theta", C.c_float)]

    def validate(self):
        """DecoderConfig::validate (decoder.rs:22-41)."""
        _check(lib().vox_config_validate(C.byref(self)))


class CtxOptions(C.Structure):
    _fields_ = [("device", C.c_int), ("n_layers", SZ), ("vocab", SZ), ("max_positions", SZ),
                ("weight_dtype", C.c_int), ("step_mode", C.c_int)]


STEP_AUTO, STEP_LAYERS, STEP_PERSISTENT = 0, 1, 2


class F32Slice(C.Structure):
    _fields_ = [("ptr", F32P), ("len", SZ)]


class BF16Slice(C.Structure):
    _fields_ = [("ptr", U16P), ("len", SZ)]


_NAMES = ("attention_norm", "wq", "wk", "wv", "wo", "ffn_norm", "w1", "w2", "w3")


class LayerWeightsF32(C.Structure):
    _fields_ = [(n, F32Slice) for n in _NAMES]


class LayerWeightsBF16(C.Structure):
    _fields_ = [("attention_norm", F32Slice), ("wq", BF16Slice), ("wk", BF16Slice),
                ("wv", BF16Slice), ("wo", BF16Slice), ("ffn_norm", F32Slice),
                ("w1", BF16Slice), ("w2", BF16Slice), ("w3", BF16Slice)]


class TpShard(C.Structure):
    """vox_tp_shard: the slice of the model one tensor-parallel rank holds."""

    _fields_ = [("rank", C.c_int), ("size", C.c_int), ("n_heads", SZ), ("n_kv_heads", SZ), ("hidden", SZ),
                ("vocab", SZ), ("vocab_local", SZ), ("q_head_begin", SZ), ("kv_head_begin", SZ),
                ("hidden_begin", SZ), ("vocab_begin", SZ)]


class AttentionShape(C.Structure):
    """AttentionShape (ops.rs:49-56)."""

    _fields_ = [("n_heads", SZ), ("head_dim", SZ), ("seq_len", SZ), ("n_kv_heads", SZ),
                ("sliding_window", SZ)]


class StreamPromptConfig(C.Structure):
    """StreamPromptConfig (stream.rs:4-9); StreamPromptConfig() is the default 32/6/10."""

    _fields_ = [("left_pad_tokens", SZ), ("delay_tokens", SZ), ("eos_extra_tokens", SZ)]

    def __init__(self, left_pad_tokens=32, delay_tokens=6, eos_extra_tokens=10):
        super().__init__(left_pad_tokens, delay_tokens, eos_extra_tokens)

    def right_pad_tokens(self):
        """StreamPromptConfig::right_pad_tokens (stream.rs:21-25)."""
        return int(lib().vox_stream_right_pad_tokens(C.byref(self)))


class TekkenAudioConfig(C.Structure):
    """TekkenAudioConfig (tokenizer.rs:17-23)."""

    _fields_ = [("sampling_rate", C.c_uint32), ("frame_rate", C.c_float), ("transcription_delay_ms", SZ),
                ("streaming_n_left_pad_tokens", SZ)]


class PipelineConfig(C.Structure):
    """PipelineConfig (pipeline.rs:12-18)."""

    _fields_ = [("bos_id", C.c_uint32), ("streaming_pad_id", C.c_uint32), ("samples_per_token", SZ),
                ("prompt", StreamPromptConfig)]


_lib = None

_SIGS = {
    "vox_last_error": ([], C.c_char_p),
    "vox_abi_version": ([], C.c_int),
    "vox_config_validate": ([C.POINTER(DecoderConfig)], C.c_int),
    "vox_layer_weights_validate_f32": ([C.POINTER(DecoderConfig), C.POINTER(LayerWeightsF32)], C.c_int),
    "vox_layer_weights_validate_bf16": ([C.POINTER(DecoderConfig), C.POINTER(LayerWeightsBF16)], C.c_int),
    "vox_ctx_create": ([C.POINTER(DecoderConfig), C.POINTER(CtxOptions), C.POINTER(VP)], C.c_int),
    "vox_ctx_destroy": ([VP], None),
    "vox_ctx_upload_layer_f32": ([VP, SZ, C.POINTER(LayerWeightsF32)], C.c_int),
    "vox_ctx_upload_layer_bf16": ([VP, SZ, C.POINTER(LayerWeightsBF16)], C.c_int),
    "vox_ctx_upload_embed_bf16": ([VP, U16P, SZ], C.c_int),
    "vox_ctx_upload_lm_head_bf16": ([VP, U16P, SZ], C.c_int),
    "vox_ctx_upload_final_norm": ([VP, F32P, SZ], C.c_int),
    "vox_ctx_init_random": ([VP, C.c_uint64, C.c_float], C.c_int),
    "vox_ctx_download_matrix": ([VP, SZ, C.c_int, VP, SZ], C.c_int),
    "vox_ctx_stream": ([VP], VP),
    "vox_ctx_synchronize": ([VP], C.c_int),
    "vox_ctx_record_event": ([VP, C.c_int], C.c_int),
    "vox_ctx_event_elapsed_ms": ([VP, C.c_int, C.c_int, F32P], C.c_int),
    "vox_ctx_kernel_launches": ([VP], C.c_uint64),
    "vox_kv_create": ([VP, SZ, SZ, SZ, SZ, C.POINTER(VP)], C.c_int),
    "vox_kv_create_ex": ([VP, SZ, SZ, SZ, SZ, SZ, C.POINTER(VP)], C.c_int),
    "vox_kv_destroy": ([VP], None),
    "vox_kv_create_streams": ([VP, SZ, SZ, SZ, SZ, SZ, C.POINTER(VP)], C.c_int),
    "vox_kv_n_streams": ([VP, C.POINTER(SZ)], C.c_int),
    "vox_kv_stream": ([VP, SZ, C.POINTER(VP)], C.c_int),
    "vox_kv_fill_random": ([VP, SZ, C.c_uint64, C.c_uint64, C.c_float], C.c_int),
    "vox_model_step_batch": ([VP, VP, I32P, C.POINTER(SZ), I32P, F32P], C.c_int),
    "vox_model_generate_batch": ([VP, VP, I32P, C.POINTER(SZ), SZ, I32P], C.c_int),
    "vox_kv_append_layer": ([VP, SZ, F32P, F32P, SZ], C.c_int),
    "vox_kv_layer_len_tokens": ([VP, SZ, C.POINTER(SZ)], C.c_int),
    "vox_kv_layer_pos_offset": ([VP, SZ, C.POINTER(SZ)], C.c_int),
    "vox_kv_layer_tensors": ([VP, SZ, F32P, F32P, SZ], C.c_int),
    "vox_kv_layer_device_state": ([VP, SZ, C.POINTER(C.c_int64)], C.c_int),
    "vox_kv_reset": ([VP], C.c_int),
    "vox_decoder_layer_forward_step": ([VP, SZ, VP, F32P, SZ, SZ, F32P, SZ], C.c_int),
    "vox_model_step": ([VP, VP, C.c_int32, SZ, I32P, F32P], C.c_int),
    "vox_model_generate": ([VP, VP, C.c_int32, SZ, SZ, I32P], C.c_int),
    "vox_model_prefill": ([VP, VP, I32P, SZ, SZ], C.c_int),
    "vox_model_prefill_steps": ([VP, VP, I32P, SZ, SZ], C.c_int),
    "vox_profile_gemv": ([VP, C.c_int, SZ, F32P, C.POINTER(C.c_uint64)], C.c_int),
    "vox_tp_shard_of": ([C.POINTER(DecoderConfig), SZ, C.c_int, C.c_int, C.POINTER(TpShard)], C.c_int),
    "vox_tp_unique_id": ([C.c_char_p], C.c_int),
    "vox_tp_create": ([C.POINTER(DecoderConfig), C.POINTER(CtxOptions), C.c_int, C.c_int, C.c_char_p,
                       C.POINTER(VP)], C.c_int),
    "vox_tp_destroy": ([VP], None),
    "vox_tp_ipc_handle": ([VP, C.c_char_p], C.c_int),
    "vox_tp_connect_peers": ([VP, C.c_char_p], C.c_int),
    "vox_tp_init_random": ([VP, C.c_uint64, C.c_float], C.c_int),
    "vox_tp_upload_layer_bf16": ([VP, SZ, C.c_void_p], C.c_int),
    "vox_tp_upload_embed_bf16": ([VP, U16P, SZ], C.c_int),
    "vox_tp_upload_lm_head_bf16": ([VP, U16P, SZ, F32P], C.c_int),
    "vox_tp_step": ([VP, C.c_int32, SZ, I32P, F32P], C.c_int),
    "vox_tp_prefill": ([VP, I32P, SZ, SZ], C.c_int),
    "vox_tp_generate": ([VP, C.c_int32, SZ, SZ, I32P], C.c_int),
    "vox_tp_kv_state": ([VP, SZ, C.POINTER(C.c_int64)], C.c_int),
    "vox_tp_reset": ([VP], C.c_int),
    "vox_tp_set_timeout_ms": ([VP, C.c_uint], C.c_int),
    "vox_tp_record_event": ([VP, C.c_int], C.c_int),
    "vox_tp_event_elapsed_ms": ([VP, C.c_int, C.c_int, F32P], C.c_int),
    "vox_tp_kernel_launches": ([VP], C.c_uint64),
    "vox_profile_bgemm": ([VP, C.c_int, SZ, SZ, F32P, C.POINTER(C.c_uint64)], C.c_int),
    "vox_linear_f32": ([VP, F32P, SZ, SZ, F32P, SZ, F32P, F32P], C.c_int),
    "vox_linear_bf16": ([VP, F32P, SZ, SZ, U16P, SZ, F32P, F32P], C.c_int),
    "vox_linear_batched_bf16": ([VP, F32P, SZ, SZ, U16P, SZ, F32P, F32P], C.c_int),
    "vox_add_inplace": ([VP, F32P, F32P, SZ], C.c_int),
    "vox_attention_gqa_step": ([VP, F32P, F32P, F32P, C.POINTER(AttentionShape), F32P], C.c_int),
    "vox_rms_norm_rows": ([VP, F32P, F32P, F32P, SZ, SZ, C.c_float], C.c_int),
    "vox_rope_interleaved_inplace": ([VP, F32P, SZ, SZ, SZ, SZ, C.c_float], C.c_int),
    "vox_silu_inplace": ([VP, F32P, SZ], C.c_int),
    "vox_softmax_inplace": ([VP, F32P, SZ], C.c_int),
    "vox_attention_gqa_step_noalloc": ([VP, VP, VP, C.POINTER(AttentionShape), VP, VP], C.c_int),
    "vox_weights_open": ([C.c_char_p, C.POINTER(VP)], C.c_int),
    "vox_weights_close": ([VP], None),
    "vox_weights_count": ([VP], SZ),
    "vox_weights_name": ([VP, SZ], C.c_char_p),
    "vox_weights_info": ([VP, C.c_char_p, C.POINTER(C.c_int), C.POINTER(SZ), SZ, C.POINTER(SZ)], C.c_int),
    "vox_weights_tensor_f32": ([VP, C.c_char_p, F32P, SZ, C.POINTER(SZ)], C.c_int),
    "vox_ctx_load_checkpoint": ([VP, VP], C.c_int),
    "vox_tekken_from_json": ([C.c_char_p, SZ, C.POINTER(VP)], C.c_int),
    "vox_tekken_from_path": ([C.c_char_p, C.POINTER(VP)], C.c_int),
    "vox_tekken_destroy": ([VP], None),
    "vox_tekken_default_vocab_size": ([VP], SZ),
    "vox_tekken_special_token_count": ([VP], SZ),
    "vox_tekken_special_id": ([VP, C.c_char_p, C.POINTER(C.c_uint32)], C.c_int),
    "vox_tekken_audio": ([VP, C.POINTER(TekkenAudioConfig)], C.c_int),
    "vox_tekken_transcription_delay_tokens": ([VP, C.POINTER(SZ)], C.c_int),
    "vox_tekken_default_prompt_ids": ([VP, C.POINTER(C.c_uint32), SZ, C.POINTER(SZ)], C.c_int),
    "vox_tekken_decode_token_bytes": ([VP, C.c_uint32, C.POINTER(C.POINTER(C.c_uint8)), C.POINTER(SZ)], C.c_int),
    "vox_tekken_decode_to_utf8_lossy": ([VP, C.POINTER(C.c_uint32), SZ, C.c_char_p, SZ], SZ),
    "vox_mel_create": ([C.c_int, SZ, C.POINTER(VP)], C.c_int),
    "vox_mel_destroy": ([VP], None),
    "vox_mel_left_pad_samples": ([VP], SZ),
    "vox_mel_feed": ([VP, F32P, SZ, C.POINTER(SZ)], C.c_int),
    "vox_mel_finish": ([VP, SZ], C.c_int),
    "vox_mel_frames": ([VP], SZ),
    "vox_mel_data": ([VP, SZ, SZ, F32P], C.c_int),
    "vox_conv_stem_create": ([C.c_int, SZ, SZ, F32P, F32P, F32P, F32P, C.POINTER(VP)], C.c_int),
    "vox_conv_stem_destroy": ([VP], None),
    "vox_conv_stem_process": ([VP, F32P, SZ, F32P, SZ, C.POINTER(SZ)], C.c_int),
    "vox_conv_out_len": ([SZ, SZ, SZ], SZ),
    "vox_causal_conv1d_gelu": ([C.c_int, F32P, F32P, F32P, SZ, SZ, SZ, SZ, C.c_int, F32P], C.c_int),
    "vox_encoder_kernel_launches": ([VP, VP], C.c_uint64),
    "vox_stream_prompt_config_default": ([C.POINTER(StreamPromptConfig)], None),
    "vox_stream_right_pad_tokens": ([C.POINTER(StreamPromptConfig)], SZ),
    "vox_stream_build_prompt_ids": ([C.c_uint32, C.c_uint32, C.POINTER(StreamPromptConfig),
                                     C.POINTER(C.c_uint32), SZ], SZ),
    "vox_stream_decode_ready": ([SZ, SZ], C.c_int),
    "vox_stream_decodable_token_budget": ([SZ, SZ], SZ),
    "vox_stream_finish_zero_padding_samples": ([SZ, SZ, C.POINTER(StreamPromptConfig)], SZ),
    "vox_pipeline_create": ([VP, VP, C.POINTER(PipelineConfig), SZ, C.POINTER(VP)], C.c_int),
    "vox_pipeline_destroy": ([VP], None),
    "vox_pipeline_prompt_ids": ([VP, C.POINTER(C.c_uint32), SZ], SZ),
    "vox_pipeline_adapter_tokens_total": ([VP], SZ),
    "vox_pipeline_generated_tokens": ([VP], SZ),
    "vox_pipeline_decodable_now": ([VP], SZ),
    "vox_pipeline_is_finished": ([VP], C.c_int),
    "vox_pipeline_push_adapter_tokens": ([VP, F32P, SZ], C.c_int),
    "vox_pipeline_mark_decoded": ([VP, SZ], C.c_int),
    "vox_pipeline_decode": ([VP, SZ, I32P, C.POINTER(SZ)], C.c_int),
    "vox_pipeline_finish_padding_samples": ([VP, SZ], SZ),
}


def lib():
    """Load libvoxb200.so (build it with voxtral-rust_b200/build.py)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(f"libvoxb200.so not built: run python {os.path.join(_HERE, 'build.py')}")
        L = C.CDLL(LIB_PATH)
        for name, (args, res) in _SIGS.items():
            f = getattr(L, name)
            f.argtypes = args
            f.restype = res
        _lib = L
    return _lib


def header_symbols():
    """Entry points declared in include/vox_decoder.h."""
    import re
    text = open(HEADER_PATH).read()
    return sorted(set(re.findall(r"^\s*(?:const\s+)?[\w\*]+\s+\**(vox_\w+)\s*\(", text, re.M)))


def last_error() -> str:
    return lib().vox_last_error().decode(errors="replace")


def _check(rc: int):
    if rc != OK:
        raise VoxError(rc, last_error())


def _f32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


def _p(a, t=F32P):
    return a.ctypes.data_as(t) if a is not None else None


# ---------------------------------------------------------------------------
# Context (device, stream, weights)
# ---------------------------------------------------------------------------

class Context:
    """A CUDA device plus the decoder weights it holds."""

    def __init__(self, cfg: DecoderConfig, n_layers=1, vocab=0, device=0, max_positions=0,
                 weight_dtype=WEIGHTS_BF16, step_mode=STEP_AUTO):
        self.cfg = cfg
        self.n_layers, self.vocab = n_layers, vocab
        self.weight_dtype = weight_dtype
        opt = CtxOptions(device, n_layers, vocab, max_positions, weight_dtype, step_mode)
        h = VP()
        _check(lib().vox_ctx_create(C.byref(cfg), C.byref(opt), C.byref(h)))
        self.h = h.value
        self._caches = weakref.WeakSet()

    def close(self):
        if getattr(self, "h", None):
            for kv in list(self._caches):
                kv.close()
            lib().vox_ctx_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def __enter__(self):
        return self

    def __exit__(self, *a):
        self.close()

    def upload_layer(self, layer, weights: dict):
        """weights: the nine DecoderLayerWeights tensors (decoder.rs:45-55) as
        numpy arrays; matrices f32 or uint16 bf16 bit patterns."""
        keep = {}
        mats_bf16 = weights["wq"].dtype == np.uint16
        if mats_bf16:
            s = LayerWeightsBF16()
            for n in _NAMES:
                a = weights[n]
                if n in ("attention_norm", "ffn_norm"):
                    a = _f32(a)
                    setattr(s, n, F32Slice(_p(a), a.size))
                else:
                    a = np.ascontiguousarray(a, dtype=np.uint16)
                    setattr(s, n, BF16Slice(_p(a, U16P), a.size))
                keep[n] = a
            _check(lib().vox_ctx_upload_layer_bf16(self.h, layer, C.byref(s)))
        else:
            s = LayerWeightsF32()
            for n in _NAMES:
                a = _f32(weights[n])
                setattr(s, n, F32Slice(_p(a), a.size))
                keep[n] = a
            _check(lib().vox_ctx_upload_layer_f32(self.h, layer, C.byref(s)))

    def upload_embed(self, bits):
        a = np.ascontiguousarray(bits, dtype=np.uint16)
        _check(lib().vox_ctx_upload_embed_bf16(self.h, _p(a, U16P), a.size))

    def upload_lm_head(self, bits):
        a = np.ascontiguousarray(bits, dtype=np.uint16)
        _check(lib().vox_ctx_upload_lm_head_bf16(self.h, _p(a, U16P), a.size))

    def upload_final_norm(self, gain):
        a = _f32(gain)
        _check(lib().vox_ctx_upload_final_norm(self.h, _p(a), a.size))

    def init_random(self, seed=0, std=0.02):
        _check(lib().vox_ctx_init_random(self.h, seed, std))

    MATRIX_IDS = {"wq": 0, "wk": 1, "wv": 2, "wo": 3, "w1": 4, "w2": 5, "w3": 6, "embed": 7, "lm_head": 8}

    def download_matrix(self, layer, name):
        c = self.cfg
        q_dim, kv_dim = c.n_heads * c.head_dim, c.n_kv_heads * c.head_dim
        n = {"wq": q_dim * c.dim, "wk": kv_dim * c.dim, "wv": kv_dim * c.dim, "wo": c.dim * q_dim,
             "w1": c.hidden_dim * c.dim, "w2": c.dim * c.hidden_dim, "w3": c.hidden_dim * c.dim,
             "embed": self.vocab * c.dim, "lm_head": self.vocab * c.dim}[name]
        bf16 = name == "embed" or self.weight_dtype == WEIGHTS_BF16
        out = np.empty(n, np.uint16 if bf16 else np.float32)
        _check(lib().vox_ctx_download_matrix(self.h, layer, self.MATRIX_IDS[name],
                                             out.ctypes.data_as(VP), out.nbytes))
        return out

    def synchronize(self):
        _check(lib().vox_ctx_synchronize(self.h))

    def record_event(self, slot):
        _check(lib().vox_ctx_record_event(self.h, slot))

    def elapsed_ms(self, a, b):
        ms = C.c_float()
        _check(lib().vox_ctx_event_elapsed_ms(self.h, a, b, C.byref(ms)))
        return ms.value

    def profile_gemv(self, which, n_launches):
        """Mean ms per launch and weight bytes per launch of one step GEMV
        (1 o-proj, 2 w1|w3, 3 w2, 4 LM head) timed on its own."""
        ms = C.c_float()
        nb = C.c_uint64()
        _check(lib().vox_profile_gemv(self.h, which, n_launches, C.byref(ms), C.byref(nb)))
        return ms.value, nb.value

    def profile_bgemm(self, which, n_streams, n_launches):
        """Mean ms per launch and weight bytes per launch of one multi-stream
        tensor-core GEMM (1 o-proj, 2 w1|w3, 3 w2, 4 LM head, 5 q|k|v)."""
        ms = C.c_float()
        nb = C.c_uint64()
        _check(lib().vox_profile_bgemm(self.h, which, n_streams, n_launches, C.byref(ms), C.byref(nb)))
        return ms.value, nb.value

    def kernel_launches(self):
        return int(lib().vox_ctx_kernel_launches(self.h))

    # ---- composed token loop ----
    def model_step(self, cache, token, pos, want_logits=False):
        nxt = C.c_int32()
        logits = np.empty(self.vocab, np.float32) if want_logits else None
        _check(lib().vox_model_step(self.h, cache.h, int(token), int(pos), C.byref(nxt), _p(logits)))
        return nxt.value, logits

    def model_prefill(self, cache, tokens, pos0=0):
        """Prefill (tensor-core passes where the shape allows, else token steps)."""
        t = np.ascontiguousarray(tokens, dtype=np.int32)
        _check(lib().vox_model_prefill(self.h, cache.h, _p(t, I32P), t.size, int(pos0)))

    def model_prefill_steps(self, cache, tokens, pos0=0):
        """Prefill as one token step per id."""
        t = np.ascontiguousarray(tokens, dtype=np.int32)
        _check(lib().vox_model_prefill_steps(self.h, cache.h, _p(t, I32P), t.size, int(pos0)))

    def model_generate(self, cache, token, pos, n_steps):
        out = np.empty(n_steps, np.int32)
        _check(lib().vox_model_generate(self.h, cache.h, int(token), int(pos), int(n_steps), _p(out, I32P)))
        return out

    # ---- multi-stream token loop (cache made with n_streams > 1) ----
    @staticmethod
    def _stream_inputs(cache, tokens, positions):
        t = np.ascontiguousarray(tokens, dtype=np.int32)
        p = (SZ * cache.n_streams)(*[int(x) for x in positions])
        if t.size != cache.n_streams or len(positions) != cache.n_streams:
            raise ValueError("need one token and one position per stream")
        return t, p

    def model_step_batch(self, cache, tokens, positions, want_logits=False):
        """One token per stream; returns (next tokens [B], logits [B, vocab] or None)."""
        t, p = self._stream_inputs(cache, tokens, positions)
        nxt = np.empty(cache.n_streams, np.int32)
        logits = np.empty((cache.n_streams, self.vocab), np.float32) if want_logits else None
        _check(lib().vox_model_step_batch(self.h, cache.h, _p(t, I32P), p, _p(nxt, I32P), _p(logits)))
        return nxt, logits

    def model_generate_batch(self, cache, tokens, positions, n_steps):
        """Greedy decode of n_steps per stream; returns ids [n_steps, B]."""
        t, p = self._stream_inputs(cache, tokens, positions)
        out = np.empty((n_steps, cache.n_streams), np.int32)
        _check(lib().vox_model_generate_batch(self.h, cache.h, _p(t, I32P), p, int(n_steps), _p(out, I32P)))
        return out


# ---------------------------------------------------------------------------
# RollingKvCache (kv.rs)
# ---------------------------------------------------------------------------

class RollingKvCache:
    """RollingKvCache (kv.rs:22-101) as a device ring buffer."""

    def __init__(self, ctx: Context, n_layers, n_kv_heads, head_dim, sliding_window, capacity=None,
                 n_streams=1, _view_of=None, _handle=None):
        self.ctx = ctx
        self.n_layers, self.n_kv_heads, self.head_dim = n_layers, n_kv_heads, head_dim
        self.sliding_window = sliding_window
        self.n_streams = n_streams
        self._parent = _view_of
        self._views = {}
        if _view_of is not None:  # stream view: memory owned by the parent cache
            self.h = _handle
            return
        h = VP()
        if n_streams != 1:
            if capacity is not None:
                raise ValueError("multi-stream caches use capacity = sliding_window")
            _check(lib().vox_kv_create_streams(ctx.h, n_streams, n_layers, n_kv_heads, head_dim,
                                               sliding_window, C.byref(h)))
        elif capacity is None:
            _check(lib().vox_kv_create(ctx.h, n_layers, n_kv_heads, head_dim, sliding_window, C.byref(h)))
        else:
            _check(lib().vox_kv_create_ex(ctx.h, n_layers, n_kv_heads, head_dim, sliding_window,
                                          capacity, C.byref(h)))
        self.h = h.value
        ctx._caches.add(self)

    def close(self):
        # A closed context has already freed its caches (vox_ctx_destroy).
        if self._parent is None and getattr(self, "h", None) and getattr(self.ctx, "h", None):
            lib().vox_kv_destroy(self.h)
        for v in self._views.values():
            v.h = None
        self.h = None

    def stream(self, s):
        """Single-stream view of stream s (shares memory; valid while this cache lives)."""
        if self.n_streams == 1 and s == 0:
            return self
        if s not in self._views:
            h = VP()
            _check(lib().vox_kv_stream(self.h, s, C.byref(h)))
            self._views[s] = RollingKvCache(self.ctx, self.n_layers, self.n_kv_heads, self.head_dim,
                                            self.sliding_window, _view_of=self, _handle=h.value)
        return self._views[s]

    def fill_random(self, n_tokens, seed, tensor_id, std=1.0):
        """Fill every layer with n_tokens generator tokens (bf16-rounded N(0, std^2))."""
        _check(lib().vox_kv_fill_random(self.h, n_tokens, seed, tensor_id, std))

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def append_layer(self, layer, k_new, v_new, n_new_tokens):
        k, v = _f32(k_new), _f32(v_new)
        stride = self.n_kv_heads * self.head_dim
        if k.size != n_new_tokens * stride or v.size != n_new_tokens * stride:
            raise ValueError("k_new/v_new must hold n_new_tokens * n_kv_heads * head_dim floats")
        _check(lib().vox_kv_append_layer(self.h, layer, _p(k), _p(v), n_new_tokens))

    def layer_len_tokens(self, layer):
        out = SZ()
        _check(lib().vox_kv_layer_len_tokens(self.h, layer, C.byref(out)))
        return out.value

    def layer_pos_offset(self, layer):
        out = SZ()
        _check(lib().vox_kv_layer_pos_offset(self.h, layer, C.byref(out)))
        return out.value

    def layer_tensors(self, layer):
        n = self.layer_len_tokens(layer) * self.n_kv_heads * self.head_dim
        k = np.empty(n, np.float32)
        v = np.empty(n, np.float32)
        _check(lib().vox_kv_layer_tensors(self.h, layer, _p(k), _p(v), n))
        return k, v

    def device_state(self, layer):
        out = (C.c_int64 * 3)()
        _check(lib().vox_kv_layer_device_state(self.h, layer, out))
        return tuple(out)

    def reset(self):
        _check(lib().vox_kv_reset(self.h))


# ---------------------------------------------------------------------------
# safetensors checkpoints (weights.rs)
# ---------------------------------------------------------------------------

DTYPES = ("BOOL", "U8", "I8", "F8_E5M2", "F8_E4M3", "I16", "U16", "F16", "BF16", "I32", "U32", "F32", "F64",
          "I64", "U64")
CKPT_EMBED = "mm_streams_embeddings.embedding_module.tok_embeddings.weight"
CKPT_LM_HEAD = "output.weight"
CKPT_FINAL_NORM = "norm.weight"


class WeightStore:
    """WeightStore (weights.rs:16-93): a memory-mapped, header-validated
    .safetensors file."""

    def __init__(self, path):
        h = VP()
        _check(lib().vox_weights_open(os.fsencode(path), C.byref(h)))
        self.h = h.value

    @classmethod
    def open(cls, path):
        return cls(path)

    def close(self):
        if getattr(self, "h", None):
            lib().vox_weights_close(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def __enter__(self):
        return self

    def __exit__(self, *a):
        self.close()

    def names(self):
        """names (weights.rs:44-47)."""
        n = lib().vox_weights_count(self.h)
        return [lib().vox_weights_name(self.h, i).decode() for i in range(n)]

    def info(self, name):
        """(dtype name, shape) of a tensor."""
        dt, nd = C.c_int(), SZ()
        shape = (SZ * 16)()
        _check(lib().vox_weights_info(self.h, name.encode(), C.byref(dt), shape, 16, C.byref(nd)))
        return DTYPES[dt.value], [int(shape[i]) for i in range(nd.value)]

    def tensor_f32(self, name):
        """tensor_f32 (weights.rs:49-93): returns (shape, data f32)."""
        n = SZ()
        _check(lib().vox_weights_tensor_f32(self.h, name.encode(), None, 0, C.byref(n)))
        out = np.empty(n.value, np.float32)
        _check(lib().vox_weights_tensor_f32(self.h, name.encode(), _p(out), n.value, C.byref(n)))
        return self.info(name)[1], out


def load_checkpoint(ctx: Context, store: WeightStore):
    """Upload a decoder checkpoint (layers.{l}.*, embedding, final norm, LM
    head or tied embedding) into a context."""
    _check(lib().vox_ctx_load_checkpoint(ctx.h, store.h))


# ---------------------------------------------------------------------------
# Encoder front end (mel.rs, conv.rs) on the GPU
# ---------------------------------------------------------------------------

MEL_BINS = 128


class MelCtx:
    """MelCtx (mel.rs:114-272) on the GPU: incremental log-mel frames [n, 128]."""

    def __init__(self, left_pad_samples=0, device=0):
        h = VP()
        _check(lib().vox_mel_create(device, left_pad_samples, C.byref(h)))
        self.h = h.value

    def close(self):
        if getattr(self, "h", None):
            lib().vox_mel_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def left_pad_samples(self):
        return int(lib().vox_mel_left_pad_samples(self.h))

    def feed(self, samples):
        x = _f32(samples)
        n = SZ()
        _check(lib().vox_mel_feed(self.h, _p(x), x.size, C.byref(n)))
        return n.value

    def finish(self, right_pad_samples=0):
        _check(lib().vox_mel_finish(self.h, int(right_pad_samples)))

    def frames(self):
        return int(lib().vox_mel_frames(self.h))

    def data(self, first=0, n=None):
        """(frames [n, 128], total frame count), as MelCtx::data."""
        total = self.frames()
        n = total - first if n is None else n
        out = np.empty((max(n, 0), MEL_BINS), np.float32)
        if n > 0:
            _check(lib().vox_mel_data(self.h, first, n, _p(out)))
        return out, total


class ConvStemState:
    """ConvStemState (conv.rs:134-347) on the GPU; weights [dim, cin, 3] f32."""

    def __init__(self, mel_bins, dim, conv0_weight, conv0_bias, conv1_weight, conv1_bias, device=0):
        ws = [_f32(conv0_weight), _f32(conv0_bias), _f32(conv1_weight), _f32(conv1_bias)]
        if ws[0].size != dim * mel_bins * 3 or ws[2].size != dim * dim * 3 or ws[1].size != dim or ws[3].size != dim:
            raise ValueError("conv stem weight shapes do not match mel_bins / dim")
        h = VP()
        _check(lib().vox_conv_stem_create(device, mel_bins, dim, *[_p(w) for w in ws], C.byref(h)))
        self.h = h.value
        self.mel_bins, self.dim = mel_bins, dim

    def close(self):
        if getattr(self, "h", None):
            lib().vox_conv_stem_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def process(self, mel_new):
        """New mel frames [n, mel_bins] -> new positions [m, dim]."""
        mel = _f32(mel_new)
        n = mel.size // self.mel_bins
        cap = n // 2 + 1
        out = np.empty((cap, self.dim), np.float32)
        got = SZ()
        _check(lib().vox_conv_stem_process(self.h, _p(mel), n, _p(out), cap, C.byref(got)))
        return out[:got.value].copy()


def causal_conv1d_gelu(x, weight, bias, cin, cout, length, stride, gelu=True, device=0):
    """causal_conv1d_colmajor (conv.rs:28-73), kernel 3, (+ gelu_inplace) on the GPU."""
    n = int(lib().vox_conv_out_len(length, 3, stride))
    out = np.zeros((cout, n), np.float32)
    xx, ww = _f32(x), _f32(weight)
    bb = _f32(bias) if bias is not None else None
    _check(lib().vox_causal_conv1d_gelu(device, _p(xx), _p(ww), _p(bb), cin, cout, length, stride, 1 if gelu else 0,
                                        _p(out)))
    return out


# ---------------------------------------------------------------------------
# Tekken tokenizer decode (tokenizer.rs)
# ---------------------------------------------------------------------------

class TekkenTokenizer:
    """TekkenTokenizer (tokenizer.rs:26-214); Option results are None."""

    def __init__(self, _handle):
        self.h = _handle

    @classmethod
    def from_json_str(cls, text):
        b = text.encode() if isinstance(text, str) else bytes(text)
        h = VP()
        _check(lib().vox_tekken_from_json(b, len(b), C.byref(h)))
        return cls(h.value)

    @classmethod
    def from_path(cls, path):
        h = VP()
        _check(lib().vox_tekken_from_path(os.fsencode(path), C.byref(h)))
        return cls(h.value)

    def close(self):
        if getattr(self, "h", None):
            lib().vox_tekken_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def default_vocab_size(self):
        return int(lib().vox_tekken_default_vocab_size(self.h))

    def special_token_count(self):
        return int(lib().vox_tekken_special_token_count(self.h))

    def special_id(self, text):
        v = C.c_uint32()
        return int(v.value) if lib().vox_tekken_special_id(self.h, text.encode(), C.byref(v)) else None

    def bos_id(self):
        return self.special_id("<s>")

    def eos_id(self):
        return self.special_id("</s>")

    def streaming_pad_id(self):
        return self.special_id("[STREAMING_PAD]")

    def audio(self):
        a = TekkenAudioConfig()
        return a if lib().vox_tekken_audio(self.h, C.byref(a)) else None

    def transcription_delay_tokens(self):
        v = SZ()
        return int(v.value) if lib().vox_tekken_transcription_delay_tokens(self.h, C.byref(v)) else None

    def default_prompt_ids(self):
        n = SZ()
        if not lib().vox_tekken_default_prompt_ids(self.h, None, 0, C.byref(n)):
            return None
        out = (C.c_uint32 * max(n.value, 1))()
        lib().vox_tekken_default_prompt_ids(self.h, out, n.value, C.byref(n))
        return [int(out[i]) for i in range(n.value)]

    def decode_token_bytes(self, token_id):
        p, n = C.POINTER(C.c_uint8)(), SZ()
        if not lib().vox_tekken_decode_token_bytes(self.h, int(token_id) & 0xFFFFFFFF, C.byref(p), C.byref(n)):
            return None
        return bytes(C.string_at(p, n.value)) if n.value else b""

    def decode_to_utf8_lossy(self, token_ids):
        ids = (C.c_uint32 * max(len(token_ids), 1))(*[int(i) & 0xFFFFFFFF for i in token_ids])
        n = lib().vox_tekken_decode_to_utf8_lossy(self.h, ids, len(token_ids), None, 0)
        buf = C.create_string_buffer(n + 1)
        lib().vox_tekken_decode_to_utf8_lossy(self.h, ids, len(token_ids), buf, n + 1)
        return buf.raw[:n].decode("utf-8")


# ---------------------------------------------------------------------------
# Streaming decode driver (stream.rs, pipeline.rs)
# ---------------------------------------------------------------------------

def build_prompt_ids(bos_id, streaming_pad_id, cfg: StreamPromptConfig):
    """build_prompt_ids (stream.rs:26-34)."""
    n = lib().vox_stream_build_prompt_ids(bos_id, streaming_pad_id, C.byref(cfg), None, 0)
    out = (C.c_uint32 * max(n, 1))()
    lib().vox_stream_build_prompt_ids(bos_id, streaming_pad_id, C.byref(cfg), out, n)
    return [int(out[i]) for i in range(n)]


def decode_ready(total_adapter_tokens, prompt_len):
    """decode_ready (stream.rs:36-38)."""
    return bool(lib().vox_stream_decode_ready(total_adapter_tokens, prompt_len))


def decodable_token_budget(total_adapter_tokens, prompt_len):
    """decodable_token_budget (stream.rs:47-53)."""
    return int(lib().vox_stream_decodable_token_budget(total_adapter_tokens, prompt_len))


def finish_zero_padding_samples(consumed_samples, samples_per_token, cfg: StreamPromptConfig):
    """finish_zero_padding_samples (stream.rs:60-69)."""
    return int(lib().vox_stream_finish_zero_padding_samples(consumed_samples, samples_per_token, C.byref(cfg)))


class PipelineState:
    """PipelineState (pipeline.rs:28-90).  Without a context it is the
    reference's planner; with a Context and a single-stream RollingKvCache it
    also decodes: push_adapter_tokens uploads adapter rows [n, dim] to a
    device ring and decode() runs the streaming schedule on the device."""

    def __init__(self, cfg: PipelineConfig, ctx: Context = None, cache: RollingKvCache = None,
                 adapter_capacity=4096):
        h = VP()
        _check(lib().vox_pipeline_create(ctx.h if ctx else None, cache.h if cache else None, C.byref(cfg),
                                         adapter_capacity, C.byref(h)))
        self.h = h.value
        self.ctx, self.cache = ctx, cache
        self.dim = ctx.cfg.dim if ctx else 0

    def close(self):
        if getattr(self, "h", None):
            lib().vox_pipeline_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def __enter__(self):
        return self

    def __exit__(self, *a):
        self.close()

    def prompt_ids(self):
        n = lib().vox_pipeline_prompt_ids(self.h, None, 0)
        out = (C.c_uint32 * max(n, 1))()
        lib().vox_pipeline_prompt_ids(self.h, out, n)
        return [int(out[i]) for i in range(n)]

    def adapter_tokens_total(self):
        return int(lib().vox_pipeline_adapter_tokens_total(self.h))

    def generated_tokens(self):
        return int(lib().vox_pipeline_generated_tokens(self.h))

    def decodable_now(self):
        return int(lib().vox_pipeline_decodable_now(self.h))

    def is_finished(self):
        return bool(lib().vox_pipeline_is_finished(self.h))

    def push_adapter_tokens(self, n_tokens_or_rows):
        """push_adapter_tokens: a count (planner) or adapter rows [n, dim] (decoding pipeline)."""
        if isinstance(n_tokens_or_rows, (int, np.integer)):
            _check(lib().vox_pipeline_push_adapter_tokens(self.h, None, int(n_tokens_or_rows)))
            return
        rows = _f32(n_tokens_or_rows)
        if self.dim == 0 or rows.size % self.dim:
            raise ValueError("adapter rows must be [n, dim] for a pipeline with a context")
        _check(lib().vox_pipeline_push_adapter_tokens(self.h, _p(rows), rows.size // self.dim))

    def mark_decoded(self, n_tokens):
        _check(lib().vox_pipeline_mark_decoded(self.h, int(n_tokens)))

    def decode(self, max_tokens=None):
        """Decode every decodable token (or at most max_tokens) on the device."""
        n = self.decodable_now() if max_tokens is None else int(max_tokens)
        out = np.empty(max(n, 1), np.int32)
        got = SZ()
        _check(lib().vox_pipeline_decode(self.h, n, _p(out, I32P), C.byref(got)))
        return out[:got.value].copy()

    def finish_padding_samples(self, consumed_audio_samples):
        return int(lib().vox_pipeline_finish_padding_samples(self.h, int(consumed_audio_samples)))


# ---------------------------------------------------------------------------
# Tensor-parallel single stream (one process per GPU)
# ---------------------------------------------------------------------------

def tp_shard(cfg: DecoderConfig, vocab, rank, size) -> TpShard:
    """The shard rank `rank` of `size` holds (host only)."""
    out = TpShard()
    _check(lib().vox_tp_shard_of(C.byref(cfg), vocab, rank, size, C.byref(out)))
    return out


def tp_unique_id() -> bytes:
    buf = C.create_string_buffer(128)
    _check(lib().vox_tp_unique_id(buf))
    return buf.raw


def share_tp_unique_id(rank, make=tp_unique_id, group=None) -> bytes:
    """Rank 0 makes the NCCL id; every rank of the torch.distributed group
    receives it (any backend: the id travels as a Python object)."""
    import torch.distributed as dist
    box = [make() if rank == 0 else None]
    dist.broadcast_object_list(box, src=0, group=group)
    uid = box[0]
    if not isinstance(uid, (bytes, bytearray)) or len(uid) != 128:
        raise ValueError("bad NCCL unique id")
    return bytes(uid)


class TensorParallelDecoder:
    """The token loop sharded over tp_size GPUs (one object per rank)."""

    def __init__(self, cfg: DecoderConfig, rank, size, uid: bytes, n_layers, vocab, device=0, max_positions=0):
        self.cfg, self.rank, self.size = cfg, rank, size
        self.n_layers, self.vocab = n_layers, vocab
        self.shard = tp_shard(cfg, vocab, rank, size)
        opt = CtxOptions(device, n_layers, vocab, max_positions, WEIGHTS_BF16, STEP_AUTO)
        h = VP()
        _check(lib().vox_tp_create(C.byref(cfg), C.byref(opt), rank, size, uid, C.byref(h)))
        self.h = h.value

    def close(self):
        if getattr(self, "h", None):
            lib().vox_tp_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def __enter__(self):
        return self

    def __exit__(self, *a):
        self.close()

    def init_random(self, seed=0, std=0.02):
        _check(lib().vox_tp_init_random(self.h, seed, std))

    def connect_peers(self, group=None):
        """Switch the exchange to NVLink peer memory: all-gather every rank's
        CUDA IPC handle over the torch.distributed group, then map them."""
        import torch.distributed as dist
        buf = C.create_string_buffer(64)
        _check(lib().vox_tp_ipc_handle(self.h, buf))
        handles = [None] * self.size
        dist.all_gather_object(handles, buf.raw, group=group)
        _check(lib().vox_tp_connect_peers(self.h, b"".join(handles)))

    def step(self, token, pos, want_logits=False):
        """One collective step; returns (next token, this rank's logit slice)."""
        nxt = C.c_int32()
        logits = np.empty(self.shard.vocab_local, np.float32) if want_logits else None
        _check(lib().vox_tp_step(self.h, int(token), int(pos), C.byref(nxt), _p(logits)))
        return nxt.value, logits

    def prefill(self, tokens, pos0=0):
        t = np.ascontiguousarray(tokens, dtype=np.int32)
        _check(lib().vox_tp_prefill(self.h, _p(t, I32P), t.size, int(pos0)))

    def generate(self, token, pos, n_steps):
        out = np.empty(n_steps, np.int32)
        _check(lib().vox_tp_generate(self.h, int(token), int(pos), int(n_steps), _p(out, I32P)))
        return out

    def kv_state(self, layer):
        out = (C.c_int64 * 3)()
        _check(lib().vox_tp_kv_state(self.h, layer, out))
        return tuple(out)

    def reset(self):
        """Empty the rank's cache (every rank, between the same two steps)."""
        _check(lib().vox_tp_reset(self.h))

    def set_timeout_ms(self, ms):
        """Watchdog bound on every wait of a step (vox_tp_set_timeout_ms)."""
        _check(lib().vox_tp_set_timeout_ms(self.h, int(ms)))

    def record_event(self, slot):
        _check(lib().vox_tp_record_event(self.h, slot))

    def elapsed_ms(self, a, b):
        ms = C.c_float()
        _check(lib().vox_tp_event_elapsed_ms(self.h, a, b, C.byref(ms)))
        return ms.value

    def kernel_launches(self):
        return int(lib().vox_tp_kernel_launches(self.h))


# ---------------------------------------------------------------------------
# decoder.rs / ops.rs / math.rs entry points
# ---------------------------------------------------------------------------

def decoder_layer_forward_step(ctx: Context, layer_idx, cache: RollingKvCache, hidden, pos):
    """decoder_layer_forward_step (decoder.rs:88-155)."""
    h = _f32(hidden)
    out = np.empty(ctx.cfg.dim, np.float32)
    _check(lib().vox_decoder_layer_forward_step(ctx.h, layer_idx, cache.h, _p(h), h.size, int(pos),
                                                _p(out), out.size))
    return out


def linear(ctx: Context, x, n_rows, in_dim, weight, out_dim, bias=None):
    """linear (ops.rs:11-39); weight f32 or uint16 bf16 bits, [out_dim, in_dim]."""
    x = _f32(x)
    out = np.empty(n_rows * out_dim, np.float32)
    b = _f32(bias) if bias is not None else None
    if weight.dtype == np.uint16:
        w = np.ascontiguousarray(weight)
        _check(lib().vox_linear_bf16(ctx.h, _p(x), n_rows, in_dim, _p(w, U16P), out_dim, _p(b), _p(out)))
    else:
        w = _f32(weight)
        _check(lib().vox_linear_f32(ctx.h, _p(x), n_rows, in_dim, _p(w), out_dim, _p(b), _p(out)))
    return out


def linear_batched(ctx: Context, x, n_rows, in_dim, weight, out_dim, bias=None):
    """linear (ops.rs:11-39) for up to 8 rows on the tensor cores; weight uint16 bf16 bits."""
    x = _f32(x)
    out = np.empty(n_rows * out_dim, np.float32)
    b = _f32(bias) if bias is not None else None
    w = np.ascontiguousarray(weight, dtype=np.uint16)
    _check(lib().vox_linear_batched_bf16(ctx.h, _p(x), n_rows, in_dim, _p(w, U16P), out_dim, _p(b), _p(out)))
    return out


def add_inplace(ctx: Context, dst, src):
    """add_inplace (ops.rs:41-46); returns the updated array."""
    d = _f32(dst).copy()
    s = _f32(src)
    if d.size != s.size:
        raise ValueError("length mismatch")
    _check(lib().vox_add_inplace(ctx.h, _p(d), _p(s), d.size))
    return d


def attention_gqa_step(ctx: Context, query, keys, values, shape: AttentionShape):
    """attention_gqa_step (ops.rs:66-132)."""
    q, k, v = _f32(query), _f32(keys), _f32(values)
    out = np.empty(shape.n_heads * shape.head_dim, np.float32)
    _check(lib().vox_attention_gqa_step(ctx.h, _p(q), _p(k), _p(v), C.byref(shape), _p(out)))
    return out


def rms_norm_rows(ctx: Context, x, weight, dim, eps):
    """rms_norm_rows (math.rs:11-27)."""
    x, w = _f32(x), _f32(weight)
    out = np.zeros_like(x)
    _check(lib().vox_rms_norm_rows(ctx.h, _p(out), _p(x), _p(w), x.size, dim, eps))
    return out


def rope_interleaved_inplace(ctx: Context, data, seq_len, n_heads, head_dim, pos_offset, theta):
    """rope_interleaved_inplace (math.rs:30-65); returns the rotated array."""
    d = _f32(data).copy()
    _check(lib().vox_rope_interleaved_inplace(ctx.h, _p(d), seq_len, n_heads, head_dim, pos_offset, theta))
    return d


def silu_inplace(ctx: Context, x):
    """silu_inplace (math.rs:4-9)."""
    d = _f32(x).copy()
    _check(lib().vox_silu_inplace(ctx.h, _p(d), d.size))
    return d


def softmax_inplace(ctx: Context, x):
    """softmax_inplace (math.rs:67-88)."""
    d = _f32(x).copy()
    _check(lib().vox_softmax_inplace(ctx.h, _p(d), d.size))
    return d
