"""Shared helpers for the parity tests: load the CUDA package, build oracle
models from the same seeded generator the library uses, and compare."""
from __future__ import annotations

import importlib
import os

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

# Logit tolerance of the token loop: max-abs 2e-2 and relative 1e-2 (relative
# to the largest |logit|), BF16 weights with f32 accumulation.
LOGIT_ATOL = 2e-2
LOGIT_RTOL = 1e-2

# Tensor ids of the library's counter-based generator (vox_ctx_init_random).
MATS = ("wq", "wk", "wv", "wo", "w1", "w2", "w3")
EMBED_ID, HEAD_ID = 1000000, 1000001


def vox():
    return importlib.import_module("voxtral-rust_b200")


def cuda_available() -> bool:
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False


def config_dict(dim=3072, hidden_dim=9216, n_heads=32, n_kv_heads=8, head_dim=128, sliding_window=8192,
                norm_eps=1e-5, rope_theta=1e6):
    return dict(dim=dim, hidden_dim=hidden_dim, n_heads=n_heads, n_kv_heads=n_kv_heads,
                head_dim=head_dim, sliding_window=sliding_window, norm_eps=norm_eps,
                rope_theta=rope_theta)


FULL = config_dict()


def mat_shapes(c):
    q, kv = c["n_heads"] * c["head_dim"], c["n_kv_heads"] * c["head_dim"]
    return {"wq": (q, c["dim"]), "wk": (kv, c["dim"]), "wv": (kv, c["dim"]), "wo": (c["dim"], q),
            "w1": (c["hidden_dim"], c["dim"]), "w2": (c["dim"], c["hidden_dim"]),
            "w3": (c["hidden_dim"], c["dim"])}


def oracle_layer(o, c, layer, seed=0, std=0.02, f32=False):
    """The weights vox_ctx_init_random puts on the device, made on the CPU."""
    shapes = mat_shapes(c)
    mats = {}
    for i, n in enumerate(MATS):
        r, k = shapes[n]
        tid = 16 * layer + i + 1
        mats[n] = o.gen_normal_f32(seed, tid, std, r * k) if f32 else o.gen_normal_bf16(seed, tid, std, r * k)
    ones = np.ones(c["dim"], np.float32)
    return o.LayerWeights(ones, ones, **mats)


def oracle_model(o, c, n_layers, vocab, seed=0, std=0.02):
    layers = [oracle_layer(o, c, l, seed, std) for l in range(n_layers)]
    emb = o.gen_normal_bf16(seed, EMBED_ID, std, vocab * c["dim"])
    head = o.gen_normal_bf16(seed, HEAD_ID, std, vocab * c["dim"])
    cfg = o.config(**c)
    return o.Model(cfg, layers, emb, np.ones(c["dim"], np.float32), head, vocab)


def assert_logits_close(got, ref, what=""):
    d = np.abs(got.astype(np.float64) - ref.astype(np.float64))
    scale = max(float(np.max(np.abs(ref))), 1e-30)
    assert np.all(np.isfinite(got)), f"{what}: non-finite values"
    assert float(d.max()) <= LOGIT_ATOL, f"{what}: max abs diff {d.max():.3e} > {LOGIT_ATOL}"
    assert float(d.max()) / scale <= LOGIT_RTOL, f"{what}: rel diff {d.max() / scale:.3e} > {LOGIT_RTOL}"
    return float(d.max())


def top2_margin(logits):
    i = int(np.argmax(logits))
    rest = np.delete(logits, i)
    return float(logits[i] - rest.max())


def kv_index_after_append(len_tokens, start, pos_offset, n_new, window, cap):
    """kv.rs:48-88 on indices only: drop = len + n - window (saturating); keep =
    len - drop (saturating; 0 clears); pos_offset += drop; len += n.  The
    physical start slot of the device ring advances by the tokens dropped
    that were present.  Returns (len_tokens, start, pos_offset)."""
    if n_new == 0:
        return len_tokens, start, pos_offset
    drop = max(0, len_tokens + n_new - window)
    if drop > 0:
        keep = max(0, len_tokens - drop)
        start = (start + min(len_tokens, drop)) % cap
        len_tokens = keep
        pos_offset += drop
    return len_tokens + n_new, start, pos_offset
