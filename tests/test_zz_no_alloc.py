"""GPU test of vox_attention_gqa_step_noalloc, the attention entry point for
callers that cannot allocate device memory (their memory comes from a pool
or arena they manage, or a fixed budget).  It is called through the C ABI on
device buffers that the test itself allocates with torch, and its output
must match the host-buffer entry point vox_attention_gqa_step and the CPU
oracle within the attention tolerance of the other tests, on two calls in a
row for each of several shapes (a call must not see the previous call's
leftovers in the shared scratch array).

This file is named to be collected last."""
import ctypes as C

import numpy as np
import pytest

from tests.vox_testlib import vox

pytestmark = pytest.mark.gpu

ATTN_TOL = 1e-4  # same bound as test_gpu_ops.test_attention_matches_oracle


def _run_noalloc(V, torch, q, k_tok, v_tok, shape):
    """k_tok/v_tok are the reference layout [seq, n_kv, hd]; the entry point
    takes head-major [n_kv, seq, hd] device buffers.  With seq_len 0 the key
    and value pointers are null."""
    seq, nkv, hd = shape.seq_len, shape.n_kv_heads, shape.head_dim
    dev = torch.device("cuda", 0)
    dq = torch.from_numpy(q).to(dev)
    dk = dv = None
    if seq:
        kh = np.ascontiguousarray(k_tok.reshape(seq, nkv, hd).transpose(1, 0, 2))
        vh = np.ascontiguousarray(v_tok.reshape(seq, nkv, hd).transpose(1, 0, 2))
        dk = torch.from_numpy(kh).to(dev)
        dv = torch.from_numpy(vh).to(dev)
    dout = torch.full((shape.n_heads * hd,), float("nan"), dtype=torch.float32, device=dev)
    stream = torch.cuda.current_stream(dev).cuda_stream
    torch.cuda.synchronize(dev)
    ptr = (lambda t: C.c_void_p(t.data_ptr() if t is not None else 0))
    rc = V.lib().vox_attention_gqa_step_noalloc(ptr(dq), ptr(dk), ptr(dv), C.byref(shape), ptr(dout),
                                                C.c_void_p(stream))
    assert rc == 0, V.last_error()
    torch.cuda.synchronize(dev)
    return dout.cpu().numpy()


# (n_heads, n_kv_heads, head_dim, seq_len, sliding_window): the model's decode
# shape; a masked window; 64 q heads, whose full split count would not fit the
# 1 MiB array (the entry point lowers it); an empty cache (output all zeros).
CASES = [(32, 8, 128, 1536, 8192), (32, 8, 128, 700, 300), (64, 8, 128, 2500, 0), (32, 8, 128, 0, 8192)]


def test_noalloc_attention_matches_allocating_entry_point_and_oracle(oracle):
    torch = pytest.importorskip("torch")
    V = vox()
    cfg = V.DecoderConfig(dim=8, hidden_dim=16, n_heads=2, n_kv_heads=1, head_dim=4, sliding_window=4,
                          norm_eps=1e-5, rope_theta=1e4)
    rng = np.random.default_rng(123)
    with V.Context(cfg) as ctx:
        for nh, nkv, hd, seq, win in CASES:
            q = rng.standard_normal(nh * hd).astype(np.float32)
            k = rng.standard_normal(seq * nkv * hd).astype(np.float32)
            v = rng.standard_normal(seq * nkv * hd).astype(np.float32)
            shape = V.AttentionShape(nh, hd, seq, nkv, win)
            ref = oracle.attention_gqa_step(q, k, v, nh, hd, seq, nkv, win)
            want = V.attention_gqa_step(ctx, q, k, v, shape)
            for _ in range(2):  # two calls in a row share the array
                got = _run_noalloc(V, torch, q, k, v, shape)
                assert np.all(np.isfinite(got)), (nh, seq)
                assert np.max(np.abs(got - want)) < ATTN_TOL, (nh, seq)
                assert np.max(np.abs(got - ref)) < ATTN_TOL, (nh, seq)
            if seq == 0:
                assert np.array_equal(got, np.zeros_like(got))


def test_noalloc_rejects_shapes_beyond_its_scratch():
    V = vox()
    shape = V.AttentionShape(4096, 256, 16, 4096, 0)  # one split alone needs ~4 MiB
    dummy = C.c_void_p(16)  # never dereferenced: the size check comes first
    rc = V.lib().vox_attention_gqa_step_noalloc(dummy, dummy, dummy, C.byref(shape), dummy, None)
    assert rc == V.ERR_UNSUPPORTED
    assert "1 MiB" in V.last_error()
