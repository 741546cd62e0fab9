"""GPU test of vox_attention_gqa_step_noalloc, the attention entry point for
callers that cannot allocate device memory (their memory comes from a pool
or arena they manage, or a fixed budget).  It is called through the C ABI on
device buffers that the test itself allocates with torch, and its output
must match the host-buffer entry point vox_attention_gqa_step within the
attention tolerance of the other tests, on two calls in a row with
different shapes (the second call must not see the first call's leftovers
in the shared scratch array).

This file is named to be collected last."""
import ctypes as C

import numpy as np
import pytest

from tests.vox_testlib import vox

pytestmark = pytest.mark.gpu

ATTN_TOL = 1e-4  # same bound as test_gpu_ops.test_attention_matches_oracle


def _run_noalloc(V, torch, q, k_tok, v_tok, shape):
    """k_tok/v_tok are the reference layout [seq, n_kv, hd]; the entry point
    takes head-major [n_kv, seq, hd] device buffers."""
    seq, nkv, hd = shape.seq_len, shape.n_kv_heads, shape.head_dim
    dev = torch.device("cuda", 0)
    kh = np.ascontiguousarray(k_tok.reshape(seq, nkv, hd).transpose(1, 0, 2))
    vh = np.ascontiguousarray(v_tok.reshape(seq, nkv, hd).transpose(1, 0, 2))
    dq = torch.from_numpy(q).to(dev)
    dk = torch.from_numpy(kh).to(dev)
    dv = torch.from_numpy(vh).to(dev)
    dout = torch.full((shape.n_heads * hd,), float("nan"), dtype=torch.float32, device=dev)
    stream = torch.cuda.current_stream(dev).cuda_stream
    torch.cuda.synchronize(dev)
    rc = V.lib().vox_attention_gqa_step_noalloc(C.c_void_p(dq.data_ptr()), C.c_void_p(dk.data_ptr()),
                                                C.c_void_p(dv.data_ptr()), C.byref(shape),
                                                C.c_void_p(dout.data_ptr()), C.c_void_p(stream))
    assert rc == 0, V.last_error()
    torch.cuda.synchronize(dev)
    return dout.cpu().numpy()


def test_noalloc_attention_matches_allocating_entry_point():
    torch = pytest.importorskip("torch")
    V = vox()
    cfg = V.DecoderConfig(dim=8, hidden_dim=16, n_heads=2, n_kv_heads=1, head_dim=4, sliding_window=4,
                          norm_eps=1e-5, rope_theta=1e4)
    rng = np.random.default_rng(123)
    cases = [(32, 8, 128, 1536, 8192), (32, 8, 128, 700, 300)]  # decode shape, then a masked one
    with V.Context(cfg) as ctx:
        for nh, nkv, hd, seq, win in cases:
            q = rng.standard_normal(nh * hd).astype(np.float32)
            k = rng.standard_normal(seq * nkv * hd).astype(np.float32)
            v = rng.standard_normal(seq * nkv * hd).astype(np.float32)
            shape = V.AttentionShape(nh, hd, seq, nkv, win)
            want = V.attention_gqa_step(ctx, q, k, v, shape)
            got = _run_noalloc(V, torch, q, k, v, shape)
            assert np.all(np.isfinite(got))
            assert np.max(np.abs(got - want)) < ATTN_TOL


def test_noalloc_rejects_shapes_beyond_its_scratch():
    V = vox()
    shape = V.AttentionShape(4096, 256, 16, 4096, 0)  # one split alone needs ~4 MiB
    dummy = C.c_void_p(16)  # never dereferenced: the size check comes first
    rc = V.lib().vox_attention_gqa_step_noalloc(dummy, dummy, dummy, C.byref(shape), dummy, None)
    assert rc == V.ERR_UNSUPPORTED
    assert "1 MiB" in V.last_error()
