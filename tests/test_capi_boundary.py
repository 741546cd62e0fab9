"""CPU tests of the C-ABI boundary: the library loads, exports every symbol
the header declares, and the host-only checks (config and weight validation,
error reporting) behave like the reference's Result paths.  No kernel runs."""
import ctypes as C

import numpy as np
import pytest

from tests.vox_testlib import cuda_available, vox


@pytest.fixture(scope="module")
def V():
    return vox()


def test_library_exports_every_header_symbol(V):
    syms = V.header_symbols()
    assert len(syms) >= 38
    L = V.lib()
    missing = [s for s in syms if not hasattr(L, s)]
    assert not missing, missing
    assert V.lib().vox_abi_version() == 1


def test_header_and_binding_table_agree(V):
    assert set(V.header_symbols()) == set(V._SIGS)


def cfg(V, **kw):
    base = dict(dim=8, hidden_dim=16, n_heads=2, n_kv_heads=1, head_dim=4, sliding_window=4,
                norm_eps=1e-5, rope_theta=1e4)
    base.update(kw)
    return V.DecoderConfig(**base)


@pytest.mark.parametrize("field,value,msg", [
    ("dim", 0, "dim must be > 0"),
    ("hidden_dim", 0, "hidden_dim must be > 0"),
    ("n_heads", 0, "n_heads must be > 0"),
    ("n_kv_heads", 0, "n_kv_heads must be > 0"),
    ("head_dim", 0, "head_dim must be > 0"),
    ("n_kv_heads", 3, "n_heads must be divisible by n_kv_heads"),
    ("head_dim", 2, "n_heads * head_dim must cover dim"),
    ("sliding_window", 0, "sliding_window must be > 0 for rolling attention cache"),
])
def test_config_validate_matches_reference_messages(V, field, value, msg):
    # decoder.rs:22-41
    c = cfg(V, **{field: value})
    with pytest.raises(V.VoxError) as e:
        c.validate()
    assert e.value.code == V.ERR_CONFIG
    assert e.value.message == msg
    cfg(V).validate()


def test_weight_validation_names_the_tensor(V):
    # decoder.rs:58-84: first mismatching tensor is reported by name
    c = cfg(V)
    q, kv = 8, 4
    sizes = dict(attention_norm=8, wq=q * 8, wk=kv * 8, wv=kv * 8, wo=8 * q, ffn_norm=8,
                 w1=16 * 8, w2=8 * 16, w3=16 * 8)
    arrays = {n: np.zeros(s, np.float32) for n, s in sizes.items()}
    s = V.LayerWeightsF32()
    for n, a in arrays.items():
        setattr(s, n, V.F32Slice(a.ctypes.data_as(V.F32P), a.size))
    assert V.lib().vox_layer_weights_validate_f32(C.byref(c), C.byref(s)) == 0
    bad = np.zeros(sizes["w2"] - 1, np.float32)
    s.w2 = V.F32Slice(bad.ctypes.data_as(V.F32P), bad.size)
    assert V.lib().vox_layer_weights_validate_f32(C.byref(c), C.byref(s)) == V.ERR_SHAPE
    assert V.last_error() == "w2 shape mismatch"


@pytest.mark.skipif(cuda_available(), reason="checks the no-GPU error path")
def test_ctx_create_without_gpu_fails_loudly(V):
    with pytest.raises(V.VoxError) as e:
        V.Context(cfg(V))
    assert e.value.code in (V.ERR_CUDA, V.ERR_INVALID_ARG)
