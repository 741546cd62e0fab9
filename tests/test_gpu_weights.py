"""GPU check of checkpoint loading (vox_ctx_load_checkpoint): a safetensors
file written by the test (as the reference's weights.rs test writes its own)
with the checkpoint's tensor names is loaded into a context; the device
holds exactly the file's weights (bf16 matrices bit for bit, f32 matrices
rounded to nearest even) and the token loop matches the oracle run on the
weights the oracle's own reader (weights.rs:49-93 restated) takes from the
same file."""
import numpy as np
import pytest

from oracle.safetensors_io import read_tensor_f32, write_safetensors
from tests.vox_testlib import MATS, assert_logits_close, config_dict, mat_shapes, vox

pytestmark = pytest.mark.gpu

MINI = config_dict(dim=64, hidden_dim=128, n_heads=4, n_kv_heads=2, head_dim=16, sliding_window=8,
                   rope_theta=1e4)
NAMES = {"wq": "attention.wq", "wk": "attention.wk", "wv": "attention.wv", "wo": "attention.wo",
         "w1": "feed_forward.w1", "w2": "feed_forward.w2", "w3": "feed_forward.w3"}


@pytest.fixture(scope="module")
def V():
    return vox()


def write_checkpoint(oracle, path, c, n_layers, vocab, tied=False, f32_mats=False, seed=5):
    shapes = mat_shapes(c)
    tensors = []
    for l in range(n_layers):
        for i, n in enumerate(MATS):
            r, k = shapes[n]
            if f32_mats:
                raw = oracle.gen_normal_f32(seed, 16 * l + i + 1, 0.02, r * k).astype("<f4").tobytes()
                tensors.append((f"layers.{l}.{NAMES[n]}.weight", "F32", [r, k], raw))
            else:
                raw = oracle.gen_normal_bf16(seed, 16 * l + i + 1, 0.02, r * k).astype("<u2").tobytes()
                tensors.append((f"layers.{l}.{NAMES[n]}.weight", "BF16", [r, k], raw))
        for j, nm in enumerate(("attention_norm", "ffn_norm")):  # bf16 gains around 1.0
            z = oracle.bf16_to_f32(oracle.gen_normal_bf16(seed, 900 + 2 * l + j, 0.1, c["dim"]))
            g = oracle.f32_to_bf16(np.float32(1.0) + z)
            tensors.append((f"layers.{l}.{nm}.weight", "BF16", [c["dim"]], g.astype("<u2").tobytes()))
    tensors.append(("mm_streams_embeddings.embedding_module.tok_embeddings.weight", "BF16", [vocab, c["dim"]],
                    oracle.gen_normal_bf16(seed, 1000000, 0.02, vocab * c["dim"]).astype("<u2").tobytes()))
    if not tied:
        tensors.append(("output.weight", "BF16", [vocab, c["dim"]],
                        oracle.gen_normal_bf16(seed, 1000001, 0.02, vocab * c["dim"]).astype("<u2").tobytes()))
    tensors.append(("norm.weight", "F32", [c["dim"]],
                    (1.0 + 0.1 * oracle.gen_normal_f32(seed, 950, 1.0, c["dim"])).astype("<f4").tobytes()))
    write_safetensors(path, tensors, metadata={"format": "pt"})


def oracle_from_file(oracle, path, c, n_layers, vocab):
    """The oracle model on the file's weights as the reference would read them
    (tensor_f32), matrices then held as bf16 (exact for BF16 tensors,
    nearest-even for F32 ones, as the device stores them)."""
    cfg = oracle.config(**c)
    layers = []
    for l in range(n_layers):
        mats = {n: oracle.f32_to_bf16(read_tensor_f32(path, f"layers.{l}.{NAMES[n]}.weight")[1]) for n in MATS}
        an = read_tensor_f32(path, f"layers.{l}.attention_norm.weight")[1]
        fn = read_tensor_f32(path, f"layers.{l}.ffn_norm.weight")[1]
        layers.append(oracle.LayerWeights(an, fn, **mats))
    emb = oracle.f32_to_bf16(read_tensor_f32(path, "mm_streams_embeddings.embedding_module.tok_embeddings.weight")[1])
    try:
        head = oracle.f32_to_bf16(read_tensor_f32(path, "output.weight")[1])
    except KeyError:
        head = emb
    fnorm = read_tensor_f32(path, "norm.weight")[1]
    return oracle.Model(cfg, layers, emb, fnorm, head, vocab), layers, emb, head


@pytest.mark.parametrize("tied,f32_mats", [(False, False), (True, False), (False, True)])
def test_checkpoint_loads_and_decodes(V, oracle, tmp_path, tied, f32_mats):
    c, n_layers, vocab, n_steps = MINI, 2, 300, 14
    path = str(tmp_path / "ckpt.safetensors")
    write_checkpoint(oracle, path, c, n_layers, vocab, tied=tied, f32_mats=f32_mats)
    m, layers, emb, head = oracle_from_file(oracle, path, c, n_layers, vocab)
    ids = oracle.gen_uniform_ids(0, 3000020, vocab, n_steps)
    oc = oracle.RollingKvCache(n_layers, c["n_kv_heads"], c["head_dim"], c["sliding_window"])
    with V.WeightStore(path) as ws, V.Context(V.DecoderConfig(**c), n_layers=n_layers, vocab=vocab) as ctx:
        V.load_checkpoint(ctx, ws)
        for l in range(n_layers):
            for n in MATS:
                assert np.array_equal(ctx.download_matrix(l, n), layers[l].mats[n]), (l, n)
        assert np.array_equal(ctx.download_matrix(0, "embed"), emb)
        assert np.array_equal(ctx.download_matrix(0, "lm_head"), head)
        kv = V.RollingKvCache(ctx, n_layers, c["n_kv_heads"], c["head_dim"], c["sliding_window"])
        for p in range(n_steps):
            tok, logits = ctx.model_step(kv, int(ids[p]), p, want_logits=True)
            ref_logits, ref_tok = m.step(oc, int(ids[p]), p)
            assert_logits_close(logits, ref_logits, f"step {p}")
            assert tok == ref_tok
        kv.close()


def test_checkpoint_errors(V, oracle, tmp_path):
    c = MINI
    path = str(tmp_path / "short.safetensors")
    write_checkpoint(oracle, path, c, 1, 300)
    with V.WeightStore(path) as ws:
        with V.Context(V.DecoderConfig(**c), n_layers=2, vocab=300) as ctx:   # the file has 1 layer
            with pytest.raises(V.VoxError) as e:
                V.load_checkpoint(ctx, ws)
            assert e.value.code == V.ERR_INVALID_ARG and "layers.1." in e.value.message
        with V.Context(V.DecoderConfig(**dict(c, hidden_dim=192)), n_layers=1, vocab=300) as ctx:
            with pytest.raises(V.VoxError) as e:
                V.load_checkpoint(ctx, ws)
            assert e.value.code == V.ERR_SHAPE and "w1" in e.value.message
