"""Host-side logic of the tensor-parallel mode, on CPU: which slice of the
model each rank holds, and the NCCL id exchange over a gloo group of two
ranks (the id itself is faked: no GPU here)."""
import os
import socket

import pytest
import torch.multiprocessing as mp

from tests.vox_testlib import FULL, vox


@pytest.fixture(scope="module")
def V():
    return vox()


@pytest.mark.parametrize("size", [1, 2, 4, 8])
def test_shards_partition_the_model(V, size):
    cfg = V.DecoderConfig(**FULL)
    vocab = 131072
    heads, kv, hid, voc = set(), set(), set(), set()
    for r in range(size):
        s = V.tp_shard(cfg, vocab, r, size)
        assert (s.rank, s.size) == (r, size)
        assert s.n_heads == 32 // size and s.n_kv_heads == 8 // size and s.hidden == 9216 // size
        assert s.vocab == vocab and s.vocab_local == vocab // size
        # a rank's q heads attend to exactly its kv heads (group of 4)
        assert s.q_head_begin // 4 == s.kv_head_begin and s.n_heads == 4 * s.n_kv_heads
        heads |= set(range(s.q_head_begin, s.q_head_begin + s.n_heads))
        kv |= set(range(s.kv_head_begin, s.kv_head_begin + s.n_kv_heads))
        hid |= set(range(s.hidden_begin, s.hidden_begin + s.hidden))
        voc |= set(range(s.vocab_begin, s.vocab_begin + s.vocab_local))
    assert heads == set(range(32)) and kv == set(range(8))
    assert hid == set(range(9216)) and voc == set(range(vocab))


def test_shard_errors(V):
    cfg = V.DecoderConfig(**FULL)
    with pytest.raises(V.VoxError) as e:
        V.tp_shard(cfg, 131072, 0, 3)  # 8 kv heads do not split 3 ways
    assert e.value.code == V.ERR_UNSUPPORTED
    with pytest.raises(V.VoxError) as e:
        V.tp_shard(cfg, 131072, 2, 2)
    assert e.value.code == V.ERR_INVALID_ARG
    with pytest.raises(V.VoxError) as e:
        V.tp_shard(cfg, 131071, 0, 2)  # vocab rows must split evenly
    assert e.value.code == V.ERR_UNSUPPORTED
    bad = V.DecoderConfig(**dict(FULL, sliding_window=0))
    with pytest.raises(V.VoxError) as e:
        V.tp_shard(bad, 131072, 0, 2)  # decoder.rs:22-41 checks first
    assert e.value.code == V.ERR_CONFIG


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _exchange(rank, world, port, q):
    import torch.distributed as dist

    from tests.vox_testlib import vox as _vox
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    V = _vox()
    uid = V.share_tp_unique_id(rank, make=lambda: bytes(range(128)))
    q.put((rank, uid))
    dist.barrier()
    dist.destroy_process_group()


def test_unique_id_reaches_every_rank():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_exchange, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    assert got[0] == got[1] == bytes(range(128))
