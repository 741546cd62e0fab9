"""safetensors checkpoints on the host (no GPU): the reference's own
WeightStore test (weights.rs:141-193, values in tests/golden/) through the
library's C ABI and the oracle's numpy restatement of tensor_f32, both
readers agreeing on random files, and the format errors the safetensors
crate raises."""
import json
import os
import struct

import numpy as np
import pytest

from oracle.safetensors_io import read_tensor_f32, write_safetensors
from tests.vox_testlib import vox

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


@pytest.fixture(scope="module")
def V():
    return vox()


@pytest.fixture(scope="module")
def ref_tests():
    with open(os.path.join(GOLDEN, "reference_unit_tests.json")) as f:
        return json.load(f)


def test_loads_f32_and_bf16_tensors(V, ref_tests, tmp_path):
    t = ref_tests["loads_f32_and_bf16_tensors"]  # weights.rs:141-193
    a = np.array(t["a"]["values"], "<f4").tobytes()
    b = np.array(t["b"]["words"], "<u2").tobytes()
    path = str(tmp_path / "basic.safetensors")
    write_safetensors(path, [("a", "F32", t["a"]["shape"], a), ("b", "BF16", t["b"]["shape"], b)])
    with V.WeightStore.open(path) as ws:
        names = ws.names()
        assert "a" in names and "b" in names
        shape, data = ws.tensor_f32("a")
        assert shape == t["a"]["shape"] and data.tolist() == t["a"]["values"]
        shape, data = ws.tensor_f32("b")
        assert shape == t["b"]["shape"] and len(data) == 2
        assert np.max(np.abs(data - np.array(t["b"]["expect"], np.float32))) < t["b"]["tol"]
    # the oracle's restatement agrees
    assert read_tensor_f32(path, "a")[1].tolist() == t["a"]["values"]
    assert read_tensor_f32(path, "b")[1].tolist() == t["b"]["expect"]


def test_random_files_match_oracle_reader(V, tmp_path):
    rng = np.random.default_rng(3)
    tensors = []
    for i in range(12):
        shape = [int(x) for x in rng.integers(0, 7, int(rng.integers(0, 4)))]
        n = int(np.prod(shape)) if shape else 1
        if i % 3 == 0:
            raw = rng.standard_normal(n).astype("<f4").tobytes()
            dt = "F32"
        elif i % 3 == 1:
            raw = rng.integers(0, 65536, n).astype("<u2").tobytes()
            dt = "BF16"
        else:
            raw = rng.integers(0, 255, n * 4).astype(np.uint8).tobytes()
            dt = "I32"
        tensors.append((f"t{i}.weight", dt, shape, raw))
    path = str(tmp_path / "rand.safetensors")
    write_safetensors(path, tensors, metadata={"format": "pt"})
    with V.WeightStore(path) as ws:
        assert sorted(ws.names()) == sorted(t[0] for t in tensors)
        for name, dt, shape, raw in tensors:
            assert ws.info(name) == (dt, shape)
            if dt == "I32":
                with pytest.raises(V.VoxError) as e:
                    ws.tensor_f32(name)
                assert e.value.code == V.ERR_FORMAT and "unsupported dtype" in e.value.message
                continue
            got_shape, got = ws.tensor_f32(name)
            ref_shape, ref = read_tensor_f32(path, name)
            assert got_shape == ref_shape
            assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))  # bit-exact, NaNs included
        with pytest.raises(V.VoxError) as e:
            ws.tensor_f32("missing")
        assert e.value.code == V.ERR_INVALID_ARG


def _raw_file(path, header_bytes, data=b"", length=None):
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(header_bytes) if length is None else length))
        f.write(header_bytes)
        f.write(data)


def test_format_errors(V, tmp_path):
    p = str(tmp_path / "bad.safetensors")
    with pytest.raises(V.VoxError) as e:
        V.WeightStore(str(tmp_path / "absent.safetensors"))
    assert e.value.code == V.ERR_IO
    cases = [
        (lambda: open(p, "wb").write(b"\x01\x02"), "shorter"),                                   # < 8 bytes
        (lambda: _raw_file(p, b"{}", length=10 ** 9), "too large"),                             # > 1e8
        (lambda: _raw_file(p, b"{}", length=64), "beyond the file"),
        (lambda: _raw_file(p, b"[1,2]   "), "start with"),
        (lambda: _raw_file(p, b'{"a":{"dtype":"F32","shape":[2],"data_offsets":[0,8]}'), "JSON"),
        (lambda: _raw_file(p, b'{"a":{"dtype":"F32","shape":[2],"data_offsets":[0,4]}}', b"\0" * 4), "need"),
        (lambda: _raw_file(p, b'{"a":{"dtype":"F32","shape":[1],"data_offsets":[4,8]}}', b"\0" * 8), "offset"),
        (lambda: _raw_file(p, b'{"a":{"dtype":"F32","shape":[1],"data_offsets":[0,4]}}', b"\0" * 8), "cover"),
        (lambda: _raw_file(p, b'{"a":{"dtype":"Q4","shape":[1],"data_offsets":[0,1]}}', b"\0"), "unknown dtype"),
        (lambda: _raw_file(p, b'{"a":{"dtype":"F32","shape":[-1],"data_offsets":[0,4]}}', b"\0" * 4), "shape"),
    ]
    for make, msg in cases:
        make()
        with pytest.raises(V.VoxError) as e:
            V.WeightStore(p)
        assert e.value.code == V.ERR_FORMAT, msg
        assert msg in e.value.message, (msg, e.value.message)
    # an empty checkpoint and a metadata-only header are valid
    _raw_file(p, b'{"__metadata__":{"k":"v"}}')
    with V.WeightStore(p) as ws:
        assert ws.names() == []
