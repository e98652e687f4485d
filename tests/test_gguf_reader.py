"""The GGUF reader (strata_mlx_b200/gguf.py) on files written by gguf-py's own writer, and Q6_K's three parts against
gguf-py's dequantizer (the reference's tests/test_dense.py:27-37 and tests/test_gguf.py). No GPU."""

import os

import gguf
import numpy as np
import pytest
from gguf import GGMLQuantizationType as Q

from strata_mlx_b200 import gguf as G
from strata_mlx_b200.synthetic import blocks_numpy


def q6k_bytes(rows, cols, seed=0):
    rng = np.random.default_rng(seed)
    n = rows * cols // 256
    b = rng.integers(0, 256, (n, 210), dtype=np.uint8)
    b[:, 208:210] = rng.uniform(-0.01, 0.01, (n, 1)).astype("<f2").view(np.uint8)
    return b.reshape(rows, -1)


@pytest.fixture(scope="module")
def written(tmp_path_factory):
    rng = np.random.default_rng(1)
    path = str(tmp_path_factory.mktemp("gguf") / "model.gguf")
    w = gguf.GGUFWriter(path, "test")
    w.add_uint32("test.count", 7)
    w.add_string("test.name", "experts")
    w.add_array("test.list", [1, 2, 3])
    t = {
        "q6k": (q6k_bytes(12, 1024), Q.Q6_K),
        "iq3s": (blocks_numpy("IQ3_S", 4, 16, 512, rng).reshape(4, 16, -1), Q.IQ3_S),
        "q8": (blocks_numpy("Q8_0", 1, 8, 256, rng).reshape(8, -1), Q.Q8_0),
        "f16": (rng.standard_normal((6, 64)).astype(np.float16), None),
        "f32": (rng.standard_normal((3, 32)).astype(np.float32), None),
    }
    for name, (a, q) in t.items():
        if q is None:
            w.add_tensor(name, a)
        else:
            w.add_tensor(name, a, raw_dtype=q)
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()
    return path, t


def test_the_reader_gives_every_tensor_its_bytes_shape_and_type(written):
    path, t = written
    f = G.GGUF(path)
    assert f.version == 3
    assert f.metadata["test.count"] == 7 and f.metadata["test.name"] == "experts" and f.metadata["test.list"] == [1, 2, 3]
    shapes = {"q6k": (12, 1024), "iq3s": (4, 16, 512), "q8": (8, 256), "f16": (6, 64), "f32": (3, 32)}
    types = {"q6k": "Q6_K", "iq3s": "IQ3_S", "q8": "Q8_0", "f16": "F16", "f32": "F32"}
    assert list(f.tensors) == list(t)
    for name, (a, _) in t.items():
        got = f[name]
        assert got.shape == shapes[name] and got.type == types[name] and name in f
        assert np.array_equal(got.data, np.ascontiguousarray(a).view(np.uint8).reshape(-1))
        assert got.quantized == (types[name] not in ("F16", "F32"))
    assert np.array_equal(G.to_float(f["f16"]), t["f16"][0].astype(np.float32))
    assert np.array_equal(G.to_float(f["f32"]), t["f32"][0])


def test_the_parts_are_the_weights(written):
    f = G.GGUF(written[0])
    t = f["q6k"]
    codes, scales, d = G.q6k_parts(t)
    assert codes.dtype == np.int8 and scales.dtype == np.int8 and d.dtype == np.float16
    assert codes.shape == (12, 1024) and scales.shape == (12, 64) and d.shape == (12, 4)
    assert codes.min() >= -32 and codes.max() <= 31
    want = gguf.quants.dequantize(t.data.reshape(12, -1), Q.Q6_K).reshape(t.shape)
    w = codes.astype(np.float64) * np.repeat(scales, 16, 1) * np.repeat(d.astype(np.float64), 256, 1)
    assert np.abs(w - want).max() <= 1e-6 * np.abs(want).max()
    np.testing.assert_array_equal(G.to_float(t), want)  # the same float32 operations: the same bits


def test_shards_of_a_split_file_and_of_one_file():
    assert G.shards("/m/a-00002-of-00003.gguf") == [f"/m/a-0000{i}-of-00003.gguf" for i in (1, 2, 3)]
    assert G.shards("/m/a.gguf") == ["/m/a.gguf"]


def test_a_file_that_is_not_gguf_is_refused(tmp_path):
    p = tmp_path / "x.gguf"
    p.write_bytes(b"NOPE" + bytes(64))
    with pytest.raises(ValueError, match="not a GGUF"):
        G.GGUF(str(p))


def test_the_type_table_has_every_block_type_the_kernels_take():
    from strata_mlx_b200._lib import KINDS

    names = {v[0]: v for v in G.TYPES.values()}
    for kind in KINDS:
        assert kind in names
    assert names["Q2_0"] == ("Q2_0", 64, 18) and names["Q6_K"] == ("Q6_K", 256, 210)
