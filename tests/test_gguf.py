"""The GGUF reader (ef_gguf_*, gguf.py) on files written by gguf-py 0.19.0
(an independent writer of the format): metadata values, the tensor table,
tensor bytes; the structural checks of the reference's parser (js/gguf.js
:324-438) on damaged files; and, on the GPU, weights loaded from a file that
dequantize to the CPU decoder's values."""
import struct

import numpy as np
import pytest
import torch

import gguf as gg
import oracle
from elffuss_engine_b200 import formats
from elffuss_engine_b200._lib import EfError
from elffuss_engine_b200.gguf import GGUFFile


def _write(path, tensors, meta=True, alignment=None):
    w = gg.GGUFWriter(str(path), "llama")
    if alignment:
        w.add_custom_alignment(alignment)
    if meta:
        w.add_uint32("test.u32", 7)
        w.add_int64("test.i64", -5)
        w.add_float32("test.f32", 0.25)
        w.add_bool("test.bool", True)
        w.add_string("test.str", "hola")
        w.add_array("test.arr", [1, 2, 3])
        w.add_array("test.strs", ["a", "bc"])
    for name, t, raw, rows, k in tensors:
        w.add_tensor(name, raw.reshape(rows, -1), raw_dtype=gg.GGMLQuantizationType[t])   # [rows][row bytes]
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()


def _tensors():
    out = []
    for i, (t, rows, k) in enumerate([("Q8_0", 48, 256), ("Q4_K", 40, 512), ("Q6_K", 16, 256), ("IQ2_XXS", 8, 256),
                                      ("Q4_0", 24, 128), ("Q5_K", 17, 512), ("Q2_K", 9, 256), ("IQ1_S", 5, 256)]):
        out.append((f"blk.{i}.w", t, formats.synth(t, rows, k, seed=i), rows, k))
    return out


def test_reads_metadata_table_and_bytes(tmp_path):
    p = tmp_path / "m.gguf"
    ts = _tensors()
    _write(p, ts)
    f = GGUFFile(p)
    assert f.version == 3 and f.alignment == 32
    assert f.meta["general.architecture"] == "llama"
    assert f.meta["test.u32"] == 7 and f.meta["test.i64"] == -5 and f.meta["test.f32"] == 0.25
    assert f.meta["test.bool"] is True and f.meta["test.str"] == "hola"
    assert f.meta["test.arr"] == [1, 2, 3] and f.meta["test.strs"] == ("string[]", 2)
    assert [t.name for t in f.tensors] == [n for n, *_ in ts]
    for (name, t, raw, rows, k) in ts:
        info = f.by_name[name]
        assert formats.type_name(info.type_id) == t and info.k == k and info.rows == rows
        assert info.nbytes == formats.tensor_bytes(t, rows, k)
        assert info.file_offset % 32 == 0
        assert f.tensor_bytes(name) == raw.tobytes()
    f.close()


def test_custom_alignment(tmp_path):
    p = tmp_path / "a.gguf"
    _write(p, _tensors()[:2], meta=False, alignment=64)
    f = GGUFFile(p)
    assert f.alignment == 64 and all(t.file_offset % 64 == 0 for t in f.tensors)
    assert f.tensor_bytes("blk.1.w") == _tensors()[1][2].tobytes()


def _damage(tmp_path, fn):
    p = tmp_path / "ok.gguf"
    _write(p, _tensors()[:1])
    b = bytearray(p.read_bytes())
    fn(b)
    q = tmp_path / "bad.gguf"
    q.write_bytes(bytes(b))
    return q


@pytest.mark.parametrize("what,fn,msg", [
    ("magic", lambda b: b.__setitem__(slice(0, 4), b"GGUX"), "magic"),
    ("version 1", lambda b: b.__setitem__(slice(4, 8), struct.pack("<I", 1)), "GGUFv1"),
    ("big-endian", lambda b: b.__setitem__(slice(4, 8), struct.pack(">I", 3)), "big-endian"),
    ("truncated", lambda b: b.__delitem__(slice(len(b) - 100, len(b))), "past the end"),
    ("header cut", lambda b: b.__delitem__(slice(30, len(b))), "truncated"),
])
def test_structural_checks(tmp_path, what, fn, msg):
    with pytest.raises(EfError, match=msg):
        GGUFFile(_damage(tmp_path, fn))


def test_offset_must_be_the_running_sum(tmp_path):
    p = tmp_path / "o.gguf"
    _write(p, _tensors()[:2], meta=False)
    b = bytearray(p.read_bytes())
    name = b"blk.1.w"
    at = b.index(name) + len(name)                 # then n_dims u32, 2 dims u64, type i32, offset u64
    off_at = at + 4 + 16 + 4
    struct.pack_into("<Q", b, off_at, struct.unpack_from("<Q", b, off_at)[0] + 32)
    q = tmp_path / "o2.gguf"
    q.write_bytes(bytes(b))
    with pytest.raises(EfError, match="expected"):
        GGUFFile(q)


@pytest.mark.gpu
def test_weights_from_file_dequantize_exactly(tmp_path, ops):
    p = tmp_path / "w.gguf"
    ts = _tensors()
    _write(p, ts)
    f = GGUFFile(p)
    for (name, t, raw, rows, k) in ts:
        w = f.load_weight(ops, name)
        got = ops.dequant(t, w, rows * k // formats.block_info(t)[0]).cpu().numpy().reshape(-1)
        assert np.array_equal(got, oracle.dequant(t, raw))
