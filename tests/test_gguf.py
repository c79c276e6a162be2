"""GGUF ingestion (feml_b200_gguf_*, feml_b200.gguf): files written by
llama.cpp's own Python package (gguf-py, in this image) are read back with
identical metadata, tensor tables and bytes; malformed files are rejected
with an error, never read out of range. No GPU needed."""
import struct

import numpy as np
import pytest

import feml_b200 as F
from feml_b200 import DType
from feml_b200.gguf import GGUFFile
from oracle import oracle as O

gguf = pytest.importorskip("gguf")
from gguf import GGMLQuantizationType as T  # noqa: E402


def _write(path, alignment=None, extra_kv=True):
    rng = np.random.default_rng(11)
    w = gguf.GGUFWriter(str(path), "llama")
    if alignment:
        w.add_custom_alignment(alignment)
    tensors = {}
    if extra_kv:
        w.add_uint8("t.u8", 200)
        w.add_int8("t.i8", -5)
        w.add_uint16("t.u16", 60000)
        w.add_int16("t.i16", -30000)
        w.add_uint32("t.u32", 4000000000)
        w.add_int32("t.i32", -2000000000)
        w.add_float32("t.f32", 0.25)
        w.add_bool("t.bool", False)
        w.add_string("t.str", "mul_mat ✓")
        w.add_uint64("t.u64", 2**40 + 3)
        w.add_int64("t.i64", -(2**40))
        w.add_float64("t.f64", 1e-300)
        w.add_array("t.arr_i", [1, -2, 3])
        w.add_array("t.arr_f", [0.5, 1.5])
        w.add_array("t.arr_s", ["tok", "", "end"])
    x = (rng.standard_normal((6, 512)) * 0.02).astype(np.float32)
    tensors["f32"] = x
    w.add_tensor("f32", x)
    h = x.astype(np.float16)
    tensors["f16"] = h
    w.add_tensor("f16", h)
    for name, t in (("q8_0", T.Q8_0), ("q4_0", T.Q4_0)):
        q = gguf.quants.quantize(x, t)
        tensors[name] = q
        w.add_tensor(name, q, raw_dtype=t)
    q4k = O.quantize(O.DT_Q4_K, x)
    tensors["q4_k"] = q4k
    w.add_tensor("q4_k", q4k, raw_dtype=T.Q4_K)
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()
    return tensors


@pytest.fixture(scope="module")
def gguf_path(tmp_path_factory):
    p = tmp_path_factory.mktemp("gguf") / "model.gguf"
    tensors = _write(p)
    return p, tensors


def test_reads_metadata_written_by_gguf_py(gguf_path):
    p, _ = gguf_path
    with GGUFFile(p) as f:
        md = f.metadata
        assert f.version == 3 and f.alignment == 32
    assert md["general.architecture"] == "llama"
    assert md["t.u8"] == 200 and md["t.i8"] == -5 and md["t.u16"] == 60000 and md["t.i16"] == -30000
    assert md["t.u32"] == 4000000000 and md["t.i32"] == -2000000000
    assert md["t.f32"] == 0.25 and md["t.bool"] is False and md["t.str"] == "mul_mat ✓"
    assert md["t.u64"] == 2**40 + 3 and md["t.i64"] == -(2**40) and md["t.f64"] == 1e-300
    assert md["t.arr_i"].tolist() == [1, -2, 3]
    assert md["t.arr_f"].tolist() == [0.5, 1.5]
    assert md["t.arr_s"] == ["tok", "", "end"]


def test_tensor_table_and_bytes_match_gguf_py_reader(gguf_path):
    p, tensors = gguf_path
    ref = gguf.GGUFReader(str(p))
    want = {t.name: t for t in ref.tensors}
    dtypes = {"f32": DType.F32, "f16": DType.F16, "q8_0": DType.Q8_0, "q4_0": DType.Q4_0, "q4_k": DType.Q4_K}
    with GGUFFile(p) as f:
        assert [t.name for t in f.tensors] == [t.name for t in ref.tensors]
        for t in f.tensors:
            r = want[t.name]
            assert t.dtype == dtypes[t.name]
            assert t.ggml_type == int(r.tensor_type)
            assert t.shape == tuple(int(v) for v in r.shape)
            assert t.offset == int(r.data_offset) and t.nbytes == int(r.n_bytes)
            assert t.offset % f.alignment == 0
            got = f.tensor_bytes(t.name)
            assert not got.flags.writeable
            assert np.array_equal(got, np.frombuffer(np.ascontiguousarray(tensors[t.name]).tobytes(), np.uint8))
            assert t.nbytes == t.dtype.row_size(t.shape[0]) * int(np.prod(t.shape[1:]))


def test_custom_alignment(tmp_path):
    p = tmp_path / "a.gguf"
    _write(p, alignment=256, extra_kv=False)
    with GGUFFile(p) as f:
        assert f.alignment == 256 and f.data_offset % 256 == 0
        assert all(t.offset % 256 == 0 for t in f.tensors)
        ref = gguf.GGUFReader(str(p))
        assert [t.offset for t in f.tensors] == [int(t.data_offset) for t in ref.tensors]


# ---- malformed files ---------------------------------------------------------
def _s(b):
    return struct.pack("<Q", len(b)) + b


def _header(n_tensors, n_kv, version=3):
    return b"GGUF" + struct.pack("<IQQ", version, n_tensors, n_kv)


def _tensor_info(name, dims, ggml_type, offset):
    return _s(name) + struct.pack("<I", len(dims)) + b"".join(struct.pack("<Q", d) for d in dims) + \
        struct.pack("<IQ", ggml_type, offset)


def _file(infos, data_len, kvs=b"", n_kv=0, version=3):
    body = _header(len(infos), n_kv, version) + kvs + b"".join(infos)
    pad = (-len(body)) % 32
    return body + b"\0" * pad + b"\x11" * data_len


def _open_bytes(tmp_path, data):
    p = tmp_path / "bad.gguf"
    p.write_bytes(data)
    return GGUFFile(p)


def test_minimal_hand_written_file(tmp_path):
    data = _file([_tensor_info(b"w", [64, 2], 8, 0)], 2 * 68)
    with _open_bytes(tmp_path, data) as f:
        (t,) = f.tensors
        assert t.dtype == DType.Q8_0 and t.shape == (64, 2) and t.nbytes == 136
        assert bytes(f.tensor_bytes("w")) == b"\x11" * 136


@pytest.mark.parametrize("case", ["magic", "version", "truncated_header", "truncated_info", "data_past_eof",
                                  "misaligned", "five_dims", "bad_block", "duplicate_tensor", "bad_kv_type",
                                  "string_past_eof", "huge_count", "nul_in_name"])
def test_malformed_files_are_rejected(tmp_path, case):
    good = _file([_tensor_info(b"w", [64, 2], 8, 0)], 136)
    if case == "magic":
        data = b"GGUX" + good[4:]
    elif case == "version":
        data = _file([_tensor_info(b"w", [64, 2], 8, 0)], 136, version=1)
    elif case == "truncated_header":
        data = good[:20] + b"\0" * 4
    elif case == "truncated_info":
        data = _header(1, 0) + _tensor_info(b"w", [64, 2], 8, 0)[:30]
    elif case == "data_past_eof":
        data = _file([_tensor_info(b"w", [64, 2], 8, 0)], 100)
    elif case == "misaligned":
        data = _file([_tensor_info(b"w", [64, 2], 8, 4)], 200)
    elif case == "five_dims":
        data = _file([_tensor_info(b"w", [32, 1, 1, 1, 1], 8, 0)], 68)
    elif case == "bad_block":
        data = _file([_tensor_info(b"w", [40, 2], 8, 0)], 200)
    elif case == "duplicate_tensor":
        data = _file([_tensor_info(b"w", [32], 8, 0), _tensor_info(b"w", [32], 8, 64)], 200)
    elif case == "bad_kv_type":
        data = _file([], 0, kvs=_s(b"k") + struct.pack("<I", 99) + b"\0" * 8, n_kv=1)
    elif case == "string_past_eof":
        data = _header(0, 1) + _s(b"k") + struct.pack("<I", 8) + struct.pack("<Q", 1 << 40) + b"abc"
    elif case == "nul_in_name":
        data = _file([_tensor_info(b"w\0x", [32], 8, 0)], 68)
    else:  # huge_count
        data = _header(1 << 60, 0) + b"\0" * 64
    with pytest.raises(F.FemlError) as ei:
        _open_bytes(tmp_path, data)
    assert "gguf" in str(ei.value)


def test_missing_file_and_names(tmp_path, gguf_path):
    with pytest.raises(F.FemlError):
        GGUFFile(tmp_path / "nope.gguf")
    p, _ = gguf_path
    with GGUFFile(p) as f:
        with pytest.raises(F.FemlError):
            f.tensor("absent")
    with pytest.raises(F.FemlError):
        f.tensor_bytes("f32")  # closed


def test_unknown_and_unmapped_types_are_listed(tmp_path):
    # BF16 (ggml id 30): size known, no feml dtype; id 200: unknown, size 0
    data = _file([_tensor_info(b"b", [8], 30, 0), _tensor_info(b"u", [8], 200, 32)], 64)
    with _open_bytes(tmp_path, data) as f:
        b, u = f.tensors
        assert b.dtype is None and b.nbytes == 16
        assert u.dtype is None and u.nbytes == 0
        with pytest.raises(F.FemlError):
            f.tensor_bytes("u")


def test_mutated_files_never_read_out_of_range(tmp_path, gguf_path):
    """Random byte flips and truncations of a valid file: every open either
    succeeds (then every tensor's bytes lie inside the file) or raises
    FemlError; none crashes the process."""
    p, _ = gguf_path
    good = p.read_bytes()
    rng = np.random.default_rng(2024)
    bad = tmp_path / "mut.gguf"
    for trial in range(600):
        data = bytearray(good)
        if trial % 3 == 0:
            data = data[: int(rng.integers(0, len(data)))]
        else:
            head = min(len(data), 1200)  # header, metadata and tensor table
            for _ in range(int(rng.integers(1, 6))):
                data[int(rng.integers(0, head))] = int(rng.integers(0, 256))
        bad.write_bytes(bytes(data))
        try:
            f = GGUFFile(bad)
        except F.FemlError:
            continue
        with f:
            f.metadata  # noqa: B018 (parses every value)
            for t in f.tensors:
                assert t.offset + t.nbytes <= len(data)
                if t.nbytes:
                    assert f.tensor_bytes(t.name).size == t.nbytes
