"""The safetensors reader (lrm_st_*, rosylnalive_b200.safetensors) against the reference's own test cases
(tests/Lrm.Tensor.Tests/SafetensorsTests.fs): the writer known-answer vector S1, the malformed-file list, escaped
names, unaligned headers, and the tiny golden model file read bit for bit. No GPU: the library's reader is host code."""

import hashlib
import json
import os

import numpy as np
import pytest

from rosylnalive_b200 import safetensors as ST
from rosylnalive_b200.native import SafetensorsFormatError

HERE = os.path.dirname(os.path.abspath(__file__))

# S1 (SafetensorsTests.fs:13-46): four tensors (an astral name, a scalar, an empty tensor) and two metadata entries
# whose values need escaping. The reference states the header bytes, the file length (338) and the SHA-256.
S1_NAME = "é\U0001F600"
S1_VALUE = "\"q\"\\\n\x7f\t"
S1_METADATA = {"lrm.test": "saïtensors!", "a": S1_VALUE}
S1_TENSORS = {"x": ("F32", np.array([1.0, -2.0], np.float32)), S1_NAME: ("BF16", np.array([[0x3F80]], np.uint16)),
              "b": ("I64", np.array(7, np.int64)), "e": ("U8", np.zeros(0, np.uint8))}
S1_HEADER = ('{"__metadata__":{"a":"\\"q\\"\\\\\\n\\u007f\\t","lrm.test":"sa\\u00eftensors!"},'
             '"b":{"dtype":"I64","shape":[],"data_offsets":[0,8]},'
             '"e":{"dtype":"U8","shape":[0],"data_offsets":[8,8]},'
             '"x":{"dtype":"F32","shape":[2],"data_offsets":[8,16]},'
             '"\\u00e9\\ud83d\\ude00":{"dtype":"BF16","shape":[1,1],"data_offsets":[16,18]}}' + " " * 7)
S1_SHA256 = "49fc00c6aa63a8f23a5488fe2bd49a8768779e8f5b943a166013f4b2140666ce"


def raw_file_bytes(header: bytes, data: bytes) -> bytes:
    return len(header).to_bytes(8, "little") + header + data


def raw_file(header: str, data: bytes) -> bytes:
    return raw_file_bytes(header.encode("utf-8"), data)


def s1_bytes() -> bytes:
    data = np.int64(7).tobytes() + np.array([1.0, -2.0], np.float32).tobytes() + np.uint16(0x3F80).tobytes()
    return raw_file(S1_HEADER, data)


def esc(hexd: str) -> str:
    return "\\u" + hexd


def entry(dtype, shape, b, e):
    return f'{{"dtype":"{dtype}","shape":{shape},"data_offsets":[{b},{e}]}}'


@pytest.fixture
def write_file(tmp_path):
    def w(data: bytes) -> str:
        p = tmp_path / "t.safetensors"
        p.write_bytes(data)
        return str(p)
    return w


def test_s1_fixture_is_the_reference_vector():
    b = s1_bytes()
    assert int.from_bytes(b[:8], "little") == 312 and len(b) == 338
    assert hashlib.sha256(b).hexdigest() == S1_SHA256


def test_writer_reproduces_s1_byte_for_byte(tmp_path):
    p = tmp_path / "s1.safetensors"
    ST.write(str(p), S1_TENSORS, S1_METADATA)
    assert p.read_bytes() == s1_bytes()


def test_reader_opens_s1(write_file):
    path = write_file(s1_bytes())
    with ST.SafetensorsFile.open(path) as f:
        assert f.header_length == 312 and f.data_offset == 320 and f.length == 338
        assert f.names == ["b", "e", "x", S1_NAME]  # code point order
        assert f.metadata == [("a", S1_VALUE), ("lrm.test", "saïtensors!")]
        assert f.read_f32("x").tolist() == [1.0, -2.0]
        assert f.read_bf16(S1_NAME).tolist() == [[0x3F80]]
        assert f.read_i64("b").shape == () and int(f.read_i64("b")) == 7
        assert f.read_u8("e").size == 0
        assert f.is_aligned
        with pytest.raises(ValueError):
            f.read("x", "F64")
        with pytest.raises(KeyError):
            f.read("nope")
    assert ST.validate(s1_bytes()) == (312, 4)


OK = entry("F32", "[1]", 0, 4)
MALFORMED_TEXT = [
    ("not JSON", '{"a":', b"\0" * 4),
    ("not an object", "[1, 2]", b"\0" * 4),
    ("leading space", " {}", b""),
    ("duplicate name", '{"a":' + OK + ',"a":' + OK + "}", b"\0" * 4),
    ("unknown dtype", '{"a":' + entry("BOOL", "[4]", 0, 4) + "}", b"\0" * 4),
    ("negative dimension", '{"a":' + entry("U8", "[-4]", 0, 4) + "}", b"\0" * 4),
    ("fractional dimension", '{"a":' + entry("U8", "[4.0]", 0, 4) + "}", b"\0" * 4),
    ("size mismatch", '{"a":' + entry("F32", "[2]", 0, 4) + "}", b"\0" * 4),
    ("end beyond the data", '{"a":' + entry("U8", "[8]", 0, 8) + "}", b"\0" * 4),
    ("reversed offsets", '{"a":' + entry("U8", "[0]", 4, 0) + "}", b"\0" * 4),
    ("hole", '{"a":' + entry("U8", "[2]", 2, 4) + "}", b"\0" * 4),
    ("overlap", '{"a":' + entry("U8", "[3]", 0, 3) + ',"b":' + entry("U8", "[2]", 2, 4) + "}", b"\0" * 4),
    ("trailing bytes", '{"a":' + entry("U8", "[2]", 0, 2) + "}", b"\0" * 4),
    ("offsets not a pair", '{"a":{"dtype":"U8","shape":[4],"data_offsets":[0]}}', b"\0" * 4),
    ("missing field", '{"a":{"dtype":"U8","shape":[4]}}', b"\0" * 4),
    ("unknown field", '{"a":{"dtype":"U8","shape":[4],"data_offsets":[0,4],"x":1}}', b"\0" * 4),
    ("empty name", '{"":' + OK + "}", b"\0" * 4),
    ("metadata not strings", '{"__metadata__":{"k":1},"a":' + OK + "}", b"\0" * 4),
    ("metadata not an object", '{"__metadata__":[],"a":' + OK + "}", b"\0" * 4),
    ("lone high surrogate in a name", '{"' + esc("d800") + '":' + OK + "}", b"\0" * 4),
    ("lone low surrogate in a name", '{"a' + esc("dc00") + 'b":' + OK + "}", b"\0" * 4),
    ("high surrogate without its low half", '{"' + esc("d83d") + esc("0041") + '":' + OK + "}", b"\0" * 4),
    ("lone surrogate in a metadata key", '{"__metadata__":{"' + esc("dc00") + '":"v"},"a":' + OK + "}", b"\0" * 4),
    ("lone surrogate in a metadata value", '{"__metadata__":{"k":"' + esc("dc00") + '"},"a":' + OK + "}", b"\0" * 4),
    ("lone surrogate in a dtype", '{"a":' + entry("U" + esc("d800"), "[4]", 0, 4) + "}", b"\0" * 4),
    ("lone surrogate in a field name",
     '{"a":{"dtype":"U8","shape":[4],"data_offsets":[0,4],"' + esc("d800") + '":1}}', b"\0" * 4),
]
MALFORMED_BYTES = [
    ("invalid UTF-8 in a name", b'{"a' + b"\xff" + ('":' + OK + "}").encode()),
    ("invalid UTF-8 in a metadata value", b'{"__metadata__":{"k":"v' + b"\xc3" + ('"},"a":' + OK + "}").encode()),
    ("a UTF-8 encoded surrogate (CESU-8)", b'{"a' + b"\xed\xa0\x80" + ('":' + OK + "}").encode()),
    ("an overlong UTF-8 encoding", b'{"' + b"\xc1\x81" + ('":' + OK + "}").encode()),
]


def expect_format_error(write_file, data: bytes):
    with pytest.raises(SafetensorsFormatError):
        ST.validate(data)
    path = write_file(data)
    with pytest.raises(SafetensorsFormatError) as e:
        ST.SafetensorsFile.open(path)
    assert os.path.realpath(path) in str(e.value)  # the message names the file


def test_reader_rejects_short_and_oversized_headers(write_file):
    expect_format_error(write_file, b"\x01\x02")
    expect_format_error(write_file, (100).to_bytes(8, "little") + b"\0" * 8)
    expect_format_error(write_file, (100_000_001).to_bytes(8, "little") + b"\0" * 8)


@pytest.mark.parametrize("label,header,data", MALFORMED_TEXT, ids=[m[0] for m in MALFORMED_TEXT])
def test_reader_rejects_malformed_headers(write_file, label, header, data):
    expect_format_error(write_file, raw_file(header, data))


@pytest.mark.parametrize("label,header", MALFORMED_BYTES, ids=[m[0] for m in MALFORMED_BYTES])
def test_reader_rejects_invalid_utf8(write_file, label, header):
    expect_format_error(write_file, raw_file_bytes(header, b"\0" * 4))


def test_reader_decodes_escaped_names_in_code_point_order():
    header = ('{"' + esc("d83d") + esc("de00") + '":' + entry("U8", "[2]", 0, 2) + ',"' + esc("0041") + '":' +
              entry("U8", "[2]", 2, 4) + "}")
    path = None
    data = raw_file(header, b"\0" * 4)
    assert ST.validate(data) == (len(header), 2)
    import tempfile
    with tempfile.TemporaryDirectory() as d:
        path = os.path.join(d, "n.safetensors")
        with open(path, "wb") as f:
            f.write(data)
        with ST.SafetensorsFile.open(path) as st:
            assert st.names == ["A", "\U0001F600"]


def test_reader_accepts_any_header_length_and_records_alignment(write_file):
    header = '{"a":' + entry("U8", "[4]", 0, 4) + "}"
    path = write_file(raw_file(header, bytes([1, 2, 3, 4])))
    with ST.SafetensorsFile.open(path) as f:
        assert f.header_length == len(header) == 53  # not a multiple of 8
        assert not f.is_aligned
        assert f.read_u8("a").tolist() == [1, 2, 3, 4]


def test_reader_reads_the_tiny_golden_model_bit_for_bit():
    # tests/golden/tiny_g1_model.safetensors is the reference's goldens/tiny/g1/model/model.safetensors, copied whole
    # (SHA-256 from its SHA256SUMS); tiny_g1.npz holds the same tensors extracted by the fixture script.
    path = os.path.join(HERE, "golden", "tiny_g1_model.safetensors")
    with open(path, "rb") as f:
        assert hashlib.sha256(f.read()).hexdigest() == \
            "7ade5616bee29bf1008e4a2902cd7aa6b334e3571aa978356d7adfe08e058b2e"
    z = np.load(os.path.join(HERE, "golden", "tiny_g1.npz"))
    want = {k[2:]: z[k] for k in z.files if k.startswith("w/")}
    with ST.SafetensorsFile.open(path) as f:
        assert sorted(f.names) == sorted(want) and f.names == sorted(want, key=lambda s: s.encode())
        for name in f.names:
            got = f.read(name)
            assert f.entry(name).dtype == "BF16"
            assert got.dtype == want[name].dtype and np.array_equal(got, want[name]), name


def test_writer_round_trip_of_random_tensors(tmp_path):
    rng = np.random.default_rng(9)
    tensors = {}
    for i, dt in enumerate(ST.DTYPES):
        shape = tuple(rng.integers(0, 4, rng.integers(0, 4)))
        a = rng.integers(0, 255, shape).astype(ST._NUMPY[dt])
        tensors[f"t{i}" + ("\U0001F600" if i % 3 == 0 else "") + ('"' if i % 4 == 1 else "")] = (dt, a)
    p = tmp_path / "r.safetensors"
    ST.write(str(p), tensors, {"k0": "v0\n"})
    with ST.SafetensorsFile.open(str(p)) as f:
        assert f.metadata == [("k0", "v0\n")]
        for name, (dt, a) in tensors.items():
            assert f.entry(name).dtype == dt
            assert np.array_equal(f.read(name), a)
    header = json.loads(p.read_bytes()[8:8 + int.from_bytes(p.read_bytes()[:8], "little")])
    assert list(header)[0] == "__metadata__"
