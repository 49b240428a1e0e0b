"""SafetensorsFile over liblrmcuda.so's validating, memory-mapped reader (lrm_st_*): the counterpart of the reference's
SafetensorsFile (src/Lrm.Tensor/Safetensors.fs:504-727). Needs no GPU.

    with SafetensorsFile.open(path) as f:
        f.names, f.metadata, f.read_bf16("model.embed_tokens.weight")

Malformed files raise SafetensorsFormatError (the reference's SafetensorsFormatException) with a message naming the
file; a missing tensor raises KeyError; reading a tensor as the wrong dtype raises ValueError.
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass

import numpy as np

from . import native as N
from .native import SafetensorsFormatError  # noqa: F401  (re-exported)

P, I32, I64, U64 = ctypes.c_void_p, ctypes.c_int32, ctypes.c_int64, ctypes.c_uint64

DTYPES = ("F32", "F64", "BF16", "F16", "I32", "U32", "U8", "I64")
_NUMPY = {"F32": np.float32, "F64": np.float64, "BF16": np.uint16, "F16": np.uint16, "I32": np.int32,
          "U32": np.uint32, "U8": np.uint8, "I64": np.int64}


class EntryC(ctypes.Structure):
    _fields_ = [("name", ctypes.c_char_p), ("dtype", I32), ("rank", I32), ("shape", ctypes.POINTER(I64)),
                ("begin", U64), ("end", U64), ("data", P)]


N.extra_signatures({
    "lrm_st_open": [ctypes.c_char_p, ctypes.POINTER(P)],
    "lrm_st_close": [P],
    "lrm_st_validate": [P, U64, ctypes.POINTER(U64), ctypes.POINTER(I64)],
    "lrm_st_info": [P, ctypes.POINTER(U64), ctypes.POINTER(U64), ctypes.POINTER(I64), ctypes.POINTER(I64),
                    ctypes.POINTER(I32)],
    "lrm_st_entry_at": [P, I64, ctypes.POINTER(EntryC)],
    "lrm_st_find": [P, ctypes.c_char_p, ctypes.POINTER(EntryC)],
    "lrm_st_metadata_at": [P, I64, ctypes.POINTER(ctypes.c_char_p), ctypes.POINTER(ctypes.c_char_p)],
})


@dataclass(frozen=True)
class Entry:
    """SafetensorsEntry: a tensor's name, dtype, shape and byte range within the data section."""

    name: str
    dtype: str
    shape: tuple
    begin: int
    end: int

    @property
    def byte_length(self) -> int:
        return self.end - self.begin


def validate(data: bytes) -> tuple[int, int]:
    """SafetensorsFile.Validate: checks a whole file image in memory; returns (header length, tensor count)."""
    buf = ctypes.create_string_buffer(bytes(data), len(data))
    n, c = U64(), I64()
    N.check(N.lib().lrm_st_validate(ctypes.cast(buf, P), len(data), ctypes.byref(n), ctypes.byref(c)), None,
            "safetensors")
    return int(n.value), int(c.value)


class SafetensorsFile:
    """A validated, memory-mapped safetensors file. Entries and metadata are in code point order of their names."""

    def __init__(self, handle, path: str):
        self._h = handle
        self.path = path
        length, hlen, count, mcount, aligned = U64(), U64(), I64(), I64(), I32()
        N.check(N.lib().lrm_st_info(self._h, ctypes.byref(length), ctypes.byref(hlen), ctypes.byref(count),
                                    ctypes.byref(mcount), ctypes.byref(aligned)), None, "safetensors")
        self.length = int(length.value)
        self.header_length = int(hlen.value)
        self.data_offset = 8 + self.header_length
        self.is_aligned = bool(aligned.value)
        self.entries = [self._entry_at(i) for i in range(int(count.value))]
        self._index = {e.name: i for i, e in enumerate(self.entries)}
        self.metadata = []
        for i in range(int(mcount.value)):
            k, v = ctypes.c_char_p(), ctypes.c_char_p()
            N.check(N.lib().lrm_st_metadata_at(self._h, i, ctypes.byref(k), ctypes.byref(v)), None, "safetensors")
            self.metadata.append((k.value.decode("utf-8"), v.value.decode("utf-8")))

    @staticmethod
    def open(path: str) -> "SafetensorsFile":
        h = P()
        N.check(N.lib().lrm_st_open(str(path).encode("utf-8"), ctypes.byref(h)), None, "safetensors")
        return SafetensorsFile(h, str(path))

    def _entry_at(self, i: int) -> Entry:
        e = EntryC()
        N.check(N.lib().lrm_st_entry_at(self._h, i, ctypes.byref(e)), None, "safetensors")
        return self._entry(e)

    @staticmethod
    def _entry(e: EntryC) -> Entry:
        return Entry(e.name.decode("utf-8"), DTYPES[e.dtype], tuple(e.shape[k] for k in range(e.rank)), int(e.begin),
                     int(e.end))

    @property
    def names(self) -> list:
        return [e.name for e in self.entries]

    def __contains__(self, name: str) -> bool:
        return name in self._index

    def entry(self, name: str) -> Entry:
        if name not in self._index:
            raise KeyError(f"{self.path}: no tensor '{name}'")
        return self.entries[self._index[name]]

    def try_metadata(self, key: str):
        return next((v for k, v in self.metadata if k == key), None)

    def read(self, name: str, dtype: str | None = None) -> np.ndarray:
        """A copy of the tensor (BF16 and F16 as their uint16 bit patterns); `dtype`, when given, must match."""
        self._check_open()
        e = EntryC()
        if name not in self._index:
            raise KeyError(f"{self.path}: no tensor '{name}'")
        N.check(N.lib().lrm_st_find(self._h, name.encode("utf-8"), ctypes.byref(e)), None, "safetensors")
        ent = self._entry(e)
        if dtype is not None and ent.dtype != dtype:
            raise ValueError(f"{name} is {ent.dtype}, not {dtype}")
        raw = ctypes.string_at(e.data, ent.byte_length) if ent.byte_length else b""
        return np.frombuffer(raw, dtype=_NUMPY[ent.dtype]).reshape(ent.shape).copy()

    def read_f32(self, name):
        return self.read(name, "F32")

    def read_bf16(self, name):
        return self.read(name, "BF16")

    def read_i64(self, name):
        return self.read(name, "I64")

    def read_u8(self, name):
        return self.read(name, "U8")

    def _check_open(self):
        if self._h is None:
            raise ValueError(f"{self.path}: the file is closed")

    def close(self):
        if self._h is not None:
            N.lib().lrm_st_close(self._h)
            self._h = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def write(path: str, tensors: dict, metadata: dict | None = None) -> None:
    """Writes a safetensors file the way the reference's deterministic writer lays it out (Safetensors.fs:125-216):
    tensors in code point order of their names, packed from offset 0, the JSON header (json.dumps with ensure_ascii,
    no spaces) padded with spaces to a multiple of 8. `tensors` maps name -> (dtype name, numpy array); BF16 / F16
    arrays are uint16 bit patterns."""
    import json

    names = sorted(tensors, key=lambda s: s.encode("utf-8"))
    header, blobs, off = {}, [], 0
    if metadata:
        header["__metadata__"] = {k: metadata[k] for k in sorted(metadata, key=lambda s: s.encode("utf-8"))}
    for n in names:
        dt, a = tensors[n]
        a = np.asarray(a, dtype=_NUMPY[dt]).copy(order="C")  # keeps 0-d (scalar) shapes
        b = a.tobytes()
        header[n] = {"dtype": dt, "shape": list(a.shape), "data_offsets": [off, off + len(b)]}
        blobs.append(b)
        off += len(b)
    text = json.dumps(header, ensure_ascii=True, separators=(",", ":")).encode("ascii")
    text += b" " * ((8 - len(text) % 8) % 8)
    with open(path, "wb") as f:
        f.write(len(text).to_bytes(8, "little"))
        f.write(text)
        for b in blobs:
            f.write(b)
