"""QwenTokenizer over liblrmcuda.so's native tokenizer (lrm_tok_*): the counterpart of the reference's QwenTokenizer
(src/Lrm.Tokenizer/QwenTokenizer.fs:19-309), the Qwen3 byte-level BPE tokenizer with exact id parity with HF
tokenizers 0.23.3 on the pinned tokenizer.json. Needs no GPU.

    tok = QwenTokenizer.load("models/Qwen3-0.6B/tokenizer.json")   # checks the SHA-256 pin
    ids = tok.encode("Hello, world")                                # no BOS / EOS
    text = tok.decode(ids)

Encode runs, in order: added tokens on the raw text (leftmost-longest), then for each stretch between them the
oracle's NFC (Unicode 9.0 semantics), the Split pre-tokenizer and byte-level BPE. A malformed or unsupported
tokenizer.json raises TokenizerFormatError (the reference's InvalidDataException) with the reference's message.

The stage functions (nfc, split, char_class, contraction_letter, byte_char) expose the pipeline's steps for tests and
diagnostics, as the reference's Nfc, PreTokenizer, CharClass and ByteLevel modules do.
"""

from __future__ import annotations

import ctypes
import hashlib
import os
from dataclasses import dataclass

from . import native as N

P, I32, I64, U64 = ctypes.c_void_p, ctypes.c_int32, ctypes.c_int64, ctypes.c_uint64
PI32, PU64 = ctypes.POINTER(I32), ctypes.POINTER(U64)

N.extra_signatures({
    "lrm_tok_parse": [P, U64, ctypes.POINTER(P)],
    "lrm_tok_free": [P],
    "lrm_tok_info": [P, PI32, PI32, PI32],
    "lrm_tok_clear_cache": [P],
    "lrm_tok_cached_pieces": [P, ctypes.POINTER(I64)],
    "lrm_tok_added_at": [P, I32, PI32, ctypes.POINTER(ctypes.c_char_p), PI32],
    "lrm_tok_encode": [P, ctypes.c_char_p, U64, PI32, U64, PU64],
    "lrm_tok_encode_bytes": [P, ctypes.c_char_p, U64, PI32, U64, PU64],
    "lrm_tok_decode_bytes": [P, PI32, U64, ctypes.c_char_p, U64, PU64],
    "lrm_tok_decode": [P, PI32, U64, ctypes.c_char_p, U64, PU64],
    "lrm_tok_id_of": [P, ctypes.c_char_p, PI32],
    "lrm_tok_token_of": [P, I32, ctypes.c_char_p, U64, PU64, PI32],
    "lrm_tok_nfc": [ctypes.c_char_p, U64, ctypes.c_char_p, U64, PU64],
    "lrm_tok_split": [ctypes.c_char_p, U64, PU64, U64, PU64],
    "lrm_tok_char_class": [ctypes.c_uint32],
    "lrm_tok_contraction_letter": [ctypes.c_uint32],
    "lrm_tok_byte_char": [ctypes.c_uint8],
}, {"lrm_tok_char_class": I32, "lrm_tok_contraction_letter": I32, "lrm_tok_byte_char": ctypes.c_uint32})

PINNED_SHA256 = "aeb13307a71acd8fe81861d94ad54ab689df773318809eed3cbe794b4492dae4"  # QwenTokenizer.PinnedSha256
PINNED_PATH = "models/Qwen3-0.6B/tokenizer.json"  # QwenTokenizer.PinnedPath, under the data root
REAL_IDS = 151_669  # 151,643 vocabulary tokens and 26 added tokens
MODEL_ROWS = 151_936  # Qwen3-0.6B's embedding and lm_head rows
CACHE_CAPACITY = 1 << 16  # two generations of 32,768 pieces
CACHE_UNITS = 1 << 21  # two generations of 1 Mi UTF-16 units
CACHED_PIECE_UNITS = 1 << 16  # longer pieces are never cached
SPLIT_PATTERN = (r"(?i:'s|'t|'re|'ve|'m|'ll|'d)|[^\r\n\p{L}\p{N}]?\p{L}+|\p{N}| ?[^\s\p{L}\p{N}]+[\r\n]*|"
                 r"\s*[\r\n]+|\s+(?!\S)|\s+")
CLASSES = ("letter", "number", "space", "other")


class TokenizerFormatError(ValueError):
    """tokenizer.json is malformed, unsupported or not the pinned file: the reference's InvalidDataException
    (TokenizerJson.fs:23-24, QwenTokenizer.fs:275-296)."""


@dataclass(frozen=True)
class AddedToken:
    """One added token of tokenizer.json, such as <|im_start|> (AddedTokens.fs:7-13)."""

    id: int
    content: str
    special: bool


def _check(status: int):
    N.check(status, None, "tokenizer", format_error=TokenizerFormatError)


def _utf8(text: str) -> bytes:
    if not isinstance(text, str):
        raise TypeError("text must be a str")
    try:
        return text.encode("utf-8")
    except UnicodeEncodeError as e:  # a lone surrogate: the reference's ArgumentException (QwenTokenizer.fs:46-57)
        raise ValueError(f"the text holds a lone surrogate U+{ord(text[e.start]):04X} at index {e.start}") from None


def _ids_array(ids) -> ctypes.Array:
    ids = list(ids)
    for i in ids:
        if not -(1 << 31) <= int(i) < (1 << 31):
            raise ValueError(f"token id {i} is outside the model's {MODEL_ROWS} rows")
    return (I32 * len(ids))(*ids)


def _sized(call, ctype, guess: int):
    """Runs an (out, cap, count) call into a buffer of `guess` items, and once more with the exact size when the
    result did not fit."""
    n = U64(0)
    cap = max(1, guess)
    buf = ctypes.create_string_buffer(cap) if ctype is ctypes.c_char else (ctype * cap)()
    status = call(buf, cap, ctypes.byref(n))
    if status == N.LRM_ERR_ARGUMENT and n.value > cap:
        cap = n.value
        buf = ctypes.create_string_buffer(cap) if ctype is ctypes.c_char else (ctype * cap)()
        status = call(buf, cap, ctypes.byref(n))
    _check(status)
    return buf, n.value


class QwenTokenizer:
    """The Qwen3 byte-level BPE tokenizer. Immutable apart from a piece cache that never changes a result; every
    method is safe to call from many threads at once (the native calls release the GIL)."""

    def __init__(self, handle, sha256: str):
        self._h = handle
        self.sha256 = sha256
        v, m, a = I32(), I32(), I32()
        _check(N.lib().lrm_tok_info(self._h, ctypes.byref(v), ctypes.byref(m), ctypes.byref(a)))
        self.vocab_size = int(v.value)
        self.merge_count = int(m.value)
        added = []
        for i in range(int(a.value)):
            tid, content, special = I32(), ctypes.c_char_p(), I32()
            _check(N.lib().lrm_tok_added_at(self._h, i, ctypes.byref(tid), ctypes.byref(content), ctypes.byref(special)))
            added.append(AddedToken(int(tid.value), content.value.decode("utf-8"), bool(special.value)))
        self.added_tokens = added

    # ---- loading (QwenTokenizer.fs:237-309) -----------------------------------------------------------------------

    @staticmethod
    def parse(json_bytes: bytes) -> "QwenTokenizer":
        """Builds a tokenizer from tokenizer.json bytes without checking their hash; the structure is still checked."""
        if json_bytes is None:
            raise TypeError("json is None")
        data = bytes(json_bytes)
        h = P()
        _check(N.lib().lrm_tok_parse(data, len(data), ctypes.byref(h)))
        return QwenTokenizer(h, hashlib.sha256(data).hexdigest())

    @staticmethod
    def load(path: str) -> "QwenTokenizer":
        """Reads tokenizer.json and checks its SHA-256 against the pin before parsing it; FileNotFoundError when the
        file is missing, TokenizerFormatError on another hash or an unsupported configuration."""
        with open(path, "rb") as f:
            data = f.read()
        sha = hashlib.sha256(data).hexdigest()
        if sha != PINNED_SHA256:
            raise TokenizerFormatError(f"{path} has SHA-256 {sha}, but the TokenizerApi pin is {PINNED_SHA256} "
                                       "(tokenizer.json of Qwen3-0.6B)")
        t = QwenTokenizer.parse(data)
        if t.vocab_size != REAL_IDS:
            raise TokenizerFormatError(f"{path} has {t.vocab_size} real ids, expected {REAL_IDS}")
        return t

    @staticmethod
    def default_path() -> str:
        """The pinned tokenizer.json under the data root (LRM_DATA, else ./data)."""
        return os.path.join(os.environ.get("LRM_DATA", "data"), *PINNED_PATH.split("/"))

    @staticmethod
    def try_load_default():
        """The pinned tokenizer from the data root, or None when the file is absent."""
        path = QwenTokenizer.default_path()
        return QwenTokenizer.load(path) if os.path.exists(path) else None

    # ---- encode / decode -------------------------------------------------------------------------------------------

    def _handle(self):
        if self._h is None:
            raise ValueError("the tokenizer is closed")
        return self._h

    def encode(self, text: str) -> list:
        """The token ids of `text`; ValueError when it holds a lone surrogate."""
        b = _utf8(text)
        h = self._handle()
        buf, n = _sized(lambda out, cap, cnt: N.lib().lrm_tok_encode(h, b, len(b), out, cap, cnt), I32, len(b))
        return list(buf[:n])

    def encode_bytes(self, data: bytes) -> list:
        """The token ids of UTF-8 bytes decoded with one U+FFFD per maximal invalid subpart (errors="replace")."""
        b = bytes(data)
        h = self._handle()
        buf, n = _sized(lambda out, cap, cnt: N.lib().lrm_tok_encode_bytes(h, b, len(b), out, cap, cnt), I32,
                        3 * len(b))
        return list(buf[:n])

    def decode_bytes(self, ids) -> bytes:
        """Each vocabulary token's bytes and each added token's content as the ByteLevel decoder gives it; nothing for
        ids from vocab_size to MODEL_ROWS - 1; ValueError for an id below 0 or at MODEL_ROWS and above."""
        a = _ids_array(ids)
        h = self._handle()
        buf, n = _sized(lambda out, cap, cnt: N.lib().lrm_tok_decode_bytes(h, a, len(a), out, cap, cnt), ctypes.c_char,
                        8 * len(a))
        return buf.raw[:n]

    def decode(self, ids) -> str:
        """decode_bytes decoded as UTF-8 with one U+FFFD per maximal invalid subpart (errors="replace")."""
        a = _ids_array(ids)
        h = self._handle()
        buf, n = _sized(lambda out, cap, cnt: N.lib().lrm_tok_decode(h, a, len(a), out, cap, cnt), ctypes.c_char,
                        8 * len(a))
        return buf.raw[:n].decode("utf-8")

    def id_of(self, token: str):
        """The id of an added token's content or of a vocabulary token in byte-level form ("\\u0120the" for " the");
        None when there is none."""
        out = I32()
        _check(N.lib().lrm_tok_id_of(self._handle(), _utf8(token), ctypes.byref(out)))
        return None if out.value < 0 else int(out.value)

    def token_of(self, token_id: int):
        """The byte-level vocabulary string or the added token's content; None for other ids."""
        if not -(1 << 31) <= int(token_id) < (1 << 31):
            return None
        h, found = self._handle(), I32()
        n = U64()
        _check(N.lib().lrm_tok_token_of(h, int(token_id), None, 0, ctypes.byref(n), ctypes.byref(found)))
        if not found.value:
            return None
        buf = ctypes.create_string_buffer(max(1, n.value))
        _check(N.lib().lrm_tok_token_of(h, int(token_id), buf, n.value, ctypes.byref(n), ctypes.byref(found)))
        return buf.raw[:n.value].decode("utf-8")

    def clear_cache(self) -> None:
        """Forgets every cached piece (for cold-cache measurements); results never depend on the cache."""
        _check(N.lib().lrm_tok_clear_cache(self._handle()))

    @property
    def cached_pieces(self) -> int:
        n = I64()
        _check(N.lib().lrm_tok_cached_pieces(self._handle(), ctypes.byref(n)))
        return int(n.value)

    def close(self):
        if self._h is not None:
            N.lib().lrm_tok_free(self._h)
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


# ---- the stages ------------------------------------------------------------------------------------------------------

def nfc(text: str) -> str:
    """The oracle's NFC (Nfc.fs): Unicode 9.0 semantics."""
    b = _utf8(text)
    buf, n = _sized(lambda out, cap, cnt: N.lib().lrm_tok_nfc(b, len(b), out, cap, cnt), ctypes.c_char,
                    2 * len(b) + 16)
    return buf.raw[:n].decode("utf-8")


def split(text: str) -> list:
    """The Split pre-tokenizer's pieces of `text` (PreTokenizer.fs), which must already be normalized."""
    b = _utf8(text)
    buf, n = _sized(lambda out, cap, cnt: N.lib().lrm_tok_split(b, len(b), out, cap, cnt), U64, len(b))
    pieces, at = [], 0
    for e in buf[:n]:
        pieces.append(b[at:e].decode("utf-8"))
        at = e
    return pieces


def char_class(scalar: int) -> str:
    """The Split regex's class of a scalar (CharClass.fs): letter, number, space or other."""
    k = N.lib().lrm_tok_char_class(int(scalar))
    if k < 0:
        raise ValueError(f"{scalar:#x} is not a Unicode scalar")
    return CLASSES[k]


def contraction_letter(scalar: int):
    """The letter a scalar stands for in (?i:'s|'t|'re|'ve|'m|'ll|'d), or None."""
    k = N.lib().lrm_tok_contraction_letter(int(scalar))
    return chr(k) if k else None


def byte_char(byte: int) -> str:
    """ByteLevel.charOf: the character GPT-2's byte map gives a byte."""
    return chr(N.lib().lrm_tok_byte_char(int(byte)))


def byte_level(data: bytes) -> str:
    """ByteLevel.encode: the byte-level string of raw bytes."""
    return "".join(byte_char(b) for b in bytes(data))


# ---- the corpus runner (src/Lrm.Tokenizer/Corpus.fs) ----------------------------------------------------------------

@dataclass(frozen=True)
class CorpusCase:
    """One line of a tokenizer corpus, run: its id, category (the line's cat, or probe-<kind>), kind, result, token
    count and, when it failed, why."""

    id: str
    category: str
    kind: str
    passed: bool
    tokens: int
    detail: str


def _compare_ids(want: list, got: list):
    if list(want) == list(got):
        return None
    i = next((k for k in range(min(len(want), len(got))) if want[k] != got[k]), min(len(want), len(got)))
    window = lambda a: " ".join(str(x) for x in a[max(0, i - 3):i + 4])  # noqa: E731
    return (f"ids differ at {i} (expected {len(want)} ids, got {len(got)}): expected ... {window(want)} ..., "
            f"got ... {window(got)} ...")


def _from_utf16_hex(h: str) -> str:
    """A string from UTF-16 code units in big-endian hex, 4 digits each; lone surrogates stay lone."""
    units = [int(h[4 * i:4 * i + 4], 16) for i in range(len(h) // 4)]
    return b"".join(u.to_bytes(2, "little") for u in units).decode("utf-16-le", errors="surrogatepass")


def run_case(t: QwenTokenizer, line: dict, fallback_id: str) -> CorpusCase:
    """Runs one corpus line by its kind (Corpus.fs:114-180): encode, encode_bytes (the bytes must decode to the
    line's text with errors=replace), decode (optionally with the bytes DecodeBytes must give) and encode_reject (a
    text with a lone surrogate that Encode must refuse). An exception fails the case."""
    kind = line.get("kind", "") if isinstance(line.get("kind", ""), str) else ""
    cid = line.get("id", fallback_id)
    cat = line.get("cat", "probe-" + kind)

    def done(passed, tokens=0, detail=""):
        return CorpusCase(cid, cat, kind, passed, tokens, detail)

    def ids(want, got):
        d = _compare_ids(want, got)
        return done(d is None, len(want), d or "")

    try:
        if kind == "encode":
            return ids(line["ids"], t.encode(line["text"]))
        if kind == "encode_bytes":
            b = bytes.fromhex(line["bytes"])
            if b.decode("utf-8", errors="replace") != line["text"]:
                return done(False, detail="the bytes do not decode to the case's text (errors=replace)")
            return ids(line["ids"], t.encode_bytes(b))
        if kind == "decode":
            want = line["ids"]
            decoded = t.decode(want)
            if "bytes" in line and t.decode_bytes(want) != bytes.fromhex(line["bytes"]):
                return done(False, detail="DecodeBytes differs from the case's bytes")
            if decoded != line["text"]:
                return done(False, detail=f"Decode gave {decoded!r}, expected {line['text']!r}")
            return done(True, len(want))
        if kind == "encode_reject":
            s = _from_utf16_hex(line["utf16"])
            try:
                t.encode(s)
            except ValueError:
                return done(True)
            return done(False, detail="Encode accepted a text with a lone surrogate")
        return done(False, detail=f"unknown kind '{kind}'")
    except Exception as e:  # noqa: BLE001 -- the reference's runner turns every exception into a failed case
        return done(False, detail=f"{type(e).__name__}: {e}")


def run_corpus(t: QwenTokenizer, text: str, source: str = "corpus") -> list:
    """Runs every non-empty line of a JSON-lines corpus (Corpus.run); a line that is not JSON fails as its own case."""
    import json

    out = []
    for n, raw in enumerate(text.split("\n"), start=1):
        raw = raw.rstrip("\r")
        if not raw:
            continue
        fallback = f"{source}:{n}"
        try:
            line = json.loads(raw)
        except ValueError as e:
            out.append(CorpusCase(fallback, "invalid", "", False, 0, f"the line is not JSON: {e}"))
            continue
        if not isinstance(line, dict):
            out.append(CorpusCase(fallback, "invalid", "", False, 0, "the line is not a JSON object"))
            continue
        out.append(run_case(t, line, fallback))
    return out
