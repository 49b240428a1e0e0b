"""The tokenizer on the ends of the path (liblrmcuda.so's lrm_tok_*, rosylnalive_b200.tokenizer), checked as the
reference checks its own (tests/Lrm.Tokenizer.Tests: PreTokenizerTests.fs, UnicodeTests.fs, ToyTests.fs and the
tokenizer.json tier of CorpusTests.fs), against the oracle's committed probes in tests/golden:

  * tokenizer_unicode-oracle.json: HF tokenizers 0.23.3's class of every scalar, contraction letters, NFC split
    points and the count and SHA-256 of every NFC probe family;
  * tokenizer_split-cases.jsonl: 4,000 texts with the oracle's Split pieces;
  * tokenizer_encode-cases.jsonl.gz and tokenizer_corpus-cases.jsonl.gz: id vectors that need the real
    tokenizer.json, which this machine does not have; those tests skip visibly unless LRM_DATA holds it.

No GPU: every test here runs on the CPU suite.
"""

from __future__ import annotations

import gzip
import hashlib
import json
import os
import subprocess
import sys
import threading

import pytest

from rosylnalive_b200 import native
from rosylnalive_b200 import tokenizer as T

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")
MAX_SCALAR = 0x110000

try:
    native.lib()
    HAVE_LIB = True
except native.NativeLibraryMissing:
    HAVE_LIB = False
pytestmark = pytest.mark.skipif(not HAVE_LIB, reason="liblrmcuda.so is not built")


def golden(name):
    return os.path.join(GOLDEN, name)


def read_lines(name):
    opener = gzip.open if name.endswith(".gz") else open
    with opener(golden(name), "rt", encoding="utf-8") as f:
        return [json.loads(ln) for ln in f if ln.strip()]


_ORACLE = {}


def oracle():
    if not _ORACLE:
        with open(golden("tokenizer_unicode-oracle.json")) as f:
            _ORACLE.update(json.load(f))
    return _ORACLE


def scalars():
    return [c for c in range(MAX_SCALAR) if c < 0xD800 or c > 0xDFFF]


def hexs(s: str) -> str:
    return " ".join(f"{ord(c):x}" for c in s)


def split_many(texts):
    """The pieces of each text, in one native call: the texts joined by '\\n', each of which must come back as a
    piece of its own (the texts hold no '\\n' and end in a letter, which keeps every separator apart)."""
    assert not any("\n" in t for t in texts)
    pieces = T.split("\n".join(texts))
    out = [[]]
    for p in pieces:
        if p == "\n":
            out.append([])
        else:
            assert "\n" not in p, repr(p)
            out[-1].append(p)
    assert len(out) == len(texts)
    return out


def nfc_many(texts):
    """The NFC of each text, in one native call. '\\n' is a starter that composes with nothing and is no split point,
    so NFC of the joined text is the join of the NFCs."""
    assert not any("\n" in t for t in texts)
    out = T.nfc("\n".join(texts)).split("\n")
    assert len(out) == len(texts)
    return out


# ---- pins (UnicodeTests.fs:367-431) ----------------------------------------------------------------------------------

DATA_PINS = {
    "tokenizer_unicode-oracle.json": "f9339ab0e55acabd0509b4f562ae831d97d167398aaeacbd47c4a49324acbb89",
    "tokenizer_split-cases.jsonl": "39bb2555c870896ecb4bc4c907c90a1dcb912aaf8ed75a143aee114c35bb3b95",
    "tokenizer_encode-cases.jsonl.gz": "3ce0e0e7473f4e6465b92ba3482c31682d61d7c48645b535a987940bdd6743dd",
    "tokenizer_corpus-cases.jsonl.gz": "35ff0c43a1bc4325588b1a22953f861784e4ca76e0f3f863a5f70ff9ceb16c66",
}


@pytest.mark.parametrize("name", sorted(DATA_PINS))
def test_oracle_data_has_the_contract_sha256(name):
    with open(golden(name), "rb") as f:
        data = f.read()
    if name.endswith(".gz"):
        data = gzip.decompress(data)
    assert hashlib.sha256(data).hexdigest() == DATA_PINS[name]


def test_probe_facts_versions_pin_and_pattern():
    meta = oracle()["meta"]
    assert meta["tokenizers"] == "0.23.3"
    assert meta["tokenizer_sha256"] == T.PINNED_SHA256
    assert meta["pattern"] == T.SPLIT_PATTERN


def test_generated_unicode_tables_match_their_sources(tmp_path):
    """csrc/unicode_tables.g.h is what gen_unicode_tables.py writes from the oracle probe and unicodedata."""
    out = tmp_path / "unicode_tables.g.h"
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    subprocess.run([sys.executable, "-m", "rosylnalive_b200.gen_unicode_tables",
                    golden("tokenizer_unicode-oracle.json"), str(out)], check=True, cwd=root, capture_output=True)
    with open(os.path.join(root, "rosylnalive_b200", "csrc", "unicode_tables.g.h")) as f:
        committed = f.read()
    assert out.read_text() == committed


# ---- byte level (PreTokenizerTests.fs:99-136, vector B1) -------------------------------------------------------------

def test_b1_byte_map():
    for b, c in [(0x00, 0x100), (0x09, 0x109), (0x0A, 0x10A), (0x20, 0x120), (0x21, 0x21), (0x7E, 0x7E),
                 (0x7F, 0x121), (0xA0, 0x142), (0xA1, 0xA1), (0xAC, 0xAC), (0xAD, 0x143), (0xFF, 0xFF)]:
        assert T.byte_char(b) == chr(c), hex(b)


def test_byte_map_is_a_bijection_with_68_moved_bytes():
    chars = [T.byte_char(b) for b in range(256)]
    assert len(set(chars)) == 256
    assert sorted(c for c in chars if ord(c) >= 0x100) == [chr(c) for c in range(0x100, 0x144)]


# ---- the Split pre-tokenizer (PreTokenizerTests.fs:11-97, vectors P1 to P18) -----------------------------------------

SPLIT_VECTORS = [
    ("Hello world", ["Hello", " world"]),
    ("it's", ["it", "'s"]),
    ("WE'RE 'Sa", ["WE", "'RE", " '", "Sa"]),
    ("x'\u017fa", ["x", "'\u017f", "a"]),
    ("  hi", [" ", " hi"]),
    ("a  \n\n  b", ["a", "  \n\n", " ", " b"]),
    ("end   ", ["end", "   "]),
    ("12345", ["1", "2", "3", "4", "5"]),
    ("x\u00bd\u216b", ["x", "\u00bd", "\u216b"]),
    (" !!\r\n\r\nx", [" !!\r\n\r\n", "x"]),
    ("\tfoo", ["\tfoo"]),
    ("\u3000\u4e2d\u6587", ["\u3000\u4e2d\u6587"]),
    ("\U0001D400\U0001D401", ["\U0001D400\U0001D401"]),
    ("a\r\nb", ["a", "\r\n", "b"]),
    ("x \u0301y", ["x", " \u0301", "y"]),
    ("'ll've", ["'ll", "'ve"]),
    ("don't'", ["don", "'t", "'"]),
    ("\U0001D7CE\U0001D7CF", ["\U0001D7CE", "\U0001D7CF"]),
]


@pytest.mark.parametrize("k", range(len(SPLIT_VECTORS)), ids=[f"P{k + 1}" for k in range(len(SPLIT_VECTORS))])
def test_split_vectors_p1_to_p18(k):
    text, pieces = SPLIT_VECTORS[k]
    assert T.split(text) == pieces


def test_every_oracle_split_case():
    cases = read_lines("tokenizer_split-cases.jsonl")
    assert len(cases) >= 4000
    bad = [(c["text"], T.split(c["text"]), c["pieces"]) for c in cases if T.split(c["text"]) != c["pieces"]]
    assert not bad, f"{len(bad)} of {len(cases)} split cases differ, first: {bad[:5]}"


def test_pieces_tile_the_text_and_the_empty_text_has_none():
    for c in read_lines("tokenizer_split-cases.jsonl"):
        assert "".join(T.split(c["text"])) == c["text"]
    assert T.split("") == []


def test_astral_letters_and_numbers_are_classified_by_scalar():
    """The cases where a UTF-16 regex engine splits surrogate pairs (UnicodeTests.fs:316-338): the state machine
    classifies scalars."""
    bold, digit = "\U0001D400\U0001D401", "\U0001D7CE"
    assert T.split("a" + bold + "b") == ["a" + bold + "b"]
    assert T.split("x" + digit + digit) == ["x", digit, digit]
    assert T.split("\U00020000a") == ["\U00020000a"]


# ---- classes (UnicodeTests.fs:74-176, vector U1) ---------------------------------------------------------------------

def test_every_scalar_class_equals_the_oracle():
    runs = oracle()["classes"]
    want_code = {"L": "letter", "N": "number", "S": "space", "O": "other"}
    bad, n = [], 0
    counts = {"letter": 0, "number": 0, "space": 0, "other": 0}
    for i, (start, k) in enumerate(runs):
        stop = runs[i + 1][0] if i + 1 < len(runs) else MAX_SCALAR
        if k == "X":
            continue
        for c in range(start, stop):
            n += 1
            got = T.char_class(c)
            counts[got] += 1
            if got != want_code[k]:
                bad.append(f"U+{c:04X} is {got}, the oracle says {want_code[k]}")
    assert n == 1_112_064
    assert not bad, bad[:20]
    assert counts["letter"] == 141_028 and counts["number"] == 1_911 and counts["space"] == 25


CONTRACTION_PROBES = [
    ("s|t|m|d", lambda ch: "'" + ch + "a", 2),
    ("r|v (first of 're 've)", lambda ch: "'" + ch + "ea", 3),
    ("e (second of 're)", lambda ch: "'r" + ch + "a", 3),
    ("e (second of 've)", lambda ch: "'v" + ch + "a", 3),
    ("l (first of 'll)", lambda ch: "'" + ch + "la", 3),
    ("l (second of 'll)", lambda ch: "'l" + ch + "a", 3),
]


@pytest.mark.parametrize("probe", range(len(CONTRACTION_PROBES)), ids=[p[0] for p in CONTRACTION_PROBES])
def test_contraction_group_matches_exactly_the_oracle_letters(probe):
    name, build, length = CONTRACTION_PROBES[probe]
    letters = [c for c in scalars() if T.char_class(c) == "letter"]
    got = set()
    for c, pieces in zip(letters, split_many([build(chr(c)) for c in letters])):
        if len(pieces) == 2 and len(pieces[0]) == length:
            got.add(c)
    want = set(oracle()["contraction_letters"][name])
    assert got == want, (sorted(want - got)[:10], sorted(got - want)[:10])


def test_contraction_letters_u1():
    """U1: D M S T d m s t U+017F, then R V r v, E e and L l."""
    got = {chr(c) for c in scalars() if T.contraction_letter(c)}
    assert got == set("DMSTdmst\u017fRVrvEeLl")
    assert T.contraction_letter(0x17F) == "s" and T.contraction_letter(ord("R")) == "r"


def test_only_u0027_opens_a_contraction():
    want = set(oracle()["apostrophes"])
    assert want == {0x27}
    cs = [c for c in scalars() if c != 0x0A]
    opens = {c for c, pieces in zip(cs, split_many(["x" + chr(c) + "sa" for c in cs]))
             if pieces == ["x", chr(c) + "s", "a"]}
    if T.split("x\nsa") == ["x", "\ns", "a"]:
        opens.add(0x0A)
    assert opens == want


# ---- NFC (UnicodeTests.fs:178-310) -----------------------------------------------------------------------------------

FAMILIES = {
    "F1": lambda ch: ch,
    "F2": lambda ch: "a" + ch + "\u0334",
    "F3": lambda ch: "a\u0345" + ch,
    "F5": lambda ch: ch + "\u0301",
    "F6": lambda ch: "a" + ch,
    "F7": lambda ch: ch + "\u0308",
    "F8": lambda ch: "\u1100" + ch,
    "F9": lambda ch: "\uac00" + ch,
}


def expect_family(name, lines):
    want = oracle()["nfc"][name]
    h = hashlib.sha256()
    for ln in lines:
        h.update(ln.encode("utf-8"))
    assert (len(lines), h.hexdigest()) == (want["count"], want["sha256"]), name


@pytest.mark.parametrize("name", sorted(FAMILIES))
def test_nfc_family_equals_the_oracle_on_every_scalar(name):
    build = FAMILIES[name]
    cs = scalars()
    batch = [c for c in cs if c != 0x0A]
    outs = dict(zip(batch, nfc_many([build(chr(c)) for c in batch])))
    outs[0x0A] = T.nfc(build("\n"))
    lines = []
    for c in cs:
        s, out = build(chr(c)), outs[c]
        if out != s:
            lines.append(f"{name} {c:x} {hexs(out)}\n")
    expect_family(name, lines)


def test_nfc_family_p_every_pair_of_reordering_marks():
    marks = [c for a, b in oracle()["marks"] for c in range(a, b + 1)]
    inputs = [(m1, m2, "a" + chr(m1) + chr(m2)) for m1 in marks for m2 in marks]
    outs = nfc_many([s for _, _, s in inputs])
    lines = [f"P {m1:x} {m2:x} {hexs(out)}\n" for (m1, m2, s), out in zip(inputs, outs) if out != s]
    expect_family("P", lines)


def test_nfc_family_k_every_canonical_decomposition_recomposed():
    inputs = ["".join(chr(int(h, 16)) for h in x.split(" ")) for x in oracle()["composition_inputs"]]
    outs = nfc_many(inputs)
    lines = [f"K {i} {hexs(out)}\n" for i, (s, out) in enumerate(zip(inputs, outs)) if out != s]
    expect_family("K", lines)


def test_ufffe_passes_through_nfc_unchanged():
    assert T.nfc("e\u0301\ufffea\u0308") == "\u00e9\ufffe\u00e4"


def test_a_mark_newer_than_unicode_9_is_not_reordered():
    """U+07FD NKO DANTAYALAN (Unicode 11, ccc 220) is inert in the oracle; a current NFC would move U+0334 before it."""
    import unicodedata

    assert unicodedata.normalize("NFC", "a\u07fd\u0334") == "a\u0334\u07fd"
    assert T.nfc("a\u07fd\u0334") == "a\u07fd\u0334"


def test_hangul_composes_by_arithmetic():
    assert T.nfc("\u1100\u1161") == "\uac00"
    assert T.nfc("\uac00\u11a8") == "\uac01"
    assert T.nfc("\u1100\u1161\u11a8") == "\uac01"


# ---- the toy tokenizer (ToyTests.fs) ---------------------------------------------------------------------------------

def bl(s: str) -> str:
    return T.byte_level(s.encode("utf-8"))


TOY_MERGES = [(" ", "t"), ("h", "e"), (" t", "he"), ("a", "a"), ("b", "c"), ("a", "b"), ("aa", "aa")]
TOY_ADDED = [("<|a|>", True), ("<|ab|>", True), ("<x>", False)]


def toy_json(edit=None) -> bytes:
    """A tokenizer.json with Qwen's configuration, the 256 byte tokens, 7 merges (ids 256-262) and 3 added tokens
    (263-265): the reference's toy model (ToyTests.fs:17-110)."""
    vocab = {T.byte_char(b): b for b in range(256)}
    for i, (l, r) in enumerate(TOY_MERGES):
        vocab[bl(l) + bl(r)] = 256 + i
    byte_level = lambda: {"type": "ByteLevel", "add_prefix_space": False, "trim_offsets": False,  # noqa: E731
                          "use_regex": False}
    root = {
        "version": "1.0", "truncation": None, "padding": None,
        "added_tokens": [{"id": 256 + len(TOY_MERGES) + i, "content": c, "single_word": False, "lstrip": False,
                          "rstrip": False, "normalized": False, "special": s} for i, (c, s) in enumerate(TOY_ADDED)],
        "normalizer": {"type": "NFC"},
        "pre_tokenizer": {"type": "Sequence", "pretokenizers": [
            {"type": "Split", "pattern": {"Regex": T.SPLIT_PATTERN}, "behavior": "Isolated", "invert": False},
            byte_level()]},
        "post_processor": byte_level(),
        "decoder": byte_level(),
        "model": {"type": "BPE", "dropout": None, "unk_token": None, "continuing_subword_prefix": "",
                  "end_of_word_suffix": "", "fuse_unk": False, "byte_fallback": False, "ignore_merges": False,
                  "vocab": vocab, "merges": [[bl(l), bl(r)] for l, r in TOY_MERGES]},
    }
    if edit:
        edit(root)
    return json.dumps(root).encode("utf-8")


_TOY = []


def toy() -> T.QwenTokenizer:
    if not _TOY:
        _TOY.append(T.QwenTokenizer.parse(toy_json()))
    return _TOY[0]


def id_of(s):
    return toy().id_of(bl(s))


def byte_ids(s):
    return [toy().id_of(T.byte_char(b)) for b in s.encode("utf-8")]


def test_bpe_merges_lowest_rank_first_and_leftmost_among_ties():
    t = toy()
    assert t.encode(" the") == [id_of(" the")]
    assert t.encode("abc") == [id_of("a"), id_of("bc")]  # 'bc' (rank 4) before 'ab' (rank 5)
    assert t.encode("aaa") == [id_of("aa"), id_of("a")]  # the leftmost 'aa' first
    assert t.encode("aaaa") == [id_of("aaaa")]
    assert t.encode("aaaaa") == [id_of("aaaa"), id_of("a")]
    assert t.encode("") == []


def test_long_texts_and_pieces_encode_like_short_ones():
    t = toy()
    ids = t.encode("a" * 100_001)
    assert len(ids) == 25_001 and all(i == id_of("aaaa") for i in ids[:25_000]) and ids[-1] == id_of("a")
    assert t.encode(" the" * 30_000) == [id_of(" the")] * 30_000
    assert t.encode(" the aa") == [id_of(" the"), id_of(" "), id_of("aa")]


def test_added_tokens_match_first_leftmost_longest_on_the_raw_text():
    t = toy()
    assert t.encode("<|ab|>") == [264]
    assert t.encode("<|a|><|ab|>") == [263, 264]
    assert t.encode("x<x>y") == byte_ids("x") + [265] + byte_ids("y")
    assert t.encode("<|a") == byte_ids("<|a")
    assert t.encode("<<x>") == byte_ids("<") + [265]


def test_nfc_runs_on_each_stretch_between_added_tokens():
    t = toy()
    assert t.encode("e\u0301") == byte_ids("\u00e9")
    assert t.encode("e<x>\u0301") == byte_ids("e") + [265] + byte_ids("\u0301")


@pytest.mark.parametrize("units", ["d800", "0061dc00", "0061d800d8000062", "dfff0061"])
def test_a_lone_surrogate_is_rejected(units):
    s = T._from_utf16_hex(units)
    with pytest.raises(ValueError):
        toy().encode(s)


def test_a_surrogate_pair_is_encoded():
    s = T._from_utf16_hex("d83dde00")
    assert s == "\U0001F600"
    assert toy().encode(s) == byte_ids(s)


def test_invalid_utf8_at_the_c_abi_is_refused():
    import ctypes

    t = toy()
    n = ctypes.c_uint64()
    bad = b"a\xed\xa0\x80b"  # a UTF-8-encoded surrogate
    assert native.lib().lrm_tok_encode(t._h, bad, len(bad), None, 0, ctypes.byref(n)) == native.LRM_ERR_ARGUMENT
    assert "not valid UTF-8" in native.last_error()


def test_encode_bytes_replaces_each_maximal_invalid_subpart():
    t = toy()
    assert t.encode_bytes(b"\x80") == byte_ids("\ufffd")
    assert t.encode_bytes(b"\xe4\xb8") == byte_ids("\ufffd")
    assert t.encode_bytes(b"a\xf0\x80b") == byte_ids("a\ufffd\ufffdb")
    for raw in [b"\xed\xa0\x80", b"\xf4\x90\x80\x80", b"\xc0\xaf", b"\xe0\x80\xaf", b"\xf0\x9f\x98", b"\xff\xfe",
                b"\xe2\x82\xacx\xe2\x82"]:
        assert t.encode_bytes(raw) == byte_ids(raw.decode("utf-8", errors="replace")), raw


def test_decode_bytes_of_tokens_added_tokens_and_rows_with_no_token():
    t = toy()
    assert t.decode_bytes([id_of(" the")]) == b" the"
    assert t.decode([263, 265]) == "<|a|><x>"
    assert t.decode_bytes([]) == b""
    assert t.decode_bytes([t.vocab_size, 151_935]) == b""
    zhong = byte_ids("\u4e2d")
    assert t.decode([zhong[0], 151_700, zhong[1], zhong[2]]) == "\u4e2d"


def test_decode_is_errors_replace():
    t = toy()
    zhong = byte_ids("\u4e2d")
    assert t.decode([zhong[0]]) == "\ufffd"
    assert t.decode([zhong[0], zhong[1], id_of("a")]) == "\ufffda"


@pytest.mark.parametrize("bad", [-1, T.MODEL_ROWS, 2**31 - 1])
def test_ids_outside_the_model_raise(bad):
    with pytest.raises(ValueError):
        toy().decode_bytes([bad])
    with pytest.raises(ValueError):
        toy().decode([1, bad])


def test_id_of_and_token_of():
    t = toy()
    assert t.id_of("<|ab|>") == 264
    assert t.id_of(bl(" the")) == 258
    assert t.id_of(" the") is None
    assert t.token_of(258) == bl(" the")
    assert t.token_of(265) == "<x>"
    assert t.token_of(266) is None and t.token_of(-1) is None
    assert t.vocab_size == 266 and t.merge_count == 7
    assert [a.special for a in t.added_tokens] == [True, True, False]


def _pre(r):
    return r["pre_tokenizer"]["pretokenizers"]


REFUSALS = [
    ("another regex", lambda r: _pre(r)[0]["pattern"].__setitem__("Regex", r"\p{L}+|\s+")),
    ("behaviour Removed", lambda r: _pre(r)[0].__setitem__("behavior", "Removed")),
    ("ByteLevel with use_regex", lambda r: _pre(r)[1].__setitem__("use_regex", True)),
    ("ByteLevel without use_regex", lambda r: _pre(r)[1].pop("use_regex")),
    ("add_prefix_space", lambda r: _pre(r)[1].__setitem__("add_prefix_space", True)),
    ("NFKC", lambda r: r["normalizer"].__setitem__("type", "NFKC")),
    ("dropout", lambda r: r["model"].__setitem__("dropout", 0.1)),
    ("byte fallback", lambda r: r["model"].__setitem__("byte_fallback", True)),
    ("ignore_merges", lambda r: r["model"].__setitem__("ignore_merges", True)),
    ("an unknown token", lambda r: r["model"].__setitem__("unk_token", "<unk>")),
    ("a normalized added token", lambda r: r["added_tokens"][0].__setitem__("normalized", True)),
    ("an lstrip added token", lambda r: r["added_tokens"][1].__setitem__("lstrip", True)),
    ("an added token id gap", lambda r: r["added_tokens"][2].__setitem__("id", 300)),
    ("a merge of an unknown token", lambda r: r["model"]["merges"].append(["zz", "a"])),
    ("a merge whose result is missing", lambda r: r["model"]["merges"].append(["b", "b"])),
    ("a vocabulary id gap", lambda r: r["model"]["vocab"].__setitem__(bl(" the"), 999)),
    ("a decoder that is not ByteLevel", lambda r: r["decoder"].__setitem__("type", "WordPiece")),
    ("a model that is not BPE", lambda r: r["model"].__setitem__("type", "Unigram")),
]


def test_the_toy_file_parses():
    assert T.QwenTokenizer.parse(toy_json()).vocab_size == 266


@pytest.mark.parametrize("k", range(len(REFUSALS)), ids=[r[0] for r in REFUSALS])
def test_loader_refuses(k):
    with pytest.raises(T.TokenizerFormatError, match="tokenizer.json"):
        T.QwenTokenizer.parse(toy_json(REFUSALS[k][1]))


def test_loader_refusal_messages_follow_the_reference():
    def msg(edit):
        with pytest.raises(T.TokenizerFormatError) as e:
            T.QwenTokenizer.parse(toy_json(edit))
        return str(e.value)

    assert "tokenizer.json: normalizer.type is 'NFKC', only 'NFC' is supported" in msg(REFUSALS[5][1])
    assert "added token ids must follow the vocabulary (265 expected, 300 found)" in msg(REFUSALS[12][1])
    assert "model.merges[7] names 'zz', which is not in the vocabulary" in msg(REFUSALS[13][1])
    assert "model.vocab has no token for byte 0x41" in msg(
        lambda r: r["model"]["vocab"].__setitem__("AA", r["model"]["vocab"].pop("A")))
    with pytest.raises(T.TokenizerFormatError, match="is not valid JSON"):
        T.QwenTokenizer.parse(b'{"model": ')
    with pytest.raises(T.TokenizerFormatError, match="appears twice"):
        T.QwenTokenizer.parse(toy_json(lambda r: r["added_tokens"][2].__setitem__("content", "<|a|>")))
    with pytest.raises(T.TokenizerFormatError, match="repeats the pair"):
        T.QwenTokenizer.parse(toy_json(lambda r: r["model"]["merges"].append([bl("a"), bl("a")])))


def test_string_merges_are_accepted():
    t = T.QwenTokenizer.parse(toy_json(lambda r: r["model"].__setitem__(
        "merges", [f"{bl(l)} {bl(r)}" for l, r in TOY_MERGES])))
    assert t.encode(" the aaaa") == toy().encode(" the aaaa")


def test_load_refuses_a_file_whose_sha256_is_not_the_pin(tmp_path):
    p = tmp_path / "tokenizer.json"
    p.write_bytes(toy_json())
    with pytest.raises(T.TokenizerFormatError) as e:
        T.QwenTokenizer.load(str(p))
    assert T.PINNED_SHA256 in str(e.value)
    with pytest.raises(FileNotFoundError):
        T.QwenTokenizer.load(str(tmp_path / "absent.json"))


def test_the_pin():
    assert T.PINNED_SHA256 == "aeb13307a71acd8fe81861d94ad54ab689df773318809eed3cbe794b4492dae4"
    assert T.PINNED_PATH == "models/Qwen3-0.6B/tokenizer.json"


def _parallel(fn, items, threads=8):
    out = [None] * len(items)

    def work(k):
        for i in range(k, len(items), threads):
            out[i] = fn(items[i])

    ts = [threading.Thread(target=work, args=(k,)) for k in range(threads)]
    for th in ts:
        th.start()
    for th in ts:
        th.join()
    return out


def test_encode_is_thread_safe_8_threads_give_the_sequential_ids():
    t = T.QwenTokenizer.parse(toy_json())
    texts = [c["text"] for c in read_lines("tokenizer_split-cases.jsonl")]
    sequential = [t.encode(s) for s in texts]
    t.clear_cache()
    assert _parallel(t.encode, texts) == sequential
    assert t.cached_pieces > 0


def _word(i):
    letters = []
    n = i
    while True:
        letters.append(chr(97 + n % 26))
        if n < 26:
            break
        n = n // 26 - 1
    return " w" + "".join(reversed(letters))


def test_piece_cache_holds_at_most_capacity_over_generation_swaps():
    t = T.QwenTokenizer.parse(toy_json())
    cold = T.QwenTokenizer.parse(toy_json())
    cap = T.CACHE_CAPACITY
    assert cap == 65_536
    words = [_word(i) for i in range(3 * cap)]
    assert len(set(words)) == len(words)
    t.clear_cache()
    assert t.cached_pieces == 0
    most, first = 0, []
    for w in words:
        first.append(t.encode(w))
        most = max(most, t.cached_pieces)
    assert cap // 2 < most <= cap
    assert [t.encode(w) for w in words] == first
    for i in range(0, len(words), 97):
        cold.clear_cache()
        assert cold.encode(words[i]) == first[i]
    p = T.QwenTokenizer.parse(toy_json())
    assert _parallel(p.encode, words) == first
    assert p.cached_pieces <= cap + 2 * 8


def test_only_pieces_of_at_most_cached_piece_units_are_cached():
    t = T.QwenTokenizer.parse(toy_json())
    limit = T.CACHED_PIECE_UNITS
    assert limit == 65_536

    def cached_after(text):
        t.clear_cache()
        ids = t.encode(text)
        assert t.encode(text) == ids
        return t.cached_pieces

    assert cached_after("b" * 300) == 1
    assert cached_after("b" * limit) == 1
    assert cached_after("b" * (limit + 1)) == 0
    assert cached_after("\U0001F600" * (limit // 2)) == 1  # 2 UTF-16 units each
    assert cached_after("\U0001F600" * (limit // 2 + 1)) == 0


def test_piece_cache_holds_about_cache_units_of_long_pieces():
    t = T.QwenTokenizer.parse(toy_json())
    limit = T.CACHED_PIECE_UNITS
    assert T.CACHE_UNITS == 1 << 21
    most = 0
    for i in range(64):
        t.encode("b" * (limit - i))
        most = max(most, t.cached_pieces)
    assert T.CACHE_UNITS // 2 // limit < most <= (T.CACHE_UNITS + 2 * limit) // (limit - 63)


def test_decoding_the_encoding_gives_the_nfc_text_back():
    t = toy()
    for c in read_lines("tokenizer_split-cases.jsonl"):
        assert t.decode(t.encode(c["text"])) == T.nfc(c["text"])


# ---- the corpus runner on the toy tokenizer (CorpusTests.fs) ---------------------------------------------------------

def test_corpus_runner_applies_each_kind_rule():
    t = toy()
    lines = [
        {"kind": "encode", "id": "e-ok", "text": " the", "ids": [258]},
        {"kind": "encode", "id": "e-bad", "text": " the", "ids": [258, 1]},
        {"kind": "encode_bytes", "id": "b-ok", "bytes": "61f08062", "text": "a\ufffd\ufffdb",
         "ids": byte_ids("a\ufffd\ufffdb")},
        {"kind": "encode_bytes", "id": "b-text", "bytes": "80", "text": "x", "ids": []},
        {"kind": "decode", "id": "d-ok", "ids": [263, 265], "text": "<|a|><x>", "bytes": b"<|a|><x>".hex()},
        {"kind": "decode", "id": "d-bytes", "ids": [263], "text": "<|a|>", "bytes": "00"},
        {"kind": "decode", "id": "d-text", "ids": [263], "text": "<x>"},
        {"kind": "encode_reject", "id": "r-ok", "utf16": "0061d800"},
        {"kind": "encode_reject", "id": "r-bad", "utf16": "0061"},
        {"kind": "teleport", "id": "k-bad"},
        {"kind": "decode", "id": "d-range", "ids": [-1], "text": ""},
    ]
    text = "\n".join(json.dumps(x) for x in lines) + "\n\nnot json\n"
    got = {c.id: c for c in T.run_corpus(t, text)}
    assert {k for k, c in got.items() if c.passed} == {"e-ok", "b-ok", "d-ok", "r-ok"}
    assert "ids differ at 1" in got["e-bad"].detail
    assert "errors=replace" in got["b-text"].detail
    assert "DecodeBytes differs" in got["d-bytes"].detail
    assert "Decode gave" in got["d-text"].detail
    assert "accepted a text with a lone surrogate" in got["r-bad"].detail
    assert "unknown kind 'teleport'" in got["k-bad"].detail
    assert got["d-range"].detail.startswith("ValueError")
    assert got["corpus:13"].category == "invalid"
    assert got["e-ok"].category == "probe-encode" and got["e-ok"].tokens == 1


# ---- with the real tokenizer.json (skipped visibly without it) -------------------------------------------------------

_REAL = []


def real():
    if not _REAL:
        _REAL.append(T.QwenTokenizer.try_load_default())
    if _REAL[0] is None:
        pytest.skip(f"tokenizer.json is not at {T.QwenTokenizer.default_path()} (set LRM_DATA): SKIPPED, not passed")
    return _REAL[0]


ENCODE_VECTORS = [
    ("Hello world", [9707, 1879]),
    ("using System;", [970, 739, 26]),
    ("<|im_start|>user\nHi<|im_end|>", [151644, 872, 198, 13048, 151645]),
    ("e\u0301", [963]),
    ("\U0001F600", [141334]),
    ("a\u07fd\u0334", [64, 155, 121, 136, 112]),
    ("x\ufffe\u0301", [87, 5564, 122, 53839]),
    ("public static int Add(int a, int b) => a + b;",
     [888, 1099, 526, 2691, 1548, 264, 11, 526, 293, 8, 589, 264, 488, 293, 26]),
    ("", []),
    (" ", [220]),
    ("\u4e2d\u6587", [104811]),
]
DECODE_VECTORS = [([151643], "<|endoftext|>"), ([9707, 1879], "Hello world"), ([160, 151700, 116, 255], "\u4e2d"),
                  ([5691], "\ufffd"), ([151669], ""), ([], "")]


@pytest.mark.parametrize("k", range(len(ENCODE_VECTORS)), ids=[f"E{k + 1}" for k in range(len(ENCODE_VECTORS))])
def test_real_encode_vectors(k):
    text, ids = ENCODE_VECTORS[k]
    assert real().encode(text) == ids


@pytest.mark.parametrize("k", range(len(DECODE_VECTORS)), ids=[f"D{k + 1}" for k in range(len(DECODE_VECTORS))])
def test_real_decode_vectors(k):
    ids, text = DECODE_VECTORS[k]
    assert real().decode(ids) == text


def test_real_added_tokens_a1_round_trip():
    t = real()
    assert len(t.added_tokens) == 26
    assert [a.id for a in t.added_tokens] == list(range(151643, 151669))
    assert all(a.special == (a.id <= 151656) for a in t.added_tokens)
    for a in t.added_tokens:
        assert t.encode(a.content) == [a.id] and t.decode([a.id]) == a.content and t.id_of(a.content) == a.id


def test_real_counts_and_every_id_maps_to_its_token_and_back():
    t = real()
    assert (t.vocab_size, t.merge_count) == (T.REAL_IDS, 151_387)
    for i in range(t.vocab_size):
        assert t.id_of(t.token_of(i)) == i
    assert t.encode("Hello")[0] != 151643  # no BOS


@pytest.mark.parametrize("name", ["tokenizer_encode-cases.jsonl.gz", "tokenizer_corpus-cases.jsonl.gz"])
def test_real_corpus_is_exact(name):
    t = real()
    with gzip.open(golden(name), "rt", encoding="utf-8") as f:
        cases = T.run_corpus(t, f.read(), name)
    bad = [c for c in cases if not c.passed]
    assert not bad, f"{len(bad)} of {len(cases)} differ, first: {bad[:5]}"
