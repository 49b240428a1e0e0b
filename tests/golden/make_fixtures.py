"""Extracts the reference's committed tiny-model goldens into tests/golden/tiny_g1.npz.

Run once in a checkout that holds the reference (it is read-only input here):

    python tests/golden/make_fixtures.py /path/to/reference

Source: the reference's goldens/tiny/g1 set (README "The tiny set"): HF-named bf16 weights (model/model.safetensors),
the pinned RoPE inverse frequencies and T_spec table (rope.safetensors), torch32 (fwd_f32.*) and torch64p (fwd_f64p.*)
forward taps for prompts p0 (T=13) and p1 (T=1), logits for p2 (T=70) and the 64-step greedy ids and margins
(greedy.safetensors). Nothing is recomputed: the arrays are copied as they are, bit for bit, so the tests can run
where the reference is absent (the GPU box). The model file is also copied whole (tiny_g1_model.safetensors, checked
against the reference's SHA256SUMS) for the safetensors reader's tests, and the tokenizer oracle's Unicode and split
probes (tokenizer_unicode-oracle.json, tokenizer_split-cases.jsonl).
"""

from __future__ import annotations

import gzip
import json
import os
import struct
import sys

import numpy as np

_DTYPES = {"F32": np.float32, "F64": np.float64, "I64": np.int64, "U32": np.uint32, "BF16": np.uint16,
           "I32": np.int32, "U16": np.uint16}


def read_safetensors(path: str) -> dict:
    """Minimal safetensors reader (8-byte little-endian header length, JSON header, raw little-endian data).
    BF16 tensors come back as their uint16 bit patterns."""
    with open(path, "rb") as f:
        raw = f.read()
    (n,) = struct.unpack_from("<Q", raw, 0)
    header = json.loads(raw[8:8 + n])
    base = 8 + n
    out = {}
    for name, meta in header.items():
        if name == "__metadata__":
            continue
        dt = _DTYPES[meta["dtype"]]
        lo, hi = meta["data_offsets"]
        out[name] = np.frombuffer(raw[base + lo:base + hi], dtype=dt).reshape(meta["shape"]).copy()
    return out


def main(reference_root: str) -> None:
    g = os.path.join(reference_root, "goldens", "tiny", "g1")
    arrays = {}
    with open(os.path.join(g, "model", "config.json")) as f:
        arrays["config_json"] = np.frombuffer(f.read().encode(), np.uint8)
    with open(os.path.join(g, "manifest.json")) as f:
        manifest = json.load(f)
    for name, t in read_safetensors(os.path.join(g, "model", "model.safetensors")).items():
        arrays["w/" + name] = t
    rope = read_safetensors(os.path.join(g, "rope.safetensors"))
    for k, v in rope.items():
        arrays["rope/" + k] = v
    for p in ("p0", "p1", "p2"):
        for oracle, tag in (("fwd_f32", "torch32"), ("fwd_f64p", "torch64p")):
            for k, v in read_safetensors(os.path.join(g, f"{oracle}.{p}.safetensors")).items():
                arrays[f"{tag}/{p}/{k}"] = v
    for k, v in read_safetensors(os.path.join(g, "greedy.safetensors")).items():
        arrays["greedy/" + k] = v
    for pr in manifest["prompts"]:
        arrays["prompt/" + pr["name"]] = np.array(pr["ids"], np.int64)
    here = os.path.dirname(os.path.abspath(__file__))
    out = os.path.join(here, "tiny_g1.npz")
    np.savez_compressed(out, **arrays)
    print(f"wrote {out}: {len(arrays)} arrays, {os.path.getsize(out)} bytes")
    # The model file itself, byte for byte, for the safetensors reader's tests; its SHA-256 must be the one the
    # reference's goldens/tiny/g1/model/SHA256SUMS lists.
    import hashlib
    import shutil

    src = os.path.join(g, "model", "model.safetensors")
    with open(os.path.join(g, "model", "SHA256SUMS")) as f:
        want = next(ln.split()[0] for ln in f if ln.strip().endswith("model.safetensors"))
    with open(src, "rb") as f:
        got = hashlib.sha256(f.read()).hexdigest()
    if got != want:
        raise SystemExit(f"{src}: SHA-256 {got}, SHA256SUMS says {want}")
    dst = os.path.join(here, "tiny_g1_model.safetensors")
    shutil.copyfile(src, dst)
    os.chmod(dst, 0o644)
    print(f"copied {src} -> {dst} (SHA-256 {got})")
    # The tokenizer oracle's probes that need no tokenizer.json (tests/Lrm.Tokenizer.Tests/oracle, pinned by the
    # SHA-256s of docs/contracts/tokenizer.md "Vectors"): Unicode classes, contraction letters, NFC split points and
    # probe digests, and 4,000 pre-tokenizer split cases.
    for name, want in (("unicode-oracle.json", "f9339ab0e55acabd0509b4f562ae831d97d167398aaeacbd47c4a49324acbb89"),
                       ("split-cases.jsonl", "39bb2555c870896ecb4bc4c907c90a1dcb912aaf8ed75a143aee114c35bb3b95")):
        src = os.path.join(reference_root, "tests", "Lrm.Tokenizer.Tests", "oracle", name)
        with open(src, "rb") as f:
            data = f.read()
        got = hashlib.sha256(data).hexdigest()
        if got != want:
            raise SystemExit(f"{src}: SHA-256 {got}, the tokenizer contract pins {want}")
        dst = os.path.join(here, "tokenizer_" + name)
        with open(dst, "wb") as f:
            f.write(data)
        print(f"copied {src} -> {dst} (SHA-256 {got})")
    # The id vectors that need the real tokenizer.json (the 1,800 oracle probe cases and O1's 5,597-case corpus,
    # goldens/tokenizer/g1), gzip-compressed with a zero timestamp; the tests check the SHA-256 of the content.
    for src_rel, name, want in (
            ("tests/Lrm.Tokenizer.Tests/oracle/encode-cases.jsonl", "tokenizer_encode-cases.jsonl.gz",
             "3ce0e0e7473f4e6465b92ba3482c31682d61d7c48645b535a987940bdd6743dd"),
            ("goldens/tokenizer/g1/cases.jsonl", "tokenizer_corpus-cases.jsonl.gz",
             "35ff0c43a1bc4325588b1a22953f861784e4ca76e0f3f863a5f70ff9ceb16c66")):
        src = os.path.join(reference_root, *src_rel.split("/"))
        with open(src, "rb") as f:
            data = f.read()
        got = hashlib.sha256(data).hexdigest()
        if got != want:
            raise SystemExit(f"{src}: SHA-256 {got}, the tokenizer contract pins {want}")
        dst = os.path.join(here, name)
        with open(dst, "wb") as f:
            f.write(gzip.compress(data, compresslevel=9, mtime=0))
        print(f"copied {src} -> {dst} (SHA-256 of the content {got})")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        raise SystemExit("usage: python tests/golden/make_fixtures.py <reference checkout>")
    main(sys.argv[1])
