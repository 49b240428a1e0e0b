"""Pins the parity oracle (oracle/) against the reference's goldens and known-answer vectors.

Sources of the expected values:
- goldens/tiny/g1 (torch32 / torch64p taps, greedy ids, T_spec), copied bit for bit into tests/golden/tiny_g1.npz
  by tests/golden/make_fixtures.py;
- the CpuReferenceSemantics contract vectors (docs/contracts/cpu-reference.md, "Vectors");
- the ReferenceOracles contract's inv_freq bits, T_spec entries and table digests
  (docs/contracts/reference-oracles.md, "Vectors");
- the tiny model's acceptance bounds (cpu-reference.md "Acceptance on the tiny model": 1e-12 F64 vs torch64p,
  1e-6 per op F32, chain floor 1e-5 F32).
"""

import hashlib
import json
import struct

import numpy as np
import pytest

from oracle import oracle as O
from rosylnalive_b200 import rope as R


def f32bits(x):
    return struct.unpack("<I", struct.pack("<f", x))[0]


def bits_f32(b):
    return struct.unpack("<f", struct.pack("<I", b))[0]


def rel_l2(a, ref):
    a = np.asarray(a, np.float64)
    ref = np.asarray(ref, np.float64)
    return float(np.linalg.norm(a - ref) / max(np.linalg.norm(ref), 1e-300))


def tiny_model(z, mode_table=None):
    cfg = json.loads(bytes(z["config_json"]).decode())
    c = O.Config(cfg["num_hidden_layers"], cfg["hidden_size"], cfg["num_attention_heads"],
                 cfg["num_key_value_heads"], cfg["head_dim"], cfg["intermediate_size"], cfg["vocab_size"],
                 cfg["rms_norm_eps"], cfg["max_position_embeddings"])
    cos, sin = O.rope_table(z["rope/inv_freq.bits"], c.max_pos)
    w = {k[2:]: z[k] for k in z.files if k.startswith("w/")}
    return O.Model.from_hf(c, w, cos, sin)


# ---- CpuReferenceSemantics vectors ---------------------------------------------------------------------------


def test_fused_dot_step():
    x = np.array([1.0, 1.0 + 2.0 ** -12], np.float32)
    y = np.array([-1.0, 1.0 + 2.0 ** -12], np.float32)
    assert f32bits(O.dot(x, y, "f32")) == 0x3A000400


def test_index_order():
    assert O.dot(np.array([1, 1e8, -1e8], np.float32), np.ones(3, np.float32), "f32") == 0.0


def test_rmsnorm_vector():
    w = O.narrow_rne(np.array([1.0, 2.0], np.float32))
    y = O.rmsnorm(np.array([[3.0, 4.0]], np.float32), w, 0.0, "f32")
    assert [f32bits(v) for v in y[0]] == [0x3F593924, 0x4010D0C3]
    y0 = O.rmsnorm(np.array([[3.0, 4.0]], np.float32), np.zeros(2, np.uint16), 0.0, "f32")
    assert np.all(y0 == 0)


def test_attention_vector():
    q = np.array([[1.0, 0.0]])
    k = np.array([[0.0, 5.0], [np.log(3.0), 7.0]])
    v = np.array([[4.0, 8.0], [0.0, 4.0]])
    y = O.attention(q, k, v, 1, 1, 2, past=1, scale=1.0, mode="f64")
    assert np.allclose(y[0], [1.0, 5.0], atol=1e-15)


def test_attention_scale():
    assert O.attention_scale(32, "f64") == 0.1767766952966369
    assert f32bits(O.attention_scale(128, "f32")) == 0x3DB504F3


def test_embed_gather_out_of_range_is_qnan_row():
    table = O.narrow_rne(np.arange(8, dtype=np.float32).reshape(4, 2))
    y = O.embed_gather(table, np.array([1, 7], np.uint32), "f32")
    assert np.all(y[1].view(np.uint32) == 0x7FC00000)
    y64 = O.embed_gather(table, np.array([9], np.uint32), "f64")
    assert np.all(y64.view(np.uint64) == 0x7FF8000000000000)
    assert np.array_equal(y[0], [2.0, 3.0])


def test_argmax_vectors():
    assert O.argmax_rows(np.array([[1, 3, 3]], np.float32))[0] == 1
    assert O.argmax_rows(np.array([[-0.0, 0.0]], np.float32))[0] == 0
    assert O.argmax_rows(np.array([[1.0, np.nan, 2.0]], np.float32))[0] == 0xFFFFFFFF


# ---- RoPE: T_spec without libm guesses -----------------------------------------------------------------------

TINY_INV = [0x3F800000, 0x3ED7E89B, 0x3E361887, 0x3D99940D, 0x3D0186E3, 0x3C5A7BF2, 0x3BB8449C, 0x3B1B690D,
            0x3A83126F, 0x39DD1725, 0x393A7753, 0x389D43A4, 0x3804A2B2, 0x375FBA4F, 0x36BCB0C1, 0x361F23E4]


def test_inv_freq_bits_pinned(tiny_golden):
    assert list(tiny_golden["rope/inv_freq.bits"]) == TINY_INV
    tiny = np.array(TINY_INV, np.uint32)
    assert hashlib.sha256(tiny.tobytes()).hexdigest() == \
        "7f7aa6f39d2fd0a08c069fbf6d7cf6679288240227d78c053382b884db09abee"
    qwen = R.QWEN3_INV_FREQ_BITS
    assert [int(b) for b in qwen[:8]] == [0x3F800000, 0x3F4E4BAD, 0x3F263DE0, 0x3F05F6EF, 0x3ED7E89B, 0x3EADFCFF,
                                          0x3E8C3504, 0x3E61F835]
    assert [int(b) for b in qwen[-4:]] == [0x361F23E4, 0x36003DEC, 0x35CEAF79, 0x35A68E4C]
    assert hashlib.sha256(qwen.tobytes()).hexdigest() == \
        "138c99b109d7affbfba059e435670918fe4531bce4709b6e86f3f22f7ef80f6e"


def test_tiny_t_spec_equals_golden(tiny_golden):
    cos, sin = O.rope_table(tiny_golden["rope/inv_freq.bits"], 512)
    assert np.array_equal(cos.view(np.uint32), tiny_golden["rope/t_spec.cos"].view(np.uint32))
    assert np.array_equal(sin.view(np.uint32), tiny_golden["rope/t_spec.sin"].view(np.uint32))
    assert hashlib.sha256(cos.tobytes() + sin.tobytes()).hexdigest() == \
        "615b420404dd336bbf4509e20dd121daefdcc0cd8039048ca71097b1b6d60801"


def test_qwen_t_spec_digest_and_entries():
    cos, sin = O.rope_table(R.QWEN3_INV_FREQ_BITS, 8192)
    assert hashlib.sha256(cos.tobytes() + sin.tobytes()).hexdigest() == \
        "da820d286cb666557f4cae3fa7f806c07d941653769e10c09021555a8f6ebfaf"
    c, s = cos.view(np.uint32), sin.view(np.uint32)
    assert (c[4095, 0], s[4095, 0]) == (0xBD871E6C, 0xBF7F7136)
    assert (c[4095, 63], s[4095, 63]) == (0x3F7FFF27, 0x3BA683B4)
    assert (c[8191, 1], s[8191, 1]) == (0xBF7C693C, 0xBE2ADD27)


def test_tiny_t_spec_entries():
    cos, sin = O.rope_table(np.array(TINY_INV, np.uint32), 512)
    c, s = cos.view(np.uint32), sin.view(np.uint32)
    for pos, j, cb, sb in [(0, 0, 0x3F800000, 0), (1, 0, 0x3F0A5140, 0x3F576AA4), (1, 15, 0x3F800000, 0x361F23E4),
                           (13, 3, 0x3F0FB02C, 0x3F53DF36), (100, 7, 0x3F78D5F0, 0x3E708F27),
                           (511, 0, 0xBEF17FE5, 0x3F61BBB4), (511, 15, 0x3F7FFFF4, 0x3A9ED44F)]:
        assert (c[pos, j], s[pos, j]) == (cb, sb)


def test_exact_cos_sin_of_one():
    import ctypes
    cc, ss = ctypes.c_double(), ctypes.c_double()
    assert O.lib().oracle_cos_sin(1.0, ctypes.byref(cc), ctypes.byref(ss)) == 0
    assert struct.unpack("<Q", struct.pack("<d", cc.value))[0] == 0x3FE14A280FB5068C
    assert struct.unpack("<Q", struct.pack("<d", ss.value))[0] == 0x3FEAED548F090CEE


# ---- the tiny model against torch32 and torch64p ---------------------------------------------------------------


@pytest.mark.parametrize("prompt", ["p0", "p1"])
def test_tiny_taps_f64_vs_torch64p(tiny_golden, prompt):
    m = tiny_model(tiny_golden)
    taps = {}
    O.forward(m, O.Cache.new(m.config, "f64"), 0, tiny_golden[f"prompt/{prompt}"], "f64", taps)
    assert len(taps) == 39
    for k, v in taps.items():
        assert rel_l2(v, tiny_golden[f"torch64p/{prompt}/{k}"]) <= 1e-12, k


@pytest.mark.parametrize("prompt", ["p0", "p1"])
def test_tiny_taps_f32_vs_torch32(tiny_golden, prompt):
    m = tiny_model(tiny_golden)
    taps = {}
    O.forward(m, O.Cache.new(m.config, "f32"), 0, tiny_golden[f"prompt/{prompt}"], "f32", taps)
    for k, v in taps.items():
        assert rel_l2(v, tiny_golden[f"torch32/{prompt}/{k}"]) <= 1e-5, k
    lg = taps["logits"].astype(np.float64)
    assert np.max(np.abs(lg - tiny_golden[f"torch32/{prompt}/logits"])) <= 2e-3


def test_tiny_p2_logits_crossing_a_64_key_block(tiny_golden):
    m = tiny_model(tiny_golden)
    for mode, tag, bound in (("f64", "torch64p", 1e-12), ("f32", "torch32", 1e-5)):
        lg = O.forward(m, O.Cache.new(m.config, mode), 0, tiny_golden["prompt/p2"], mode)
        assert rel_l2(lg, tiny_golden[f"{tag}/p2/logits"]) <= bound


@pytest.mark.parametrize("prompt", ["p0", "p1"])
@pytest.mark.parametrize("mode,tag", [("f32", "torch32"), ("f64", "torch64p")])
def test_tiny_64_greedy_steps(tiny_golden, prompt, mode, tag):
    m = tiny_model(tiny_golden)
    ids = O.greedy(m, tiny_golden[f"prompt/{prompt}"], 64, mode)
    assert np.array_equal(ids, tiny_golden[f"greedy/{prompt}.ids.{tag}"])


def test_prefill_equals_token_by_token_decode(tiny_golden):
    m = tiny_model(tiny_golden)
    prompt = tiny_golden["prompt/p0"]
    c1 = O.Cache.new(m.config, "f32")
    full = O.forward(m, c1, 0, prompt, "f32")
    c2 = O.Cache.new(m.config, "f32")
    rows = [O.forward(m, c2, i, [t], "f32") for i, t in enumerate(prompt)]
    assert np.array_equal(np.concatenate(rows).view(np.uint32), full.view(np.uint32))
    for a, b in zip(c1.keys + c1.values, c2.keys + c2.values):
        assert np.array_equal(a.view(np.uint32), b.view(np.uint32))


def test_thread_count_invariance(tiny_golden):
    m = tiny_model(tiny_golden)
    prompt = tiny_golden["prompt/p2"]
    a = O.forward(m, O.Cache.new(m.config, "f32"), 0, prompt, "f32", threads=1)
    b = O.forward(m, O.Cache.new(m.config, "f32"), 0, prompt, "f32", threads=7)
    assert np.array_equal(a.view(np.uint32), b.view(np.uint32))
