"""Parity oracle: ctypes wrapper over oracle/_build/liblrm_oracle.so plus the Qwen3 forward composition.

TEST INFRASTRUCTURE ONLY. This module is the checker the CUDA path is compared against. Only tests/,
``__graft_entry__.smoke()`` and bench.py's CPU-baseline leg import it; the product package never does.

Parity is pinned against the reference's committed goldens (goldens/tiny/g1) by tests/test_oracle_golden.py.

The composition follows the reference's only Qwen3 forward, tests/Lrm.Tensor.Tests/TinyModel.fs:144-204 (one
forward over ids at positions pos0..pos0+T-1, K after norm+RoPE and raw V written into the cache), and its greedy
schedule TinyModel.fs:219-236 (one prefill, then single-token steps, argmax of the last row).
"""

from __future__ import annotations

import ctypes
import os
import subprocess
from dataclasses import dataclass, field

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "_build", "liblrm_oracle.so")
_lib = None


def build() -> str:
    """Compiles the oracle library (make in oracle/) and returns its path."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        _lib = ctypes.CDLL(_LIB_PATH)
        _declare(_lib)
    return _lib


_f32p = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
_f64p = np.ctypeslib.ndpointer(np.float64, flags="C_CONTIGUOUS")
_u16p = np.ctypeslib.ndpointer(np.uint16, flags="C_CONTIGUOUS")
_u32p = np.ctypeslib.ndpointer(np.uint32, flags="C_CONTIGUOUS")
_L = ctypes.c_long
_I = ctypes.c_int


def _declare(L: ctypes.CDLL) -> None:
    L.oracle_rope_table.argtypes = [_u32p, _I, _I, _f32p, _f32p]
    L.oracle_rope_table.restype = _I
    L.oracle_cos_sin.argtypes = [ctypes.c_float, ctypes.POINTER(ctypes.c_double), ctypes.POINTER(ctypes.c_double)]
    L.oracle_cos_sin.restype = _I
    L.oracle_bf16_narrow_array.argtypes = [_f32p, _u16p, _L]
    for suf, T, tp in (("f32", ctypes.c_float, _f32p), ("f64", ctypes.c_double, _f64p)):
        getattr(L, f"oracle_dot_{suf}").argtypes = [tp, tp, _L]
        getattr(L, f"oracle_dot_{suf}").restype = T
        getattr(L, f"oracle_embed_gather_{suf}").argtypes = [_u16p, _L, _L, _u32p, _L, tp]
        getattr(L, f"oracle_rmsnorm_{suf}").argtypes = [tp, _L, _L, _u16p, T, tp, _I]
        getattr(L, f"oracle_matmul_bf16w_{suf}").argtypes = [tp, _L, _L, _u16p, _L, tp, _I]
        getattr(L, f"oracle_rope_apply_{suf}").argtypes = [tp, _L, _L, _L, _f32p, _f32p, _L, tp]
        getattr(L, f"oracle_attention_{suf}").argtypes = [tp, _L, tp, tp, _L, _L, _L, _L, T, tp, _I]
        getattr(L, f"oracle_silu_mul_{suf}").argtypes = [tp, tp, _L, tp]
        getattr(L, f"oracle_add_{suf}").argtypes = [tp, tp, _L, tp]
        getattr(L, f"oracle_argmax_rows_{suf}").argtypes = [tp, _L, _L, _u32p]
        getattr(L, f"oracle_logsumexp_{suf}").argtypes = [tp, _L]
        getattr(L, f"oracle_logsumexp_{suf}").restype = T
        getattr(L, f"oracle_attention_scale_{suf}").argtypes = [_L]
        getattr(L, f"oracle_attention_scale_{suf}").restype = T


def _dt(mode: str):
    if mode == "f32":
        return np.float32
    if mode == "f64":
        return np.float64
    raise ValueError(f"the oracle computes in f32 or f64, not {mode}")


def _c(a, dtype):
    return np.ascontiguousarray(a, dtype=dtype)


THREADS = os.cpu_count() or 1

# ---------------------------------------------------------------------------------------------------------------
# Ops (CpuRef.fs). `mode` is "f32" (CpuRef F32) or "f64" (CpuRef F64).


def widen(bits: np.ndarray) -> np.ndarray:
    """Exact bf16 widening (Lrm.Core Numerics.fs:24-29): the bits become the top half of a float32."""
    return (np.asarray(bits, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def narrow_rne(x: np.ndarray) -> np.ndarray:
    """float32 -> bf16 bits, round to nearest even (Lrm.Core Numerics.fs:34-45)."""
    x = _c(x, np.float32)
    y = np.empty(x.shape, np.uint16)
    lib().oracle_bf16_narrow_array(x.reshape(-1), y.reshape(-1), x.size)
    return y


def dot(x, y, mode="f32"):
    t = _dt(mode)
    return getattr(lib(), f"oracle_dot_{mode}")(_c(x, t), _c(y, t), len(x))


def embed_gather(table, ids, mode="f32"):
    table = _c(table, np.uint16)
    ids = _c(ids, np.uint32)
    y = np.empty((len(ids), table.shape[1]), _dt(mode))
    getattr(lib(), f"oracle_embed_gather_{mode}")(table, table.shape[0], table.shape[1], ids, len(ids), y)
    return y


def rmsnorm(x, w, eps, mode="f32", threads=THREADS):
    t = _dt(mode)
    x = _c(x, t)
    w = _c(w, np.uint16)
    cols = w.size
    assert x.size % cols == 0
    y = np.empty_like(x)
    getattr(lib(), f"oracle_rmsnorm_{mode}")(x, x.size // cols, cols, w, t(eps), y, threads)
    return y


def matmul_bf16w(x, w, mode="f32", threads=THREADS):
    t = _dt(mode)
    x = _c(x, t)
    w = _c(w, np.uint16)
    m, k = x.shape
    n, k2 = w.shape
    assert k == k2
    y = np.empty((m, n), t)
    getattr(lib(), f"oracle_matmul_bf16w_{mode}")(x, m, k, w, n, y, threads)
    return y


def rope_table(inv_freq_bits, max_pos):
    """T_spec (Rope.fs:167-251): returns (cos, sin), float32 [max_pos, half]."""
    bits = _c(inv_freq_bits, np.uint32)
    half = bits.size
    cos = np.empty((max_pos, half), np.float32)
    sin = np.empty((max_pos, half), np.float32)
    if lib().oracle_rope_table(bits, half, max_pos, cos, sin) != 0:
        raise ArithmeticError("a T_spec entry's float64 rounding could not be certified")
    return cos, sin


def rope_apply(x, cos, sin, heads, pos0, mode="f32"):
    t = _dt(mode)
    x = _c(x, t)
    hd = 2 * cos.shape[1]
    rows = x.shape[0]
    assert x.shape[1] == heads * hd
    if pos0 < 0 or pos0 + rows > cos.shape[0]:
        raise IndexError(f"positions {pos0}..{pos0 + rows - 1} outside the table (max_pos {cos.shape[0]})")
    y = np.empty_like(x)
    getattr(lib(), f"oracle_rope_apply_{mode}")(x, rows, heads, hd, _c(cos, np.float32), _c(sin, np.float32), pos0, y)
    return y


def attention(q, kcache, vcache, q_heads, kv_heads, head_dim, past, scale=None, mode="f32", threads=THREADS):
    t = _dt(mode)
    q = _c(q, t)
    kcache = _c(kcache, t)
    vcache = _c(vcache, t)
    rows = q.shape[0]
    if scale is None:
        scale = attention_scale(head_dim, mode)
    if past + rows > kcache.shape[0]:
        raise IndexError("positions need more cache rows")
    y = np.empty((rows, q_heads * head_dim), t)
    getattr(lib(), f"oracle_attention_{mode}")(q, rows, kcache, vcache, q_heads, kv_heads, head_dim, past, t(scale),
                                               y, threads)
    return y


def attention_scale(head_dim, mode="f32"):
    return getattr(lib(), f"oracle_attention_scale_{mode}")(head_dim)


def silu_mul(g, u, mode="f32"):
    t = _dt(mode)
    g = _c(g, t)
    u = _c(u, t)
    y = np.empty_like(g)
    getattr(lib(), f"oracle_silu_mul_{mode}")(g, u, g.size, y)
    return y


def add(a, b, mode="f32"):
    t = _dt(mode)
    a = _c(a, t)
    b = _c(b, t)
    y = np.empty_like(a)
    getattr(lib(), f"oracle_add_{mode}")(a, b, a.size, y)
    return y


def argmax_rows(x, mode="f32"):
    t = _dt(mode)
    x = _c(x, t)
    if x.ndim != 2:
        raise ValueError("a row op needs [rows, cols]")
    y = np.empty(x.shape[0], np.uint32)
    getattr(lib(), f"oracle_argmax_rows_{mode}")(x, x.shape[0], x.shape[1], y)
    return y


def logsumexp(x, mode="f64"):
    t = _dt(mode)
    x = _c(x, t)
    return getattr(lib(), f"oracle_logsumexp_{mode}")(x, x.size)


# ---------------------------------------------------------------------------------------------------------------
# The model (TinyModel.fs:14-140).


@dataclass
class Config:
    layers: int
    hidden: int
    heads: int
    kv_heads: int
    head_dim: int
    intermediate: int
    vocab: int
    eps: float
    max_pos: int


LAYER_KEYS = ("input_layernorm", "q_proj", "k_proj", "v_proj", "o_proj", "q_norm", "k_norm",
              "post_attention_layernorm", "gate_proj", "up_proj", "down_proj")

# HF weight names (TinyModel.fs:79-101).
HF_NAMES = {
    "input_layernorm": "input_layernorm.weight",
    "q_proj": "self_attn.q_proj.weight",
    "k_proj": "self_attn.k_proj.weight",
    "v_proj": "self_attn.v_proj.weight",
    "o_proj": "self_attn.o_proj.weight",
    "q_norm": "self_attn.q_norm.weight",
    "k_norm": "self_attn.k_norm.weight",
    "post_attention_layernorm": "post_attention_layernorm.weight",
    "gate_proj": "mlp.gate_proj.weight",
    "up_proj": "mlp.up_proj.weight",
    "down_proj": "mlp.down_proj.weight",
}


@dataclass
class Model:
    config: Config
    embed: np.ndarray  # bf16 bits [vocab, hidden]
    layers: list  # list of dict key -> bf16 bits
    norm: np.ndarray  # bf16 bits [hidden]
    rope_cos: np.ndarray  # f32 [max_pos, head_dim/2]
    rope_sin: np.ndarray

    @staticmethod
    def from_hf(config: Config, tensors: dict, rope_cos, rope_sin) -> "Model":
        layers = []
        for i in range(config.layers):
            layers.append({k: np.ascontiguousarray(tensors[f"model.layers.{i}.{HF_NAMES[k]}"], np.uint16)
                           for k in LAYER_KEYS})
        return Model(config, np.ascontiguousarray(tensors["model.embed_tokens.weight"], np.uint16), layers,
                     np.ascontiguousarray(tensors["model.norm.weight"], np.uint16), rope_cos, rope_sin)


@dataclass
class Cache:
    """K (after norm and RoPE) and V (raw) per layer, [max_pos, kv_heads*head_dim] in the mode's dtype."""
    keys: list
    values: list

    @staticmethod
    def new(config: Config, mode: str, max_pos: int | None = None) -> "Cache":
        t = _dt(mode)
        rows = max_pos or config.max_pos
        shape = (rows, config.kv_heads * config.head_dim)
        return Cache([np.zeros(shape, t) for _ in range(config.layers)],
                     [np.zeros(shape, t) for _ in range(config.layers)])


def forward(m: Model, cache: Cache, pos0: int, ids, mode="f32", taps: dict | None = None, logits_rows="all",
            threads=THREADS):
    """One forward (TinyModel.fs:144-204). Returns logits [T, vocab] (or [1, vocab] for logits_rows="last")."""
    c = m.config
    eps = c.eps
    scale = attention_scale(c.head_dim, mode)
    ids = np.asarray(ids, dtype=np.uint32)
    T = len(ids)
    if np.any(ids >= c.vocab):
        raise IndexError("an id is outside the vocabulary")

    def tap(name, t):
        if taps is not None:
            taps[name] = t
        return t

    x = tap("embed.out", embed_gather(m.embed, ids, mode))
    for i in range(c.layers):
        lw = m.layers[i]
        p = f"L{i}."
        h = tap(p + "input_layernorm.out", rmsnorm(x, lw["input_layernorm"], eps, mode, threads))
        q = tap(p + "attn.q_proj.out", matmul_bf16w(h, lw["q_proj"], mode, threads))
        k = tap(p + "attn.k_proj.out", matmul_bf16w(h, lw["k_proj"], mode, threads))
        v = tap(p + "attn.v_proj.out", matmul_bf16w(h, lw["v_proj"], mode, threads))
        qn = tap(p + "attn.q_norm.out", rmsnorm(q, lw["q_norm"], eps, mode, threads))
        kn = tap(p + "attn.k_norm.out", rmsnorm(k, lw["k_norm"], eps, mode, threads))
        qr = tap(p + "attn.q_rope", rope_apply(qn, m.rope_cos, m.rope_sin, c.heads, pos0, mode))
        kr = tap(p + "attn.k_rope", rope_apply(kn, m.rope_cos, m.rope_sin, c.kv_heads, pos0, mode))
        cache.keys[i][pos0:pos0 + T] = kr
        cache.values[i][pos0:pos0 + T] = v
        tap(p + "attn.v_cache", cache.values[i][pos0:pos0 + T].copy())
        o = tap(p + "attn.o_proj.in", attention(qr, cache.keys[i], cache.values[i], c.heads, c.kv_heads, c.head_dim,
                                                 pos0, scale, mode, threads))
        oo = tap(p + "attn.o_proj.out", matmul_bf16w(o, lw["o_proj"], mode, threads))
        r = tap(p + "resid_mid", add(x, oo, mode))
        h2 = tap(p + "post_attention_layernorm.out", rmsnorm(r, lw["post_attention_layernorm"], eps, mode, threads))
        g = tap(p + "mlp.gate.out", matmul_bf16w(h2, lw["gate_proj"], mode, threads))
        u = tap(p + "mlp.up.out", matmul_bf16w(h2, lw["up_proj"], mode, threads))
        d = tap(p + "mlp.down.in", silu_mul(g, u, mode))
        dd = tap(p + "mlp.down.out", matmul_bf16w(d, lw["down_proj"], mode, threads))
        x = tap(p + "out", add(r, dd, mode))
    f = tap("final_norm.out", rmsnorm(x, m.norm, eps, mode, threads))
    if logits_rows == "last":
        f = f[-1:]
    return tap("logits", matmul_bf16w(f, m.embed, mode, threads))


def greedy(m: Model, prompt, steps, mode="f32", threads=THREADS, return_logits=False):
    """The canonical greedy schedule (TinyModel.fs:219-236): prefill, then single-token decode steps."""
    cache = Cache.new(m.config, mode)
    logits = forward(m, cache, 0, prompt, mode, logits_rows="last", threads=threads)
    out_logits = [logits[-1].copy()]
    nxt = int(_argmax_checked(logits[-1:], mode)[0])
    ids = [nxt]
    for s in range(1, steps):
        logits = forward(m, cache, len(prompt) + s - 1, [nxt], mode, logits_rows="last", threads=threads)
        out_logits.append(logits[-1].copy())
        nxt = int(_argmax_checked(logits, mode)[0])
        ids.append(nxt)
    if return_logits:
        return np.array(ids, np.int64), np.stack(out_logits)
    return np.array(ids, np.int64)


def _argmax_checked(x, mode):
    r = argmax_rows(x, mode)
    if np.any(r == 0xFFFFFFFF):
        raise ValueError("argmax of a row that holds a NaN")
    return r
