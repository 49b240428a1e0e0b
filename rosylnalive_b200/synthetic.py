"""Seeded synthetic models and inputs for the BASELINE configs (no checkpoints or datasets are available or used).

Weights: i.i.d. N(0, 0.02) drawn in float32 and rounded to bf16 (round to nearest even), one independent stream per
tensor (numpy PCG64 seeded with [seed, crc32(name)]), so any tensor can be regenerated alone. RMSNorm gains
(input/post/final norms and the per-head q_norm/k_norm) are 1 + N(0, 0.02): the configs' "N(0, 0.02) weights" applied
to a gain that HF initialises at 1, so activations keep their scale through 28 layers. Prompts: ids uniform in
[0, vocab) from their own seeded stream.
"""

from __future__ import annotations

import zlib

import numpy as np

from .executor import QwenConfig, weight_shapes

# the tiny Qwen3-shaped model (2 layers, hidden 64, 4 q / 2 kv heads of 16, inter 128, vocab 256).
CONFIG1 = QwenConfig(layers=2, hidden=64, heads=4, kv_heads=2, head_dim=16, intermediate=128, vocab=256, eps=1e-6,
                     max_pos=64, rope_theta=1e6)

# Qwen3-0.6B architecture (configs 2-5): 28 layers, hidden 1024, 16 q / 8 kv heads of 128, inter 3072, vocab 151936.
QWEN3_0_6B = QwenConfig(layers=28, hidden=1024, heads=16, kv_heads=8, head_dim=128, intermediate=3072, vocab=151936,
                        eps=1e-6, max_pos=8192, rope_theta=1e6)


def bf16_rne(x: np.ndarray) -> np.ndarray:
    """float32 -> bf16 bits, round to nearest even (NaN to the canonical quiet NaN)."""
    u = np.ascontiguousarray(x, np.float32).view(np.uint32)
    r = ((u + np.uint32(0x7FFF) + ((u >> np.uint32(16)) & np.uint32(1))) >> np.uint32(16)).astype(np.uint16)
    nan = (u & np.uint32(0x7FFFFFFF)) > np.uint32(0x7F800000)
    if nan.any():
        r[nan] = np.where((u[nan] >> 31) != 0, 0xFFC0, 0x7FC0).astype(np.uint16)
    return r


def _stream(seed: int, name: str) -> np.random.Generator:
    return np.random.default_rng([seed, zlib.crc32(name.encode())])


def random_tensor(name: str, shape, seed: int = 0) -> np.ndarray:
    g = _stream(seed, name)
    x = g.standard_normal(shape, dtype=np.float32) * np.float32(0.02)
    if name.endswith("norm.weight"):
        x = x + np.float32(1.0)
    return bf16_rne(x)


CHUNK_ROWS_ELEMS = 1 << 23  # tensors above this many elements are drawn in row chunks, one stream per chunk


def _chunk(name, shape, seed, r0, r1):
    g = np.random.default_rng([seed, zlib.crc32(name.encode()), r0])
    x = g.standard_normal((r1 - r0,) + tuple(shape[1:]), dtype=np.float32) * np.float32(0.02)
    return bf16_rne(x)


def random_weights(cfg: QwenConfig, seed: int = 0, threads: int | None = None) -> dict:
    """Every weight of `cfg`, each from its own stream (large matrices from one stream per block of rows), drawn on a
    thread pool; the values do not depend on the thread count."""
    import concurrent.futures as cf
    import os

    shapes = weight_shapes(cfg)
    out = {}
    with cf.ThreadPoolExecutor(max_workers=threads or min(32, os.cpu_count() or 1)) as ex:
        futs = {}
        for name, shape in shapes.items():
            n = int(np.prod(shape))
            if n <= CHUNK_ROWS_ELEMS or len(shape) != 2:
                futs[name] = ex.submit(random_tensor, name, shape, seed)
            else:
                rows = max(1, CHUNK_ROWS_ELEMS // shape[1])
                futs[name] = [ex.submit(_chunk, name, shape, seed, r0, min(shape[0], r0 + rows))
                              for r0 in range(0, shape[0], rows)]
        for name, f in futs.items():
            out[name] = np.concatenate([c.result() for c in f]) if isinstance(f, list) else f.result()
    return out


def random_prompt(vocab: int, length: int, seed: int = 0, stream: str = "prompt") -> np.ndarray:
    return _stream(seed, stream).integers(0, vocab, length, dtype=np.int64).astype(np.uint32)


def random_prompts(vocab: int, batch: int, length: int, seed: int = 0) -> np.ndarray:
    return _stream(seed, "prompts").integers(0, vocab, (batch, length), dtype=np.int64).astype(np.uint32)
