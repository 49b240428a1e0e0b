"""RoPE inputs for the CUDA device: pinned inverse frequencies and the T_spec table.

The table T_spec (reference: src/Lrm.Tensor.CpuReference/Rope.fs:163-251, RopeTable.create) is, for pos < max_pos and
j < head_dim/2: freq = f32(f32(pos) * inv_freq[j]); cos = f32(RN64(cos freq)); sin = f32(RN64(sin freq)), with RN64 the
correctly rounded float64. It is built on the host by liblrmcuda (``lrm_rope_table``), which certifies every rounding
and raises when it cannot, and uploaded to the device's Rope arena like any other read-only tensor.
"""

from __future__ import annotations

import numpy as np

# torch's own fp32 inv_freq for theta 1e6, head_dim 128 (Qwen3-0.6B): 1 / (theta ** (arange(0, 128, 2) / 128)) in
# float32, as HF transformers' compute_default_rope_parameters gives it. Pinned as bits, because no closed-form
# float64 formula rounded to float32 reproduces all 64 entries (reference: docs/contracts/reference-oracles.md,
# "T_spec" item 1; SHA-256 138c99b1... checked in the tests).
QWEN3_INV_FREQ_BITS = np.array([
    0x3F800000, 0x3F4E4BAD, 0x3F263DE0, 0x3F05F6EF, 0x3ED7E89B, 0x3EADFCFF, 0x3E8C3504, 0x3E61F835, 0x3E361887,
    0x3E12BD91, 0x3DEC7FD6, 0x3DBE94C6, 0x3D99940D, 0x3D778513, 0x3D47763F, 0x3D20BC1D, 0x3D0186E3, 0x3CD0C1A8,
    0x3CA8398B, 0x3C879008, 0x3C5A7BF2, 0x3C301052, 0x3C0DE12D, 0x3BE4AA46, 0x3BB8449C, 0x3B947DAE, 0x3B6F520E,
    0x3B40DAC5, 0x3B1B690D, 0x3AFA78F0, 0x3AC9D75C, 0x3AA2A6F7, 0x3A83126F, 0x3A533F28, 0x3A2A3B44, 0x3A092E02,
    0x39DD1725, 0x39B229FB, 0x398F9272, 0x39676492, 0x393A7753, 0x39164324, 0x38F22CE2, 0x38C327B5, 0x389D43A4,
    0x387D75D4, 0x384C3FBE, 0x382497AB, 0x3804A2B2, 0x37D5C441, 0x37AC431D, 0x378AD0ED, 0x375FBA4F, 0x37344A0E,
    0x371148E3, 0x36EA2732, 0x36BCB0C1, 0x36980E02, 0x36751070, 0x36457BAB, 0x361F23E4, 0x36003DEC, 0x35CEAF79,
    0x35A68E4C], dtype=np.uint32)


def torch_inv_freq_bits(theta: float, head_dim: int) -> np.ndarray:
    """torch's float32 inv_freq for (theta, head_dim) as u32 bits: the computation of HF transformers'
    compute_default_rope_parameters, run in torch on the CPU (the same bits on every x86 host)."""
    import torch

    exps = torch.arange(0, head_dim, 2, dtype=torch.int64).to(dtype=torch.float) / head_dim
    inv = 1.0 / (theta ** exps)
    return inv.numpy().astype(np.float32).view(np.uint32).copy()


def t_spec(inv_freq_bits: np.ndarray, max_pos: int) -> tuple[np.ndarray, np.ndarray]:
    """T_spec (cos, sin), float32 [max_pos, head_dim/2], built by liblrmcuda's certified host routine."""
    from . import native

    return native.rope_table(np.ascontiguousarray(inv_freq_bits, np.uint32), max_pos)
