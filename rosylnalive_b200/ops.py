"""Python access to liblrmcuda.so's fast-path operators (include/lrm_cuda.h, "fast-path operators").

Arguments are torch CUDA tensors (used only as device memory and streams); every call goes through the C ABI.
"""

from __future__ import annotations

import ctypes

from . import native as N

P, I32, U32, U64 = ctypes.c_void_p, ctypes.c_int32, ctypes.c_uint32, ctypes.c_uint64

GEMM_F32, GEMM_RESID, GEMM_SWIGLU, GEMM_PARTIAL, GEMM_BF16 = range(5)


class GemmDesc(ctypes.Structure):
    _fields_ = [("m", I32), ("n", I32), ("k", I32), ("a", U64), ("b", U64), ("epilogue", I32), ("bn", I32),
                ("splits", I32), ("out", U64), ("ldo", I32), ("resid", U64), ("ldr", I32), ("split_stride", U64),
                ("cta_pair", I32)]


class PrefillAttnDesc(ctypes.Structure):
    _fields_ = [("q", U64), ("k", U64), ("v", U64), ("out", U64), ("cu_seqlens", U64), ("nseq", I32),
                ("max_len", I32), ("q_heads", I32), ("kv_heads", I32), ("head_dim", I32), ("total_tokens", I32),
                ("scale", ctypes.c_float)]


class DecodeAttnDesc(ctypes.Structure):
    _fields_ = [("q", U64), ("pool", U64), ("page_table", U64), ("seq_len", U64), ("slots", U64), ("out", U64),
                ("workspace", U64), ("batch", I32), ("q_heads", I32), ("kv_heads", I32), ("head_dim", I32),
                ("pages_per_seq", I32), ("pages_per_split", I32), ("scale", ctypes.c_float)]


class DecodeGemmDesc(ctypes.Structure):
    _fields_ = [("m", I32), ("n", I32), ("k", I32), ("w", U64), ("b", U64), ("epilogue", I32), ("splits", I32),
                ("ss", U64), ("nss", I32), ("hidden", I32), ("ss_stride", U64), ("eps", ctypes.c_float),
                ("x", U64), ("gain", U64), ("u", U64), ("ss_out", U64), ("act", U64), ("ld_act", I32)]


DEC_SWIGLU, DEC_RESID = 1, 2

N.extra_signatures({
    "lrm_op_set_device": [I32],
    "lrm_op_error_word": [ctypes.POINTER(U32), I32],
    "lrm_op_gemm_bf16": [P, ctypes.POINTER(GemmDesc)],
    "lrm_op_prefill_attention": [P, ctypes.POINTER(PrefillAttnDesc)],
    "lrm_op_decode_attention_workspace": [I32, I32, I32, I32],
    "lrm_op_decode_attention": [P, ctypes.POINTER(DecodeAttnDesc)],
    "lrm_op_decode_attention_static": [P, ctypes.POINTER(DecodeAttnDesc)],
    "lrm_op_wait_probe": [P, U32, U32],
    "lrm_op_argmax_rows": [P, P, I32, I32, P],
    "lrm_op_decode_gemm": [P, ctypes.POINTER(DecodeGemmDesc)],
}, {"lrm_op_decode_attention_workspace": U64})

# Scratch built into liblrmcuda.so for lrm_op_decode_attention_static (LRM_DECODE_ATTN_STATIC_SCRATCH_BYTES).
DECODE_ATTN_STATIC_SCRATCH_BYTES = 16 << 20


def _stream(stream):
    import torch

    s = stream if stream is not None else torch.cuda.current_stream()
    return ctypes.c_void_p(s.cuda_stream)


def set_device(index: int):
    N.check(N.lib().lrm_op_set_device(index), None, "set_device")


def error_word(clear: bool = True) -> int:
    v = ctypes.c_uint32()
    N.check(N.lib().lrm_op_error_word(ctypes.byref(v), 1 if clear else 0), None, "error_word")
    return v.value


def argmax_rows(logits, out, stream=None):
    """out[r] (uint32 as int32 storage) = the lowest index of the maximum of logits[r] (fp32 [rows, vocab] on the
    device), or 0xFFFFFFFF for a row holding a NaN: the engine's greedy pick."""
    N.check(N.lib().lrm_op_argmax_rows(_stream(stream), ctypes.c_void_p(logits.data_ptr()), logits.shape[0],
                                       logits.shape[1], ctypes.c_void_p(out.data_ptr())), None, "argmax_rows")


def wait_probe(polls: int, code: int, stream=None):
    """Launches a kernel whose bounded wait cannot complete: after `polls` polls it records `code` in the error word
    and returns (the path every kernel takes when a wait runs out)."""
    N.check(N.lib().lrm_op_wait_probe(_stream(stream), polls, code), None, "wait_probe")


def gemm(a, b, out, epilogue=GEMM_F32, resid=None, splits=1, bn=0, ldo=None, split_stride=0, cta_pair=0,
         stream=None):
    """out = epilogue(a @ b.T); a bf16 [m, k], b bf16 [n, k] (torch CUDA tensors). cta_pair: 0 chooses, 1 one CTA
    per 128-row tile, 2 two-SM clusters sharing 256 x 256 tiles (bn 256)."""
    m, k = a.shape
    n, k2 = b.shape
    assert k == k2
    d = GemmDesc(m, n, k, a.data_ptr(), b.data_ptr(), epilogue, bn, splits, out.data_ptr(),
                 ldo if ldo is not None else (m if epilogue == GEMM_PARTIAL else out.shape[-1]),
                 resid.data_ptr() if resid is not None else 0, resid.shape[-1] if resid is not None else 0,
                 split_stride, cta_pair)
    N.check(N.lib().lrm_op_gemm_bf16(_stream(stream), ctypes.byref(d)), None, "gemm")


def decode_gemm_resid(w, b, x, gain=None, u=None, ss_out=None, splits=0, stream=None):
    """x [n, m] fp32 += b @ w.T (w bf16 [m, k], b bf16 [n, k]); with gain also u [n, m] = bf16(gain * x) and
    ss_out [m / 128, n] = the sums of x^2 over 128-column groups. K split over a cluster of `splits` CTAs."""
    m, k = w.shape
    n = b.shape[0]
    d = DecodeGemmDesc(m, n, k, w.data_ptr(), b.data_ptr(), DEC_RESID, splits, 0, 0, 0,
                       ss_out.shape[1] if ss_out is not None else 0, 0.0, x.data_ptr(),
                       gain.data_ptr() if gain is not None else 0, u.data_ptr() if u is not None else 0,
                       ss_out.data_ptr() if ss_out is not None else 0, 0, 0)
    N.check(N.lib().lrm_op_decode_gemm(_stream(stream), ctypes.byref(d)), None, "decode_gemm")


def decode_gemm_swiglu(w, b, ss, hidden, eps, act, splits=0, stream=None):
    """act [n, m / 2] bf16 = silu(r g) * (r u) of y = b @ w.T (gate and up rows of w interleaved in blocks of 64),
    r[t] = 1 / sqrt(sum_g ss[g, t] / hidden + eps)."""
    m, k = w.shape
    n = b.shape[0]
    d = DecodeGemmDesc(m, n, k, w.data_ptr(), b.data_ptr(), DEC_SWIGLU, splits, ss.data_ptr(), ss.shape[0], hidden,
                       ss.shape[1], eps, 0, 0, 0, 0, act.data_ptr(), act.shape[1])
    N.check(N.lib().lrm_op_decode_gemm(_stream(stream), ctypes.byref(d)), None, "decode_gemm")


def prefill_attention(q, k, v, out, cu_seqlens, max_len, scale, stream=None):
    """Causal GQA attention of packed sequences: q [T, qh, 128], k/v [T, kvh, 128], cu_seqlens int32 [nseq + 1]."""
    d = PrefillAttnDesc(q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(), cu_seqlens.data_ptr(),
                        cu_seqlens.numel() - 1, max_len, q.shape[1], k.shape[1], q.shape[2], q.shape[0], scale)
    N.check(N.lib().lrm_op_prefill_attention(_stream(stream), ctypes.byref(d)), None, "prefill_attention")


def decode_attention_workspace(batch, kv_heads, pages_per_seq, pages_per_split) -> int:
    return int(N.lib().lrm_op_decode_attention_workspace(batch, kv_heads, pages_per_seq, pages_per_split))


def decode_attention(q, pool, page_table, seq_len, slots, out, workspace, pages_per_split, scale, stream=None):
    """Paged decode attention: q [B, qh, 128], pool [pages, kvh, 2, 16, 128], page_table int32 [seqs, pages_per_seq],
    seq_len int32 [seqs], slots int32 [B]."""
    d = DecodeAttnDesc(q.data_ptr(), pool.data_ptr(), page_table.data_ptr(), seq_len.data_ptr(), slots.data_ptr(),
                       out.data_ptr(), workspace.data_ptr(), q.shape[0], q.shape[1], pool.shape[1], q.shape[2],
                       page_table.shape[1], pages_per_split, scale)
    N.check(N.lib().lrm_op_decode_attention(_stream(stream), ctypes.byref(d)), None, "decode_attention")


def decode_attention_static(q, pool, page_table, seq_len, slots, out, pages_per_split, scale, stream=None):
    """decode_attention for callers that cannot allocate device memory: the split scratch is the 16 MiB array built
    into liblrmcuda.so (DECODE_ATTN_STATIC_SCRATCH_BYTES); the caller passes only inputs and the output. Calls that
    overlap on the GPU share that array and race; the first call on a device should come before any stream capture."""
    d = DecodeAttnDesc(q.data_ptr(), pool.data_ptr(), page_table.data_ptr(), seq_len.data_ptr(), slots.data_ptr(),
                       out.data_ptr(), 0, q.shape[0], q.shape[1], pool.shape[1], q.shape[2], page_table.shape[1],
                       pages_per_split, scale)
    N.check(N.lib().lrm_op_decode_attention_static(_stream(stream), ctypes.byref(d)), None,
            "decode_attention_static")
