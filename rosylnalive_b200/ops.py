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
                ("splits", I32), ("out", U64), ("ldo", I32), ("resid", U64), ("ldr", I32), ("split_stride", U64)]


N.extra_signatures({
    "lrm_op_set_device": [I32],
    "lrm_op_error_word": [ctypes.POINTER(U32), I32],
    "lrm_op_gemm_bf16": [P, ctypes.POINTER(GemmDesc)],
})


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


def gemm(a, b, out, epilogue=GEMM_F32, resid=None, splits=1, bn=0, ldo=None, split_stride=0, stream=None):
    """out = epilogue(a @ b.T); a bf16 [m, k], b bf16 [n, k] (torch CUDA tensors)."""
    m, k = a.shape
    n, k2 = b.shape
    assert k == k2
    d = GemmDesc(m, n, k, a.data_ptr(), b.data_ptr(), epilogue, bn, splits, out.data_ptr(),
                 ldo if ldo is not None else (m if epilogue == GEMM_PARTIAL else out.shape[-1]),
                 resid.data_ptr() if resid is not None else 0, resid.shape[-1] if resid is not None else 0,
                 split_stride)
    N.check(N.lib().lrm_op_gemm_bf16(_stream(stream), ctypes.byref(d)), None, "gemm")
