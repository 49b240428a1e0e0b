"""ctypes binding of liblrmcuda.so (include/lrm_cuda.h). The product path has no fallback: if the library is
missing, every entry point raises ``NativeLibraryMissing`` naming the build command."""

from __future__ import annotations

import ctypes
import os

import numpy as np

from .gpu_core import GpuContractException

PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(PKG, "liblrmcuda.so")


class NativeLibraryMissing(RuntimeError):
    pass


class CudaDeviceError(RuntimeError):
    """A CUDA runtime/driver failure (LRM_ERR_CUDA): the analogue of the reference's D3D12DeviceLostException."""


class CudaTimeoutError(TimeoutError):
    """A wait ran past its limit (LRM_ERR_TIMEOUT); the device stays usable."""


LRM_OK, LRM_ERR_CONTRACT, LRM_ERR_CUDA, LRM_ERR_TIMEOUT, LRM_ERR_ARGUMENT, LRM_ERR_OUT_OF_MEMORY, LRM_ERR_STATE, \
    LRM_ERR_NO_DEVICE, LRM_ERR_FORMAT = range(9)


class SafetensorsFormatError(ValueError):
    """A file breaks the safetensors format (LRM_ERR_FORMAT): the reference's SafetensorsFormatException
    (src/Lrm.Tensor/Safetensors.fs:16). The message names the file."""

LRM_CUDA_DEBUG = 0x1
LRM_CUDA_TIME_DISPATCHES = 0x2


class DeviceInfoC(ctypes.Structure):
    _fields_ = [("index", ctypes.c_int32), ("name", ctypes.c_char * 256), ("vendor_id", ctypes.c_uint32),
                ("pci_device_id", ctypes.c_uint32), ("driver", ctypes.c_char * 64), ("memory_bytes", ctypes.c_int64),
                ("sm_count", ctypes.c_int32), ("cc_major", ctypes.c_int32), ("cc_minor", ctypes.c_int32),
                ("accepted", ctypes.c_int32), ("rejection", ctypes.c_char * 256)]


class CompletionC(ctypes.Structure):
    _fields_ = [("fence", ctypes.c_uint64), ("dispatches", ctypes.c_uint32), ("timer_count", ctypes.c_uint32)]


_lib = None

P = ctypes.c_void_p
I32, U32, U64, I64 = ctypes.c_int32, ctypes.c_uint32, ctypes.c_uint64, ctypes.c_int64
PU32, PU64, PI64, PI32 = (ctypes.POINTER(t) for t in (U32, U64, I64, I32))

# name -> argtypes (restype lrm_status = int32 unless listed in _RESTYPES)
SIGNATURES = {
    "lrm_cuda_abi_version": [],
    "lrm_cuda_last_error": [P, ctypes.c_char_p, ctypes.c_size_t],
    "lrm_cuda_device_count": [PI32],
    "lrm_cuda_device_info": [I32, ctypes.POINTER(DeviceInfoC)],
    "lrm_cuda_create": [I32, U32, ctypes.POINTER(P)],
    "lrm_cuda_destroy": [P],
    "lrm_cuda_create_heap": [P, I32, PU32, PU64],
    "lrm_cuda_load_kernels": [P, ctypes.c_char_p],
    "lrm_cuda_kernel_present": [P, U32, PI32],
    "lrm_cuda_begin": [P, ctypes.POINTER(P)],
    "lrm_cuda_submit": [P, PU64],
    "lrm_cuda_list_free": [P],
    "lrm_cuda_wait": [P, U64, U32, ctypes.POINTER(CompletionC)],
    "lrm_cuda_timer_result": [P, U64, U32, PU32, PI64, PI64],
    "lrm_cuda_write_table": [P, P, U64],
    "lrm_cuda_upload": [P, I32, U64, P, U64],
    "lrm_cuda_download": [P, I32, U64, P, U64],
    "lrm_cuda_dispatch": [P, U32, PU32],
    "lrm_cuda_barrier": [P],
    "lrm_cuda_copy": [P, I32, U64, I32, U64, U64],
    "lrm_cuda_timer_begin": [P, PU32],
    "lrm_cuda_timer_end": [P, U32],
    "lrm_cuda_denormal_probe": [P, PU32, PU32],
    "lrm_rope_table": [PU32, I32, I32, ctypes.POINTER(ctypes.c_float), ctypes.POINTER(ctypes.c_float)],
}
_RESTYPES = {"lrm_cuda_abi_version": I32, "lrm_cuda_last_error": ctypes.c_size_t}


def extra_signatures(sigs: dict, restypes: dict | None = None) -> None:
    """Other modules (the Qwen engine) register their entry points here before the library is loaded."""
    SIGNATURES.update(sigs)
    _RESTYPES.update(restypes or {})
    if _lib is not None:
        _declare(_lib)


def _declare(L):
    for name, args in SIGNATURES.items():
        fn = getattr(L, name)
        fn.argtypes = args
        fn.restype = _RESTYPES.get(name, I32)


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise NativeLibraryMissing(f"{LIB_PATH} is not built: run `python -m rosylnalive_b200.build`")
        _lib = ctypes.CDLL(LIB_PATH)
        _declare(_lib)
    return _lib


def last_error(dev=None) -> str:
    buf = ctypes.create_string_buffer(2048)
    lib().lrm_cuda_last_error(dev, buf, len(buf))
    return buf.value.decode(errors="replace")


def check(status: int, dev=None, what: str = "", format_error=None):
    if status == LRM_OK:
        return
    msg = last_error(dev)
    if what:
        msg = f"{what}: {msg}"
    if status in (LRM_ERR_CONTRACT, LRM_ERR_STATE):
        raise GpuContractException(msg)
    if status == LRM_ERR_TIMEOUT:
        raise CudaTimeoutError(msg)
    if status in (LRM_ERR_ARGUMENT,):
        raise ValueError(msg)
    if status == LRM_ERR_NO_DEVICE:
        raise LookupError(msg)
    if status == LRM_ERR_OUT_OF_MEMORY:
        raise MemoryError(msg)
    if status == LRM_ERR_FORMAT:
        raise (format_error or SafetensorsFormatError)(msg)
    raise CudaDeviceError(msg)


def ptr(a: np.ndarray):
    return ctypes.c_void_p(a.ctypes.data)


def rope_table(inv_freq_bits: np.ndarray, max_pos: int):
    bits = np.ascontiguousarray(inv_freq_bits, np.uint32)
    half = bits.size
    cos = np.empty((max_pos, half), np.float32)
    sin = np.empty((max_pos, half), np.float32)
    fp = ctypes.POINTER(ctypes.c_float)
    check(lib().lrm_rope_table(bits.ctypes.data_as(PU32), half, max_pos, cos.ctypes.data_as(fp),
                               sin.ctypes.data_as(fp)), None, "lrm_rope_table")
    return cos, sin
