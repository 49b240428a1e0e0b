"""liblrmcuda.so without a GPU: it loads, exports every function include/*.h declares, and its host-only helpers
(the certified T_spec builder) match the reference's pinned digests. No kernel is launched here."""

import hashlib
import os
import re
import subprocess
import sys

import numpy as np
import pytest

from rosylnalive_b200 import native as N
from rosylnalive_b200 import rope as R

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_functions():
    names = set()
    inc = os.path.join(ROOT, "include")
    for f in os.listdir(inc):
        if not f.endswith(".h"):
            continue
        text = open(os.path.join(inc, f)).read()
        text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
        for m in re.finditer(r"^\s*(?:lrm_status|int32_t|size_t|void|uint32_t|int)\s+\*?\s*(lrm_\w+)\s*\(", text,
                             flags=re.M):
            names.add(m.group(1))
    return names


def test_header_declares_the_boundary():
    names = declared_functions()
    for required in ("lrm_cuda_create", "lrm_cuda_create_heap", "lrm_cuda_write_table", "lrm_cuda_upload",
                     "lrm_cuda_download", "lrm_cuda_begin", "lrm_cuda_dispatch", "lrm_cuda_barrier", "lrm_cuda_copy",
                     "lrm_cuda_timer_begin", "lrm_cuda_timer_end", "lrm_cuda_submit", "lrm_cuda_wait",
                     "lrm_cuda_last_error", "lrm_cuda_destroy"):
        assert required in names


def test_library_exports_every_declared_symbol():
    out = subprocess.run(["nm", "-D", "--defined-only", N.LIB_PATH], capture_output=True, text=True, check=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if line.strip()}
    missing = declared_functions() - exported
    assert not missing, f"declared but not exported: {sorted(missing)}"


def test_library_loads_and_reports_abi():
    assert N.lib().lrm_cuda_abi_version() == 1
    for name in N.SIGNATURES:
        assert hasattr(N.lib(), name)


def test_product_t_spec_equals_pinned_tables(tiny_golden):
    cos, sin = N.rope_table(tiny_golden["rope/inv_freq.bits"], 512)
    assert np.array_equal(cos.view(np.uint32), tiny_golden["rope/t_spec.cos"].view(np.uint32))
    assert np.array_equal(sin.view(np.uint32), tiny_golden["rope/t_spec.sin"].view(np.uint32))
    cos, sin = N.rope_table(R.QWEN3_INV_FREQ_BITS, 8192)
    assert hashlib.sha256(cos.tobytes() + sin.tobytes()).hexdigest() == \
        "da820d286cb666557f4cae3fa7f806c07d941653769e10c09021555a8f6ebfaf"


def test_torch_inv_freq_matches_pins(tiny_golden):
    assert np.array_equal(R.torch_inv_freq_bits(1e6, 128), R.QWEN3_INV_FREQ_BITS)
    assert np.array_equal(R.torch_inv_freq_bits(1e6, 32), tiny_golden["rope/inv_freq.bits"])


def test_rope_table_rejects_bad_arguments():
    with pytest.raises(ValueError):
        N.rope_table(np.array([0x7F800000], np.uint32), 4)  # inf


def test_device_info_layout_matches_the_raw_binding():
    # The F# binding passes lrm_device_info as 616 raw bytes and decodes fields at these offsets.
    import ctypes

    C = N.DeviceInfoC
    assert ctypes.sizeof(C) == 616
    want = {"index": 0, "name": 4, "vendor_id": 260, "pci_device_id": 264, "driver": 268, "memory_bytes": 336,
            "sm_count": 344, "cc_major": 348, "cc_minor": 352, "accepted": 356, "rejection": 360}
    assert {k: getattr(C, k).offset for k in want} == want


def test_operators_refuse_sizes_past_their_int32_bound():
    # Each check returns before any CUDA call, so this runs without a GPU; the pointers are never dereferenced.
    import ctypes

    from rosylnalive_b200 import ops as O

    fake = ctypes.c_void_p(0x10000)
    big = (1 << 30) + 1
    assert N.lib().lrm_op_argmax_rows(None, fake, 1, big, fake) == N.LRM_ERR_ARGUMENT
    assert N.lib().lrm_op_argmax_rows(None, fake, 1, 0, fake) == N.LRM_ERR_ARGUMENT
    d = O.DecodeGemmDesc(m=128, n=64, k=big, w=0x10000, b=0x10000, epilogue=O.DEC_RESID)
    assert N.lib().lrm_op_decode_gemm(None, ctypes.byref(d)) == N.LRM_ERR_ARGUMENT
    d.k, d.m = 1024, big
    assert N.lib().lrm_op_decode_gemm(None, ctypes.byref(d)) == N.LRM_ERR_ARGUMENT
    g = O.GemmDesc(m=128, n=128, k=(1 << 31) - 1, a=0x10000, b=0x10000, epilogue=O.GEMM_F32)
    assert N.lib().lrm_op_gemm_bf16(None, ctypes.byref(g)) == N.LRM_ERR_ARGUMENT


def test_product_path_fails_loudly_without_the_library():
    # No CPU fallback: with liblrmcuda.so absent, the first call into the product raises NativeLibraryMissing.
    code = (
        "import rosylnalive_b200.native as N\n"
        "N.LIB_PATH = '/nonexistent/liblrmcuda.so'\n"
        "from rosylnalive_b200 import ops, rope as R\n"
        "for call in (lambda: R.t_spec(R.QWEN3_INV_FREQ_BITS, 16), lambda: ops.error_word()):\n"
        "    try:\n"
        "        call()\n"
        "        print('RAN')\n"
        "    except N.NativeLibraryMissing:\n"
        "        print('MISSING')\n"
    )
    out = subprocess.run([sys.executable, "-c", code], cwd=ROOT, capture_output=True, text=True, timeout=300)
    assert out.stdout.split() == ["MISSING", "MISSING"], out.stdout + out.stderr
