"""A bounded in-kernel wait that runs out (GPU tier). Every wait of this library's kernels (TMA stages, MMA
completion, accumulator hand-off) is ptx::mbar_wait: a bounded spin that, when it gives up, records a code in the
device's error word and lets the kernel return, so the host sees an error status instead of a hung GPU -- the CUDA
counterpart of the reference's device wait timeout (src/Lrm.Gpu.D3D12/Backend.fs:109, Context.fs:200-234).

lrm_op_wait_probe runs that same wait on an mbarrier nothing arrives on (no copy is ever issued), with a short poll
limit. The test checks that the kernel returns, that its code is in the error word, and that the device still runs a
GEMM bit for bit as before. Nothing faults, traps or hangs."""

import time

import pytest

from tests.conftest import cuda_available

pytestmark = pytest.mark.gpu

if cuda_available():
    import torch

    from rosylnalive_b200 import ops


def test_bounded_wait_gives_up_with_a_code_and_the_device_stays_usable():
    ops.set_device(0)
    assert ops.error_word(clear=True) == 0
    g = torch.Generator(device="cuda").manual_seed(11)
    a = torch.randn(256, 1024, device="cuda", generator=g).to(torch.bfloat16)
    b = (torch.randn(512, 1024, device="cuda", generator=g) * 0.02).to(torch.bfloat16)
    before = torch.empty(256, 512, device="cuda")
    ops.gemm(a, b, before)
    torch.cuda.synchronize()
    assert ops.error_word(clear=False) == 0

    t0 = time.time()
    ops.wait_probe(1000, 0x7E57)
    torch.cuda.synchronize()  # the kernel returned: its wait gave up after 1,000 polls
    elapsed = time.time() - t0
    assert elapsed < 10.0, elapsed
    assert ops.error_word(clear=False) == 0x7E57
    assert ops.error_word(clear=True) == 0x7E57
    assert ops.error_word(clear=False) == 0

    after = torch.empty_like(before)
    ops.gemm(a, b, after)
    torch.cuda.synchronize()
    assert torch.equal(before, after)
    assert ops.error_word(clear=False) == 0

    # the first writer wins: a second code does not replace one the host has not cleared
    ops.wait_probe(10, 0x1)
    ops.wait_probe(10, 0x2)
    torch.cuda.synchronize()
    assert ops.error_word(clear=True) == 0x1


def test_wait_probe_refuses_bad_arguments():
    ops.set_device(0)
    with pytest.raises(ValueError):
        ops.wait_probe(0, 1)
    with pytest.raises(ValueError):
        ops.wait_probe(1 << 25, 1)
    with pytest.raises(ValueError):
        ops.wait_probe(10, 0)
