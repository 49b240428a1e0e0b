"""Decode attention without device allocation (lrm_op_decode_attention_static), on the GPU.

Some callers cannot allocate device memory per call -- a host that sizes all device memory once (as the reference's
device contract does with its single CreateHeap), a serving loop with a fixed budget, code inside a stream capture --
so they cannot hand lrm_op_decode_attention its split-K workspace. The static entry point uses a 16 MiB scratch array
built into the library instead. This file checks it, through the C ABI, against the workspace entry point on two
calls in a row (the second with shorter sequences, so stale scratch from the first call must not leak into it), and
that oversized calls are refused. It is named to run last: it must pass alone in a fresh process and after the rest.
"""

import numpy as np
import pytest

from tests.conftest import cuda_available

pytestmark = pytest.mark.gpu

if cuda_available():
    import torch

    from rosylnalive_b200 import ops

QH, KVH, HD = 16, 8, 128
SCALE = float(np.float32(HD ** -0.5))


def rel(a, b):
    a = a.double().flatten()
    b = b.double().flatten()
    return float((a - b).norm() / b.norm())


def paged_case(lens, seed):
    g = torch.Generator(device="cpu").manual_seed(seed)
    B = len(lens)
    maxp = (max(lens) + 15) // 16
    npages = sum((L + 15) // 16 for L in lens) + 5
    perm = torch.randperm(npages, generator=g)
    table = torch.zeros(B, maxp, dtype=torch.int32)
    nxt = 0
    for b, L in enumerate(lens):
        for p in range((L + 15) // 16):
            table[b, p] = int(perm[nxt])
            nxt += 1
    pool = torch.randn(npages, KVH, 2, 16, HD, generator=g).to(torch.bfloat16).cuda()
    q = torch.randn(B, QH, HD, generator=g).to(torch.bfloat16).cuda()
    return q, pool, table.cuda(), torch.tensor(lens, dtype=torch.int32, device="cuda")


@pytest.fixture(autouse=True)
def _device():
    ops.set_device(0)
    yield
    torch.cuda.synchronize()
    assert ops.error_word() == 0


def run_both(q, pool, table, lens, pps):
    B = q.shape[0]
    slots = torch.arange(B, dtype=torch.int32, device="cuda")
    ws = torch.empty(ops.decode_attention_workspace(B, KVH, table.shape[1], pps) // 4, device="cuda")
    ref = torch.full_like(q, float("nan"))
    ops.decode_attention(q, pool, table, lens, slots, ref, ws, pps, SCALE)
    got = torch.full_like(q, float("nan"))
    ops.decode_attention_static(q, pool, table, lens, slots, got, pps, SCALE)
    torch.cuda.synchronize()
    return ref, got


def test_static_scratch_matches_workspace_entry_point_twice():
    q, pool, table, lens = paged_case([4096, 1000, 17, 1, 333, 2048, 4095, 64], seed=1)
    ref1, got1 = run_both(q, pool, table, lens, 8)
    assert not torch.isnan(got1.float()).any()
    assert rel(got1, ref1) <= 1e-2
    assert torch.equal(got1, ref1)
    # Second call in a row: shorter sequences use fewer splits, so the first call's partials stay in the scratch
    # beyond what this call writes; the output must still match.
    lens2 = torch.tensor([100, 5, 17, 1, 300, 16, 4000, 63], dtype=torch.int32, device="cuda")
    q2 = (q.float() * -0.5).to(torch.bfloat16)
    ref2, got2 = run_both(q2, pool, table, lens2, 8)
    assert not torch.isnan(got2.float()).any()
    assert rel(got2, ref2) <= 1e-2
    assert torch.equal(got2, ref2)


def test_static_scratch_refuses_oversized_calls():
    q, pool, table, lens = paged_case([32], seed=2)
    need = ops.decode_attention_workspace(4096, KVH, 4096, 1)
    assert need > ops.DECODE_ATTN_STATIC_SCRATCH_BYTES
    big_q = torch.zeros(4096, QH, HD, dtype=torch.bfloat16, device="cuda")
    big_table = torch.zeros(4096, 4096, dtype=torch.int32, device="cuda")
    big_lens = torch.ones(4096, dtype=torch.int32, device="cuda")
    slots = torch.arange(4096, dtype=torch.int32, device="cuda")
    with pytest.raises(ValueError, match="scratch"):
        ops.decode_attention_static(big_q, pool, big_table, big_lens, slots, big_q, 1, SCALE)
