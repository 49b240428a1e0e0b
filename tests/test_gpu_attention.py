"""BASELINE config 2, the standalone GQA attention op, against the oracle (GPU tier): 16 query / 8 KV heads,
head_dim 128, causal; Q/K/V ~ N(0, 1) from a seed with per-head RMSNorm then RoPE (theta 1e6, T_spec) applied to Q
and K, rounded to bf16 (the kernels' input type). The reference is CpuRef's attention (Rows.attention, sequential
FMA, exact softmax) on the same bf16 values in F64 and F32; the bf16 output is held to relL2 <= 1e-2 against F64
(one bf16 rounding of the output and of the softmax weights is about 2^-9 each)."""

import numpy as np
import pytest

from oracle import oracle as O
from tests.conftest import cuda_available

pytestmark = pytest.mark.gpu

if cuda_available():
    import torch

    from rosylnalive_b200 import ops
    from rosylnalive_b200 import rope as R
    from rosylnalive_b200 import synthetic as S

QH, KVH, HD = 16, 8, 128
SCALE = float(np.float32(HD ** -0.5))


def rel(a, b):
    a = np.asarray(a, np.float64).ravel()
    b = np.asarray(b, np.float64).ravel()
    return float(np.linalg.norm(a - b) / np.linalg.norm(b))


def bf16_round(x):
    return O.widen(S.bf16_rne(x)).reshape(x.shape)


def make_qkv(T, seed, cos, sin):
    g = np.random.default_rng(seed)
    q = g.standard_normal((T, QH * HD), dtype=np.float32)
    k = g.standard_normal((T, KVH * HD), dtype=np.float32)
    v = g.standard_normal((T, KVH * HD), dtype=np.float32)
    ones = S.bf16_rne(np.ones(HD, np.float32))
    q = O.rope_apply(O.rmsnorm(q, ones, 1e-6), cos, sin, QH, 0)
    k = O.rope_apply(O.rmsnorm(k, ones, 1e-6), cos, sin, KVH, 0)
    return bf16_round(q), bf16_round(k), bf16_round(v)


def to_dev(x, shape):
    return torch.from_numpy(np.ascontiguousarray(x, np.float32)).reshape(shape).to("cuda", torch.bfloat16)


@pytest.fixture(scope="module")
def tables():
    return R.t_spec(R.QWEN3_INV_FREQ_BITS, 4200)


@pytest.fixture(autouse=True)
def _device():
    ops.set_device(0)
    yield
    torch.cuda.synchronize()
    assert ops.error_word() == 0


@pytest.mark.parametrize("lens", [(2048,) * 8, (70, 129, 1, 64)])
def test_prefill_attention(tables, lens):
    cos, sin = tables
    qs, ks, vs = zip(*(make_qkv(L, 100 + i, cos, sin) for i, L in enumerate(lens)))
    q, k, v = (np.concatenate(x) for x in (qs, ks, vs))
    T = q.shape[0]
    cu = torch.tensor(np.concatenate([[0], np.cumsum(lens)]), dtype=torch.int32, device="cuda")
    out = torch.full((T, QH, HD), float("nan"), device="cuda", dtype=torch.bfloat16)
    ops.prefill_attention(to_dev(q, (T, QH, HD)), to_dev(k, (T, KVH, HD)), to_dev(v, (T, KVH, HD)), out, cu,
                          max(lens), SCALE)
    torch.cuda.synchronize()
    got = out.float().cpu().numpy().reshape(T, QH * HD)
    start = 0
    for i, L in enumerate(lens):
        sl = slice(start, start + L)
        r64 = O.attention(q[sl], k[sl], v[sl], QH, KVH, HD, 0, SCALE, "f64")
        assert rel(got[sl], r64) <= 1e-2, (i, rel(got[sl], r64))
        start += L


@pytest.mark.parametrize("lens,pps", [((4096,) * 8, 32), ((4093, 17, 1, 64, 65, 1000, 16, 4096), 32),
                                      ((300, 2000), 1), ((4096, 33), 1000)])
def test_decode_attention_paged(tables, lens, pps):
    cos, sin = tables
    B = len(lens)
    maxp = (max(lens) + 15) // 16
    npages = sum((L + 15) // 16 for L in lens) + 3
    perm = np.random.default_rng(5).permutation(npages)
    pool = np.zeros((npages, KVH, 2, 16, HD), np.float32)
    table = np.zeros((B, maxp), np.int32)
    qrows, refs = [], []
    nxt = 0
    for b, L in enumerate(lens):
        q, k, v = make_qkv(L, 200 + b, cos, sin)
        for p in range((L + 15) // 16):
            pg = int(perm[nxt])
            nxt += 1
            table[b, p] = pg
            t0, t1 = 16 * p, min(L, 16 * p + 16)
            pool[pg, :, 0, :t1 - t0] = k[t0:t1].reshape(t1 - t0, KVH, HD).transpose(1, 0, 2)
            pool[pg, :, 1, :t1 - t0] = v[t0:t1].reshape(t1 - t0, KVH, HD).transpose(1, 0, 2)
        qrows.append(q[L - 1])
        refs.append(O.attention(q[L - 1:L], k, v, QH, KVH, HD, L - 1, SCALE, "f64")[0])
    dq = to_dev(np.stack(qrows), (B, QH, HD))
    dpool = to_dev(pool, pool.shape)
    dtable = torch.from_numpy(table).cuda()
    dlens = torch.tensor(lens, dtype=torch.int32, device="cuda")
    slots = torch.arange(B, dtype=torch.int32, device="cuda")
    ws = torch.empty(ops.decode_attention_workspace(B, KVH, maxp, pps) // 4, device="cuda")
    out = torch.full((B, QH, HD), float("nan"), device="cuda", dtype=torch.bfloat16)
    ops.decode_attention(dq, dpool, dtable, dlens, slots, out, ws, pps, SCALE)
    torch.cuda.synchronize()
    got = out.float().cpu().numpy().reshape(B, QH * HD)
    for b in range(B):
        assert rel(got[b], refs[b]) <= 1e-2, (b, lens[b], rel(got[b], refs[b]))


def test_decode_attention_rejects_bad_shapes():
    q = torch.zeros(2, 16, 128, device="cuda", dtype=torch.bfloat16)
    pool = torch.zeros(4, 4, 2, 16, 128, device="cuda", dtype=torch.bfloat16)  # 4 kv heads but 16 q heads
    t = torch.zeros(2, 2, dtype=torch.int32, device="cuda")
    lens = torch.ones(2, dtype=torch.int32, device="cuda")
    ws = torch.empty(1 << 16, device="cuda")
    with pytest.raises(ValueError):
        ops.decode_attention(q, pool, t, lens, lens, q, ws, 1, 0.1)


def test_decode_attention_row_longer_than_its_page_table(tables):
    # Row 1 claims 113 keys but its page-table row holds 7 pages (112 tokens). Both kernels check every row's key
    # count against the table before reading it: that row's pages and split states are not touched, the error word
    # gets 0x2010 and the row's output is zeros; the other rows are computed as usual.
    cos, sin = tables
    lens, maxp, pps = (100, 100, 50), 7, 2
    B = len(lens)
    pool = np.zeros((B * maxp, KVH, 2, 16, HD), np.float32)
    table = np.arange(B * maxp, dtype=np.int32).reshape(B, maxp)
    qrows, refs = [], []
    for b, L in enumerate(lens):
        q, k, v = make_qkv(L, 300 + b, cos, sin)
        for p in range((L + 15) // 16):
            t0, t1 = 16 * p, min(L, 16 * p + 16)
            pool[table[b, p], :, 0, :t1 - t0] = k[t0:t1].reshape(t1 - t0, KVH, HD).transpose(1, 0, 2)
            pool[table[b, p], :, 1, :t1 - t0] = v[t0:t1].reshape(t1 - t0, KVH, HD).transpose(1, 0, 2)
        qrows.append(q[L - 1])
        refs.append(O.attention(q[L - 1:L], k, v, QH, KVH, HD, L - 1, SCALE, "f64")[0])
    dlens = torch.tensor([lens[0], maxp * 16 + 1, lens[2]], dtype=torch.int32, device="cuda")
    slots = torch.arange(B, dtype=torch.int32, device="cuda")
    ws = torch.empty(ops.decode_attention_workspace(B, KVH, maxp, pps) // 4, device="cuda")
    out = torch.full((B, QH, HD), float("nan"), device="cuda", dtype=torch.bfloat16)
    ops.decode_attention(to_dev(np.stack(qrows), (B, QH, HD)), to_dev(pool, pool.shape),
                         torch.from_numpy(table).cuda(), dlens, slots, out, ws, pps, SCALE)
    torch.cuda.synchronize()
    assert ops.error_word(clear=True) == 0x2010
    got = out.float().cpu().numpy().reshape(B, QH * HD)
    assert np.all(got[1] == 0)
    for b in (0, 2):
        assert rel(got[b], refs[b]) <= 1e-2, (b, rel(got[b], refs[b]))


def test_decode_attention_refuses_page_counts_above_2_20():
    q = torch.zeros(1, 16, 128, device="cuda", dtype=torch.bfloat16)
    pool = torch.zeros(1, 8, 2, 16, 128, device="cuda", dtype=torch.bfloat16)
    t = torch.zeros(1, 1, dtype=torch.int32, device="cuda")
    lens = torch.ones(1, dtype=torch.int32, device="cuda")
    assert ops.decode_attention_workspace(1, 8, (1 << 20) + 1, 1) == 0
    assert ops.decode_attention_workspace(1, 8, 1 << 20, (1 << 20) + 1) == 0
    with pytest.raises(ValueError):
        ops.decode_attention(q, pool, t, lens, lens, q, torch.empty(1 << 10, device="cuda"), (1 << 20) + 1, 0.1)


@pytest.mark.parametrize("case", ["past_total_tokens", "longer_than_max_len"])
def test_prefill_attention_sequence_outside_its_rows(tables, case):
    # cu_seqlens lives on the device, so only the kernel can check it. A sequence that runs past total_tokens, or is
    # longer than max_len, is not computed: the error word gets 0x3010, its rows stay as they were, and the other
    # sequence is computed as usual. The buffers hold 256 rows more than total_tokens (poisoned), which stay
    # untouched too.
    cos, sin = tables
    lens, slack = (100, 60), 256
    T = sum(lens)
    q, k, v = make_qkv(T + slack, 400, cos, sin)
    if case == "past_total_tokens":
        cu_host, max_len, bad, good = [0, 100, 100 + 60 + 200], 260, 1, 0
    else:
        cu_host, max_len, bad, good = [0, 100, 160], 64, 0, 1
    cu = torch.tensor(cu_host, dtype=torch.int32, device="cuda")
    qd, kd, vd = to_dev(q, (T + slack, QH, HD)), to_dev(k, (T + slack, KVH, HD)), to_dev(v, (T + slack, KVH, HD))
    out = torch.full((T + slack, QH, HD), float("nan"), device="cuda", dtype=torch.bfloat16)
    ops.prefill_attention(qd[:T], kd[:T], vd[:T], out[:T], cu, max_len, SCALE)
    torch.cuda.synchronize()
    assert ops.error_word(clear=True) == 0x3010
    got = out.float().cpu().numpy().reshape(T + slack, QH * HD)
    starts = (0, 100)
    b0, b1 = starts[bad], starts[bad] + lens[bad]
    assert np.all(np.isnan(got[b0:b1])) and np.all(np.isnan(got[T:]))
    sl = slice(starts[good], starts[good] + lens[good])
    r64 = O.attention(q[sl], k[sl], v[sl], QH, KVH, HD, 0, SCALE, "f64")
    assert rel(got[sl], r64) <= 1e-2, rel(got[sl], r64)
