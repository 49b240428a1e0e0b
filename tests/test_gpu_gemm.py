"""The tcgen05 GEMM (lrm_op_gemm_bf16) against an fp64 reference on the same bf16 inputs (GPU tier).

fp32 accumulation in TMEM over k <= 3072 keeps the relative L2 error near 1e-6; the bound used is 2e-5 for fp32
outputs and 1e-2 for bf16-rounded outputs (one bf16 rounding is 2^-9 relative)."""

import pytest

from tests.conftest import cuda_available

pytestmark = pytest.mark.gpu

if cuda_available():
    import torch

    from rosylnalive_b200 import ops


def rel(a, b):
    a = a.double()
    b = b.double()
    return ((a - b).norm() / b.norm().clamp_min(1e-300)).item()


def bf16(shape, scale=1.0, seed=0):
    g = torch.Generator(device="cuda").manual_seed(seed)
    return (torch.randn(*shape, generator=g, device="cuda") * scale).to(torch.bfloat16)


@pytest.fixture(autouse=True)
def _device():
    ops.set_device(0)
    assert ops.error_word() == 0
    yield
    torch.cuda.synchronize()
    assert ops.error_word() == 0


@pytest.mark.parametrize("m,n,k,bn", [(256, 256, 1024, 256), (200, 192, 512, 64), (1, 4096, 1024, 128),
                                      (384, 1024, 3072, 256), (130, 152, 64, 128), (4096, 2048, 1024, 256),
                                      (17, 64, 136, 64)])
def test_gemm_f32(m, n, k, bn):
    a, b = bf16((m, k), seed=1), bf16((n, k), 0.05, seed=2)
    out = torch.full((m, n), float("nan"), device="cuda")
    ops.gemm(a, b, out, ops.GEMM_F32, bn=bn)
    torch.cuda.synchronize()
    ref = a.double() @ b.double().T
    assert rel(out, ref) < 2e-5


def test_gemm_resid_in_place():
    m, n, k = 300, 1024, 2048
    a, b = bf16((m, k), seed=3), bf16((n, k), 0.02, seed=4)
    x = torch.randn(m, n, device="cuda")
    ref = x.double() + a.double() @ b.double().T
    ops.gemm(a, b, x, ops.GEMM_RESID, resid=x)
    torch.cuda.synchronize()
    assert rel(x, ref) < 2e-5


def test_gemm_swiglu_interleaved():
    m, n, k = 256, 768, 1024
    a, b = bf16((m, k), seed=5), bf16((n, k), 0.05, seed=6)
    out = torch.zeros(m, n // 2, device="cuda", dtype=torch.bfloat16)
    ops.gemm(a, b, out, ops.GEMM_SWIGLU, bn=256)
    torch.cuda.synchronize()
    y = a.double() @ b.double().T
    y = y.view(m, n // 128, 2, 64)
    g, u = y[:, :, 0, :], y[:, :, 1, :]
    ref = (g * torch.sigmoid(g) * u).reshape(m, n // 2)
    assert rel(out, ref) < 1e-2


def test_gemm_split_k_partials_transposed():
    feats, toks, k, splits = 4096, 64, 1024, 4
    w, x = bf16((feats, k), 0.05, seed=7), bf16((toks, k), seed=8)
    part = torch.full((splits, toks, feats), float("nan"), device="cuda")
    ops.gemm(w, x, part, ops.GEMM_PARTIAL, splits=splits, bn=64, split_stride=toks * feats)
    torch.cuda.synchronize()
    ref = x.double() @ w.double().T
    assert rel(part.sum(0), ref) < 2e-5


def test_gemm_bf16_out():
    m, n, k = 512, 1536, 1024
    a, b = bf16((m, k), seed=9), bf16((n, k), 0.05, seed=10)
    out = torch.zeros(m, n, device="cuda", dtype=torch.bfloat16)
    ops.gemm(a, b, out, ops.GEMM_BF16)
    torch.cuda.synchronize()
    assert rel(out, a.double() @ b.double().T) < 1e-2


def test_gemm_rejects_bad_arguments():
    a, b = bf16((64, 100)), bf16((64, 100))
    out = torch.zeros(64, 64, device="cuda")
    with pytest.raises(ValueError):
        ops.gemm(a, b, out)  # k = 100 is not a multiple of 8


# Two-SM clusters (cta_pair=2: tcgen05 cta_group::2, 256 x 256 tiles split over a CTA pair), including tiles whose
# second CTA holds no valid rows (m <= 128 within a tile) and ragged n.
@pytest.mark.parametrize("m,n,k", [(256, 256, 1024), (300, 520, 512), (130, 256, 64), (4096, 2048, 1024),
                                   (1000, 1024, 3072), (77, 136, 136)])
def test_gemm_pair_f32(m, n, k):
    a, b = bf16((m, k), seed=11), bf16((n, k), 0.05, seed=12)
    out = torch.full((m, n), float("nan"), device="cuda")
    ops.gemm(a, b, out, ops.GEMM_F32, bn=256, cta_pair=2)
    torch.cuda.synchronize()
    assert rel(out, a.double() @ b.double().T) < 2e-5


def test_gemm_pair_matches_single_cta_bitwise():
    m, n, k = 1536, 1280, 2048
    a, b = bf16((m, k), seed=13), bf16((n, k), 0.05, seed=14)
    o1 = torch.zeros(m, n, device="cuda")
    o2 = torch.zeros(m, n, device="cuda")
    ops.gemm(a, b, o1, ops.GEMM_F32, bn=256, cta_pair=1)
    ops.gemm(a, b, o2, ops.GEMM_F32, bn=256, cta_pair=2)
    torch.cuda.synchronize()
    assert rel(o2, a.double() @ b.double().T) < 2e-5
    assert torch.equal(o1, o2)


def test_gemm_pair_resid_swiglu_bf16():
    m, k = 1100, 1024
    a = bf16((m, k), seed=15)
    b = bf16((1024, k), 0.02, seed=16)
    x = torch.randn(m, 1024, device="cuda")
    ref = x.double() + a.double() @ b.double().T
    ops.gemm(a, b, x, ops.GEMM_RESID, resid=x, bn=256, cta_pair=2)
    torch.cuda.synchronize()
    assert rel(x, ref) < 2e-5

    bg = bf16((768, k), 0.05, seed=17)
    out = torch.zeros(m, 384, device="cuda", dtype=torch.bfloat16)
    ops.gemm(a, bg, out, ops.GEMM_SWIGLU, bn=256, cta_pair=2)
    torch.cuda.synchronize()
    y = (a.double() @ bg.double().T).view(m, 6, 2, 64)
    g, u = y[:, :, 0, :], y[:, :, 1, :]
    assert rel(out, (g * torch.sigmoid(g) * u).reshape(m, 384)) < 1e-2

    ob = torch.zeros(m, 768, device="cuda", dtype=torch.bfloat16)
    ops.gemm(a, bg, ob, ops.GEMM_BF16, bn=256, cta_pair=2)
    torch.cuda.synchronize()
    assert rel(ob, a.double() @ bg.double().T) < 1e-2


@pytest.mark.parametrize("epi", ["resid", "bf16", "swiglu"])
def test_gemm_pair_epilogues_match_single_cta_bitwise(epi):
    # The staged (shared-memory) epilogue of CTA pairs computes exactly what the per-row one does; ragged m and n.
    m, k = 1300, 1024
    n = 768 if epi == "swiglu" else 1000
    a, b = bf16((m, k), seed=18), bf16((n, k), 0.05, seed=19)
    if epi == "resid":
        x = torch.randn(m, n, device="cuda")
        o1, o2 = x.clone(), x.clone()
        ops.gemm(a, b, o1, ops.GEMM_RESID, resid=o1, bn=256, cta_pair=1)
        ops.gemm(a, b, o2, ops.GEMM_RESID, resid=o2, bn=256, cta_pair=2)
    else:
        width = n // 2 if epi == "swiglu" else n
        kind = ops.GEMM_SWIGLU if epi == "swiglu" else ops.GEMM_BF16
        o1 = torch.zeros(m, width, device="cuda", dtype=torch.bfloat16)
        o2 = torch.full((m, width), 7.0, device="cuda", dtype=torch.bfloat16)
        ops.gemm(a, b, o1, kind, bn=256, cta_pair=1)
        ops.gemm(a, b, o2, kind, bn=256, cta_pair=2)
    torch.cuda.synchronize()
    assert torch.equal(o1, o2)


def test_gemm_pair_rejects_unsupported():
    a, b = bf16((256, 256)), bf16((256, 256))
    out = torch.zeros(256, 256, device="cuda")
    with pytest.raises(ValueError):
        ops.gemm(a, b, out, ops.GEMM_F32, bn=128, cta_pair=2)
