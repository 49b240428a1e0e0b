"""The decode step's fused GEMMs (lrm_op_decode_gemm) against float64 on the same bf16 inputs (GPU tier).

The weight GEMM of a decode step, K split over a thread-block cluster and reduced through distributed shared memory,
with its consumer in the epilogue. Checked at the Qwen3-0.6B decode shapes, at token counts below, at and above one
64-token tile, and at every compiled cluster size:
  * residual (o_proj / down): x += y within fp32 accumulation error (relative L2 <= 2e-5 of y); the next norm's
    inputs u = bf16(gain * x) within one bf16 rounding, the 128-column sums of squares to 1e-5;
  * SwiGLU (gate/up): act = bf16(silu(r g) * (r u)) with the norm scale r from the sums, relative L2 <= 1e-2;
  * the split count changes the result only by fp32 summation order (relative L2 <= 1e-5)."""

import numpy as np
import pytest

from tests.conftest import cuda_available

pytestmark = pytest.mark.gpu

if cuda_available():
    import torch

    from rosylnalive_b200 import ops


def rel(a, b):
    a = np.asarray(a, np.float64).ravel()
    b = np.asarray(b, np.float64).ravel()
    return float(np.linalg.norm(a - b) / np.linalg.norm(b))


def bf16(g, shape, scale=1.0, offset=0.0):
    return (torch.randn(*shape, device="cuda", generator=g) * scale + offset).to(torch.bfloat16)


@pytest.fixture(autouse=True)
def _device():
    ops.set_device(0)
    yield
    torch.cuda.synchronize()
    assert ops.error_word() == 0


@pytest.mark.parametrize("m,k,n,splits", [(1024, 2048, 64, 0), (1024, 3072, 64, 0), (1024, 2048, 37, 8),
                                          (1024, 3072, 100, 16), (256, 512, 64, 4), (1024, 1024, 64, 1)])
def test_residual_with_norm_inputs(m, k, n, splits):
    g = torch.Generator(device="cuda").manual_seed(m + k + n + splits)
    w = bf16(g, (m, k), 0.02)
    b = bf16(g, (n, k))
    x = torch.randn(n, m, device="cuda", generator=g)
    gain = bf16(g, (m,), 0.02, 1.0)
    u = torch.full((n, m), float("nan"), device="cuda", dtype=torch.bfloat16)
    ss = torch.full((m // 128, n), float("nan"), device="cuda")
    x0 = x.double().cpu().numpy()
    ops.decode_gemm_resid(w, b, x, gain, u, ss, splits=splits)
    torch.cuda.synchronize()
    want = x0 + b.double().cpu().numpy() @ w.double().cpu().numpy().T
    got = x.double().cpu().numpy()
    assert rel(got - x0, want - x0) <= 2e-5
    u_want = (torch.from_numpy(got).float() * gain.float().cpu()).to(torch.bfloat16).float().numpy()
    assert np.array_equal(u.float().cpu().numpy(), u_want)
    ss_want = (got.reshape(n, m // 128, 128) ** 2).sum(-1).T
    assert np.max(np.abs(ss.double().cpu().numpy() - ss_want) / ss_want) <= 1e-5


def test_residual_without_gain_writes_x_only():
    g = torch.Generator(device="cuda").manual_seed(5)
    w, b = bf16(g, (1024, 2048), 0.02), bf16(g, (64, 2048))
    x = torch.randn(64, 1024, device="cuda", generator=g)
    x0 = x.double().cpu().numpy()
    ops.decode_gemm_resid(w, b, x)
    torch.cuda.synchronize()
    want = x0 + b.double().cpu().numpy() @ w.double().cpu().numpy().T
    assert rel(x.double().cpu().numpy() - x0, want - x0) <= 2e-5


@pytest.mark.parametrize("n,splits", [(64, 0), (17, 3), (100, 4), (64, 2)])
def test_swiglu_with_norm_scale(n, splits):
    m, k, hidden, eps = 6144, 1024, 1024, 1e-6
    g = torch.Generator(device="cuda").manual_seed(n + splits)
    w = bf16(g, (m, k), 0.02)
    xr = torch.randn(n, hidden, device="cuda", generator=g) * 3.0
    b = xr.to(torch.bfloat16)  # the GEMM's B is u = bf16(gain * x); any bf16 rows will do
    ss = (xr.double() ** 2).reshape(n, hidden // 128, 128).sum(-1).T.contiguous().float()
    act = torch.full((n, m // 2), float("nan"), device="cuda", dtype=torch.bfloat16)
    ops.decode_gemm_swiglu(w, b, ss, hidden, eps, act, splits=splits)
    torch.cuda.synchronize()
    y = b.double().cpu().numpy() @ w.double().cpu().numpy().T
    r = 1.0 / np.sqrt(ss.double().cpu().numpy().sum(0) / hidden + eps)
    y = y * r[:, None]
    blocks = y.reshape(n, m // 128, 2, 64)
    gate, up = blocks[:, :, 0, :].reshape(n, -1), blocks[:, :, 1, :].reshape(n, -1)
    want = gate / (1.0 + np.exp(-gate)) * up
    assert rel(act.double().cpu().numpy(), want) <= 1e-2


def test_split_counts_agree():
    g = torch.Generator(device="cuda").manual_seed(9)
    w, b = bf16(g, (1024, 3072), 0.02), bf16(g, (64, 3072))
    outs = []
    for s in (1, 2, 3, 4, 8, 16):
        x = torch.zeros(64, 1024, device="cuda")
        ops.decode_gemm_resid(w, b, x, splits=s)
        outs.append(x.double().cpu().numpy())
    torch.cuda.synchronize()
    for o in outs[1:]:
        assert rel(o, outs[0]) <= 1e-5


def test_decode_gemm_refuses_bad_arguments():
    g = torch.Generator(device="cuda").manual_seed(1)
    w, b = bf16(g, (1000, 1024), 0.02), bf16(g, (8, 1024))  # 1000 rows: not a multiple of 128
    x = torch.zeros(8, 1000, device="cuda")
    with pytest.raises(ValueError):
        ops.decode_gemm_resid(w, b, x)
    w = bf16(g, (1024, 1024), 0.02)
    with pytest.raises(ValueError):
        ops.decode_gemm_resid(w, b, torch.zeros(8, 1024, device="cuda"), splits=5)
