"""The engine's greedy pick (lrm_op_argmax_rows: a cluster of 8 CTAs a row) against the oracle's argmax_rows (GPU tier).

The contract is the reference's argmax_rows (src/Lrm.Tensor.CpuReference/CpuRef.fs:452-466): each row's lowest
maximal index, or 0xFFFFFFFF for a row holding a NaN. Checked bit for bit on the vocabulary of Qwen3 (a multiple of
4, read as float4) and on an odd one (read one float at a time), with ties inside one float4, ties across the CTAs'
chunks, a NaN row, an all -inf row and a +inf column; a misaligned row start and a bad row count are refused."""

import numpy as np
import pytest

from tests.conftest import cuda_available

pytestmark = pytest.mark.gpu

if cuda_available():
    import torch

    from rosylnalive_b200 import ops

import oracle.oracle as O


@pytest.fixture(autouse=True)
def _device():
    ops.set_device(0)
    yield
    torch.cuda.synchronize()
    assert ops.error_word() == 0


def run(x):
    d = torch.from_numpy(x).cuda()
    out = torch.full((x.shape[0],), -1, dtype=torch.int32, device="cuda")
    ops.argmax_rows(d, out)
    torch.cuda.synchronize()
    return out.cpu().numpy().view(np.uint32)


def planted(rows, vocab, seed):
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((rows, vocab)).astype(np.float32)
    chunk = ((vocab + 7) // 8 + 3) & ~3  # the kernel's columns per CTA
    x[1, [5, 6]] = 50.0                                     # a tie inside one float4: the lower index
    x[2, [chunk - 1, chunk + 3, vocab - 1]] = 60.0          # a tie across CTA chunks
    x[3, vocab // 2] = np.nan                               # a NaN row
    x[4, :] = -np.inf                                       # all -inf: index 0
    x[5, 7] = np.inf                                        # +inf wins
    x[6, vocab - 1] = 70.0                                  # the last column
    x[7, 0] = 70.0                                          # the first column
    return x


@pytest.mark.parametrize("vocab", [151936, 1001, 4, 3])
def test_argmax_rows_matches_oracle(vocab):
    if vocab > 8:
        x = planted(64, vocab, vocab)
    else:  # rows narrower than the planted columns: one NaN row and one all-equal row
        x = np.random.default_rng(vocab).standard_normal((8, vocab)).astype(np.float32)
        x[1, 0] = np.nan
        x[2, :] = 3.0
    got = run(x)
    want = O.argmax_rows(x, "f32")
    assert np.array_equal(got, want)
    if vocab > 8:
        assert got[3] == 0xFFFFFFFF and got[4] == 0 and got[5] == 7 and got[6] == vocab - 1 and got[7] == 0


def test_argmax_rows_refuses_bad_arguments():
    x = torch.zeros(2, 8, device="cuda")
    out = torch.zeros(2, dtype=torch.int32, device="cuda")
    with pytest.raises(ValueError):
        ops.argmax_rows(x[:0], out)
    flat = torch.zeros(17, device="cuda")
    with pytest.raises(ValueError):  # 4-byte offset: rows of 4 columns would start off a 16-byte boundary
        ops.argmax_rows(flat[1:].view(4, 4), out)
