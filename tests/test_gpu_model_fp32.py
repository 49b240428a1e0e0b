"""The fp32 path end to end on the CUDA device (GPU tier): the planned executor over the device contracts runs the
reference's tiny Qwen3 (goldens/tiny/g1) and BASELINE config 1, and must give the golden greedy ids and logits within
1e-4 max-abs of the CPU reference (the fp32 bar of the build's goal)."""

import json

import numpy as np
import pytest

from oracle import oracle as O
from tests.conftest import cuda_available

pytestmark = pytest.mark.gpu

if cuda_available():
    from rosylnalive_b200 import cuda_backend as CB
    from rosylnalive_b200 import executor as X
    from rosylnalive_b200 import rope as R
    from rosylnalive_b200 import synthetic as S


def tiny_setup(z):
    cfg = X.QwenConfig.from_hf(json.loads(bytes(z["config_json"]).decode()))
    weights = {k[2:]: z[k] for k in z.files if k.startswith("w/")}
    cos, sin = R.t_spec(z["rope/inv_freq.bits"], cfg.max_pos)
    return cfg, weights, cos, sin


def oracle_model(cfg, weights, cos, sin):
    oc = O.Config(cfg.layers, cfg.hidden, cfg.heads, cfg.kv_heads, cfg.head_dim, cfg.intermediate, cfg.vocab, cfg.eps,
                  cfg.max_pos)
    return O.Model.from_hf(oc, weights, cos, sin)


@pytest.fixture(scope="module")
def tiny_exec(tiny_golden):
    cfg, weights, cos, sin = tiny_setup(tiny_golden)
    b = CB.try_create()
    ex = X.Fp32Executor(b, cfg, weights, cos, sin, max_tokens=128)
    yield ex, cfg, weights, cos, sin
    b.dispose()


@pytest.mark.parametrize("prompt", ["p0", "p1"])
def test_tiny_greedy_64_steps_equal_golden(tiny_exec, tiny_golden, prompt):
    ex, cfg, weights, cos, sin = tiny_exec
    ids, logits = ex.greedy(tiny_golden[f"prompt/{prompt}"], 64, return_logits=True)
    assert np.array_equal(ids, tiny_golden[f"greedy/{prompt}.ids.torch32"])
    m = oracle_model(cfg, weights, cos, sin)
    ref_ids, ref_logits = O.greedy(m, tiny_golden[f"prompt/{prompt}"], 64, "f32", return_logits=True)
    assert np.array_equal(ids, ref_ids)
    assert np.max(np.abs(logits - ref_logits)) <= 1e-4


def test_tiny_p2_logits_all_rows(tiny_exec, tiny_golden):
    ex, cfg, weights, cos, sin = tiny_exec
    ex.reset_cache()
    logits, _ = ex.forward(0, tiny_golden["prompt/p2"], "all")
    m = oracle_model(cfg, weights, cos, sin)
    ref = O.forward(m, O.Cache.new(m.config, "f32"), 0, tiny_golden["prompt/p2"], "f32")
    assert np.max(np.abs(logits - ref)) <= 1e-4
    assert np.max(np.abs(logits - tiny_golden["torch32/p2/logits"])) <= 2e-3


def test_tiny_prefill_equals_decode_on_device(tiny_exec, tiny_golden):
    """BatchInvariance on the device: decode rows equal the same rows of one prefill, bit for bit."""
    ex, *_ = tiny_exec
    prompt = tiny_golden["prompt/p0"]
    ex.reset_cache()
    full, _ = ex.forward(0, prompt, "all")
    ex.reset_cache()
    rows = [ex.forward(i, [t], "all")[0] for i, t in enumerate(prompt)]
    assert np.array_equal(np.concatenate(rows).view(np.uint32), full.view(np.uint32))


def test_config1_fp32_greedy_and_logits():
    """2 layers, hidden 64, 4/2 heads of 16, inter 128, vocab 256, N(0,0.02) weights from seed 0,
    a 16-token prompt, 16 greedy steps."""
    cfg = S.CONFIG1
    weights = S.random_weights(cfg, seed=0)
    cos, sin = R.t_spec(R.torch_inv_freq_bits(cfg.rope_theta, cfg.head_dim), cfg.max_pos)
    prompt = S.random_prompt(cfg.vocab, 16, seed=0)
    b = CB.try_create()
    try:
        ex = X.Fp32Executor(b, cfg, weights, cos, sin, max_tokens=32)
        ids, logits = ex.greedy(prompt, 16, return_logits=True)
    finally:
        b.dispose()
    m = oracle_model(cfg, weights, cos, sin)
    ref_ids, ref_logits = O.greedy(m, prompt, 16, "f32", return_logits=True)
    assert np.array_equal(ids, ref_ids)
    assert np.max(np.abs(logits - ref_logits)) <= 1e-4


def rel_l2(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-300))


@pytest.mark.parametrize("prompt", ["p0", "p1"])
def test_tiny_taps_arena_equals_the_reference_taps(tiny_golden, prompt):
    """Every intermediate of the forward, copied into the Taps arena at record time, against the reference's torch32
    taps (goldens/tiny/g1 fwd_f32.*, rel-L2 <= 1e-5: the bar the CPU reference meets) and the CPU reference's own
    taps (max-abs <= 1e-4)."""
    cfg, weights, cos, sin = tiny_setup(tiny_golden)
    b = CB.try_create()
    try:
        ex = X.Fp32Executor(b, cfg, weights, cos, sin, max_tokens=32, taps=True)
        ex.reset_cache()
        ids = tiny_golden[f"prompt/{prompt}"]
        ex.forward(0, ids, "all")
        got = ex.read_taps()
    finally:
        b.dispose()
    m = oracle_model(cfg, weights, cos, sin)
    ref = {}
    O.forward(m, O.Cache.new(m.config, "f32"), 0, ids, "f32", ref)
    assert len(got) == 39 and set(got) == set(ref)
    for k, v in got.items():
        assert v.shape == np.asarray(ref[k]).shape, k
        assert rel_l2(v, tiny_golden[f"torch32/{prompt}/{k}"]) <= 1e-5, k
        assert np.max(np.abs(v - ref[k])) <= 1e-4, k
