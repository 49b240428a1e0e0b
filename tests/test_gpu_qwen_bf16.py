"""The bf16 fast path (QwenEngine over lrm_qwen_*) against the parity oracle (GPU tier).

Bar (from the build's goal): identical greedy tokens, and logits with cosine >= 0.9999 and max-abs <= 2e-2 against
the fp32 CPU reference on the same weights. A step whose oracle top-2 margin is below the bf16 path's logit error can
flip without the path being wrong; the tests pick prompts whose oracle margins clear that error (the reference's own
rule for greedy goldens: every step's top-2 margin >= 0.05, tools/goldens/tiny_model.py)."""

import numpy as np
import pytest

from oracle import oracle as O
from tests.conftest import cuda_available

pytestmark = pytest.mark.gpu

if cuda_available():
    from rosylnalive_b200 import executor as X
    from rosylnalive_b200 import qwen as Qw
    from rosylnalive_b200 import rope as R
    from rosylnalive_b200 import synthetic as S

# A Qwen3-shaped model small enough for the CPU oracle: head_dim 128, GQA 2, tied embeddings.
MINI = None
if cuda_available():
    MINI = X.QwenConfig(layers=3, hidden=256, heads=4, kv_heads=2, head_dim=128, intermediate=512, vocab=2048,
                        eps=1e-6, max_pos=512, rope_theta=1e6)


def cosine(a, b):
    a = np.asarray(a, np.float64).ravel()
    b = np.asarray(b, np.float64).ravel()
    return float(a @ b / (np.linalg.norm(a) * np.linalg.norm(b)))


@pytest.fixture(scope="module")
def mini():
    cfg = MINI
    weights = S.random_weights(cfg, seed=0)
    cos, sin = R.t_spec(R.torch_inv_freq_bits(cfg.rope_theta, cfg.head_dim), cfg.max_pos)
    oc = O.Config(cfg.layers, cfg.hidden, cfg.heads, cfg.kv_heads, cfg.head_dim, cfg.intermediate, cfg.vocab, cfg.eps,
                  cfg.max_pos)
    om = O.Model.from_hf(oc, weights, cos, sin)
    eng = Qw.QwenEngine(cfg, weights, cos, sin, max_seqs=8, max_tokens=1024, max_batch=8)
    yield cfg, om, eng
    eng.close()


def test_prefill_logits_match_oracle(mini):
    cfg, om, eng = mini
    prompts = [S.random_prompt(cfg.vocab, n, seed=i, stream=f"p{i}") for i, n in enumerate((70, 33, 1, 130))]
    nxt, logits = eng.prefill([0, 1, 2, 3], prompts, want_logits=True)
    for i, p in enumerate(prompts):
        ref = O.forward(om, O.Cache.new(om.config, "f32"), 0, p, "f32", logits_rows="last")[0]
        assert cosine(logits[i], ref) >= 0.9999, i
        assert np.max(np.abs(logits[i] - ref)) <= 2e-2, i
        top2 = np.sort(ref)[-2:]
        if top2[1] - top2[0] > 0.05:
            assert nxt[i] == int(np.argmax(ref))


def test_long_prefill_on_cta_pairs_matches_oracle(mini):
    # 1,200 prompt tokens: the prefill GEMMs (q/k/v with its norm/RoPE/KV epilogue, o_proj and down with the residual,
    # gate/up with SwiGLU) run on two-SM clusters from 1,024 rows on.
    cfg, om, _ = mini
    weights = S.random_weights(cfg, seed=0)
    cos, sin = R.t_spec(R.torch_inv_freq_bits(cfg.rope_theta, cfg.head_dim), cfg.max_pos)
    eng = Qw.QwenEngine(cfg, weights, cos, sin, max_seqs=4, max_tokens=2048, max_batch=4)
    try:
        lens = (500, 300, 257, 143)
        prompts = [S.random_prompt(cfg.vocab, n, seed=40 + i, stream=f"l{i}") for i, n in enumerate(lens)]
        nxt, logits = eng.prefill([0, 1, 2, 3], prompts, want_logits=True)
        for i, p in enumerate(prompts):
            ref = O.forward(om, O.Cache.new(om.config, "f32"), 0, p, "f32", logits_rows="last")[0]
            assert cosine(logits[i], ref) >= 0.9999, i
            assert np.max(np.abs(logits[i] - ref)) <= 2e-2, i
            top2 = np.sort(ref)[-2:]
            if top2[1] - top2[0] > 0.05:
                assert nxt[i] == int(np.argmax(ref))
    finally:
        eng.close()


def test_checkpoint_loader_matches_set_weight(mini, tmp_path):
    # The same weights through the library's safetensors loader: half of them in a BF16 file, half in an F32 file
    # (exact widenings of the same bf16 values, so the loader's round-to-nearest-even narrowing must give them back);
    # the prefill logits must be bit for bit those of the engine whose weights were set from arrays.
    from rosylnalive_b200 import safetensors as ST

    cfg, om, eng = mini
    weights = S.random_weights(cfg, seed=0)
    cos, sin = R.t_spec(R.torch_inv_freq_bits(cfg.rope_theta, cfg.head_dim), cfg.max_pos)
    names = sorted(weights)
    a, b = str(tmp_path / "a.safetensors"), str(tmp_path / "b.safetensors")
    ST.write(a, {n: ("BF16", weights[n]) for n in names[::2]}, {"format": "pt"})
    ST.write(b, {n: ("F32", (weights[n].astype(np.uint32) << 16).view(np.float32)) for n in names[1::2]})
    eng2 = Qw.QwenEngine(cfg, [a, b], cos, sin, max_seqs=8, max_tokens=1024, max_batch=8)
    try:
        prompts = [S.random_prompt(cfg.vocab, n, seed=50 + i, stream=f"ck{i}") for i, n in enumerate((37, 90))]
        n1, l1 = eng.prefill([0, 1], prompts, want_logits=True)
        n2, l2 = eng2.prefill([0, 1], prompts, want_logits=True)
        assert np.array_equal(n1, n2) and np.array_equal(l1, l2)
        # refused: a tensor that is not a weight of this model, and a checkpoint that misses weights
        c = str(tmp_path / "c.safetensors")
        ST.write(c, {"lm_head.weight": ("BF16", weights["model.embed_tokens.weight"])})
        with pytest.raises(ValueError):
            eng2.load_safetensors(c)
        with pytest.raises(ValueError):
            Qw.QwenEngine(cfg, [a], cos, sin, max_seqs=2, max_tokens=64, max_batch=2).close()
    finally:
        eng2.close()


def test_greedy_decode_matches_oracle(mini):
    cfg, om, eng = mini
    prompts = [S.random_prompt(cfg.vocab, n, seed=10 + i, stream=f"g{i}") for i, n in enumerate((16, 40, 5))]
    steps = 24
    ids, logits = eng.greedy(prompts, steps, slots=[5, 2, 7], want_logits=True)
    for i, p in enumerate(prompts):
        ref_ids, ref_logits = O.greedy(om, p, steps, "f32", return_logits=True)
        margins = np.diff(np.sort(ref_logits, axis=1)[:, -2:], axis=1)[:, 0]
        for s in range(steps):
            assert cosine(logits[i, s], ref_logits[s]) >= 0.9999, (i, s)
            assert np.max(np.abs(logits[i, s] - ref_logits[s])) <= 2e-2, (i, s)
        agree = ids[i] == ref_ids
        first_diff = int(np.argmin(agree)) if not agree.all() else steps
        # identical tokens up to the first step whose oracle margin is inside the bf16 error
        if first_diff < steps:
            assert margins[first_diff] < 2e-2, (i, first_diff, margins[first_diff])


def test_graph_replay_equals_eager_decode(mini):
    cfg, om, eng = mini
    prompts = [S.random_prompt(cfg.vocab, 20 + 3 * i, seed=20 + i, stream=f"r{i}") for i in range(4)]
    slots = [0, 1, 2, 3]
    first, _ = eng.prefill(slots, prompts)
    eager = [first]
    cur = first
    for _ in range(6):
        cur, _ = eng.decode(slots, cur)
        eager.append(cur)
    first2, _ = eng.prefill(slots, prompts)
    assert np.array_equal(first, first2)
    eng.capture(slots, first2)
    got = []
    for _ in range(6):
        eng.replay(1)
        got.append(eng.last_ids())
    for a, b in zip(eager[1:], got):
        assert np.array_equal(a, b)
    assert eng.seq_len(0) == len(prompts[0]) + 6


def test_replay_after_a_decode_of_other_slots(mini):
    """A captured step reads its rows' slots and previous next ids from the engine's buffers. A decode call on other
    slots replaces both, so a replay then is refused (not run on the other rows' ids); once the graph's own slots
    are decoded again, replays continue exactly as eager decoding does."""
    from rosylnalive_b200 import native as N

    cfg, om, eng = mini
    pa = [S.random_prompt(cfg.vocab, 12 + i, seed=60 + i, stream=f"ra{i}") for i in range(2)]
    pb = [S.random_prompt(cfg.vocab, 15 + i, seed=70 + i, stream=f"rb{i}") for i in range(2)]
    A, B = [4, 5], [6, 7]
    cur, _ = eng.prefill(A, pa)
    ref = [cur]
    for _ in range(3):
        cur, _ = eng.decode(A, cur)
        ref.append(cur)
    first_a, _ = eng.prefill(A, pa)
    first_b, _ = eng.prefill(B, pb)
    eng.capture(A, first_a)
    eng.replay(1)
    assert np.array_equal(eng.last_ids(), ref[1])
    eng.decode(B, first_b)
    with pytest.raises(N.GpuContractException):
        eng.replay(1)
    nxt, _ = eng.decode(A, ref[1])
    assert np.array_equal(nxt, ref[2])
    eng.replay(1)
    assert np.array_equal(eng.last_ids(), ref[3])
    assert eng.seq_len(4) == len(pa[0]) + 3


def test_decode_batch_invariance(mini):
    """A sequence decoded alone and inside a batch gives the same tokens (fixed split shapes per length)."""
    cfg, om, eng = mini
    p = S.random_prompt(cfg.vocab, 50, seed=30, stream="bi")
    others = [S.random_prompt(cfg.vocab, 9, seed=31 + i, stream=f"bo{i}") for i in range(3)]
    alone = eng.greedy([p], 8, slots=[0])
    batch = eng.greedy([p] + others, 8, slots=[0, 1, 2, 3])
    assert np.array_equal(alone[0], batch[0])


def test_decode_more_than_one_token_tile(mini):
    """A decode step of 100 sequences spans two 64-token tiles of every decode GEMM (and a 100-row prefill two CTA-pair
    row tiles): each row's logits equal, bit for bit, those of the same sequence decoded in a batch of four, and the
    first rows of each tile match the oracle within the bf16 bar."""
    cfg, om, _ = mini
    weights = S.random_weights(cfg, seed=0)
    cos, sin = R.t_spec(R.torch_inv_freq_bits(cfg.rope_theta, cfg.head_dim), cfg.max_pos)
    n = 100
    prompts = [S.random_prompt(cfg.vocab, 5 + i % 23, seed=400 + i, stream=f"t{i}") for i in range(n)]
    with Qw.QwenEngine(cfg, weights, cos, sin, max_seqs=n, max_tokens=4096, max_batch=n) as eng:
        ids, logits = eng.greedy(prompts, 3, want_logits=True)
        for group in ([0, 1, 63, 64], [65, 98, 99, 30]):
            g_ids, g_logits = eng.greedy([prompts[i] for i in group], 3, slots=list(range(4)), want_logits=True)
            for j, i in enumerate(group):
                assert np.array_equal(g_ids[j], ids[i]), i
                assert np.array_equal(g_logits[j].view(np.uint32), logits[i].view(np.uint32)), i
    for i in (0, 64, 99):
        ref_ids, ref_logits = O.greedy(om, prompts[i], 3, "f32", return_logits=True)
        for s in range(3):
            assert cosine(logits[i, s], ref_logits[s]) >= 0.9999, (i, s)
            assert np.max(np.abs(logits[i, s] - ref_logits[s])) <= 2e-2, (i, s)


def test_engine_rejects_bad_input(mini):
    cfg, om, eng = mini
    with pytest.raises(ValueError):
        eng.prefill([0], [np.array([cfg.vocab], np.uint32)])
    with pytest.raises(ValueError):
        eng.decode([0, 0], [1, 2])


def test_chunked_prefill_is_bit_identical_to_one_prefill(mini):
    """Prefill of first chunks, then extend calls with the rest (sequences at different cached lengths in one call,
    chunk sizes off the 16-token pages and 128-key tiles) gives one whole prefill's logits and decode bit for bit:
    attention reads the cached keys of earlier chunks, and every kernel computes a row the same way wherever the
    row sits in its call."""
    cfg, om, _ = mini
    weights = S.random_weights(cfg, seed=0)
    cos, sin = R.t_spec(R.torch_inv_freq_bits(cfg.rope_theta, cfg.head_dim), cfg.max_pos)
    eng = Qw.QwenEngine(cfg, weights, cos, sin, max_seqs=4, max_tokens=2048, max_batch=4)
    try:
        lens = (500, 333, 41)  # 874 rows; the chunks split A into 300 | 117 | 83 and B into 100 | 233
        p = [S.random_prompt(cfg.vocab, n, seed=80 + i, stream=f"c{i}") for i, n in enumerate(lens)]
        whole_ids, whole = eng.prefill([0, 1, 2], p, want_logits=True)
        whole_dec = [eng.decode([0, 1, 2], whole_ids, want_logits=True)[1] for _ in range(1)]
        ids1, lg1 = eng.prefill([0, 1, 2], [p[0][:300], p[1][:100], p[2]], want_logits=True)
        ids2, lg2 = eng.extend([0, 1], [p[0][300:417], p[1][100:]], want_logits=True)
        ids3, lg3 = eng.extend([0], [p[0][417:]], want_logits=True)
        assert eng.seq_len(0) == 500 and eng.seq_len(1) == 333 and eng.seq_len(2) == 41
        got = np.stack([lg3[0], lg2[1], lg1[2]])
        assert np.array_equal(got.view(np.uint32), whole.view(np.uint32))
        assert [ids3[0], ids2[1], ids1[2]] == list(whole_ids)
        dec = eng.decode([0, 1, 2], whole_ids, want_logits=True)[1]
        assert np.array_equal(dec.view(np.uint32), whole_dec[0].view(np.uint32))
    finally:
        eng.close()


def test_extend_after_decode_matches_oracle(mini):
    """A turn appended to a decoded sequence (prefill, greedy steps, then extend with new tokens) gives the oracle's
    logits for the whole sequence within the bf16 bar."""
    cfg, om, eng = mini
    prompt = S.random_prompt(cfg.vocab, 80, seed=90, stream="t0")
    turn = S.random_prompt(cfg.vocab, 40, seed=91, stream="t1")
    ids = eng.greedy([prompt], 6, slots=[3])[0]
    # the last greedy id was produced but not fed: the sequence holds the prompt and the first 5 ids
    _, logits = eng.extend([3], [np.concatenate([ids[-1:], turn]).astype(np.uint32)], want_logits=True)
    full = np.concatenate([prompt, ids, turn]).astype(np.int64)
    ref = O.forward(om, O.Cache.new(om.config, "f32"), 0, full, "f32", logits_rows="last")[0]
    assert cosine(logits[0], ref) >= 0.9999
    assert np.max(np.abs(logits[0] - ref)) <= 2e-2
    assert eng.seq_len(3) == len(full)


def test_extend_is_checked(mini):
    cfg, om, eng = mini
    eng.prefill([6], [S.random_prompt(cfg.vocab, 10, seed=92, stream="x")])
    with pytest.raises(ValueError):  # past max_pos
        eng.extend([6], [np.zeros(cfg.max_pos, np.uint32)])
    with pytest.raises(ValueError):  # a slot twice
        eng.extend([6, 6], [np.zeros(2, np.uint32), np.zeros(2, np.uint32)])
    assert eng.seq_len(6) == 10


def test_kept_graphs_serve_alternating_slot_sets(mini):
    """Two captured slot sets used in turn (as a pipeline's microbatches are): every call replays its own graph and
    gives eager decode's logits bit for bit."""
    cfg, om, eng = mini
    prompts = [S.random_prompt(cfg.vocab, 30 + 7 * i, seed=60 + i, stream=f"k{i}") for i in range(4)]
    a, b = [0, 1], [2, 3]

    def run(capture):
        first, _ = eng.prefill([0, 1, 2, 3], prompts)
        ids = {0: first[:2], 1: first[2:]}
        if capture:
            eng.capture(a)
            eng.capture(b)
        got = []
        for _ in range(3):
            for k, slots in ((0, a), (1, b)):
                nxt, lg = eng.decode(slots, ids[k], want_logits=True)
                ids[k] = nxt
                got.append(lg.copy())
        return np.stack(got)

    eager = run(False)
    graphs = run(True)
    assert np.array_equal(eager.view(np.uint32), graphs.view(np.uint32))
