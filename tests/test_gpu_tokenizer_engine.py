"""Text in, text out (GPU tier): the tokenizer at both ends of the bf16 forward path.

The toy tokenizer (the reference's toy model, ToyTests.fs:17-110: 256 byte tokens, 7 merges, 3 added tokens; built in
tests/test_tokenizer.py) encodes a prompt; the ids go through the bf16 engine's greedy schedule on a small
Qwen3-shaped model with the tokenizer's vocabulary (266 ids); the generated ids are decoded back to text. Checked:
the prompt's ids round-trip through decode/encode; the engine's greedy ids equal the CPU reference's (the oracle,
fp32) for every step up to the first whose oracle top-2 margin is inside the bf16 logit error; and the generated
text equals the text of the oracle's ids over those steps."""

import numpy as np
import pytest

from oracle import oracle as O
from tests.conftest import cuda_available
from tests.test_tokenizer import toy

pytestmark = pytest.mark.gpu

if cuda_available():
    from rosylnalive_b200 import executor as X
    from rosylnalive_b200 import qwen as Qw
    from rosylnalive_b200 import rope as R
    from rosylnalive_b200 import synthetic as S

TEXT = "the cat aab <|a|> then bc the aaaa <|ab|> déjà vu, the end"
STEPS = 16


def test_tokenizer_engine_detokenizer_round_trip():
    tok = toy()
    ids = np.array(tok.encode(TEXT), np.uint32)
    assert tok.decode(ids.tolist()) == TEXT
    assert tok.encode(tok.decode(ids.tolist())) == ids.tolist()
    cfg = X.QwenConfig(layers=2, hidden=256, heads=4, kv_heads=2, head_dim=128, intermediate=512,
                       vocab=tok.vocab_size, eps=1e-6, max_pos=128, rope_theta=1e6)
    weights = S.random_weights(cfg, seed=6)  # every oracle margin >= 0.2
    cos, sin = R.t_spec(R.torch_inv_freq_bits(cfg.rope_theta, cfg.head_dim), cfg.max_pos)
    with Qw.QwenEngine(cfg, weights, cos, sin, max_seqs=1, max_tokens=128, max_batch=1) as eng:
        got = eng.greedy([ids], STEPS)[0]
    oc = O.Config(cfg.layers, cfg.hidden, cfg.heads, cfg.kv_heads, cfg.head_dim, cfg.intermediate, cfg.vocab, cfg.eps,
                  cfg.max_pos)
    ref, ref_logits = O.greedy(O.Model.from_hf(oc, weights, cos, sin), ids, STEPS, "f32", return_logits=True)
    part = np.partition(ref_logits, -2, axis=1)
    decided = (part[:, -1] - part[:, -2]) > 2 * 2e-2
    n = int(np.argmin(decided)) if not decided.all() else STEPS
    assert n >= 4, (n, part[:, -1] - part[:, -2])
    assert np.array_equal(got[:n], ref[:n]), (got, ref)
    assert tok.decode(got[:n].tolist()) == tok.decode(ref[:n].tolist())
    text = tok.decode(got.tolist())  # every id of the vocabulary decodes (errors=replace for partial UTF-8)
    assert isinstance(text, str) and len(text) > 0
    print(f"prompt {len(ids)} ids -> generated {got.tolist()} = {text!r} ({n} steps checked against the oracle)")
