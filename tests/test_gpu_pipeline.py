"""The pipeline stage split on the GPU (QwenEngine stages, rosylnalive_b200.pipeline): a model split into stages gives
the unsplit engine's ids and logits bit for bit, in prefill (on CTA pairs from 1,024 rows) and decode; stages load
their own weights from a whole checkpoint; a stage replaced by a fresh engine and rebuilt by exact replay continues
bit-identically; and with two GPUs, DistPipeline over NCCL (one process per GPU) gives the unsplit ids."""

import multiprocessing as mp
import os
import socket
import sys
import time

import numpy as np
import pytest

from tests.conftest import cuda_available

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

if cuda_available():
    from rosylnalive_b200 import executor as X
    from rosylnalive_b200 import pipeline as PL
    from rosylnalive_b200 import qwen as Qw
    from rosylnalive_b200 import rope as R
    from rosylnalive_b200 import synthetic as S

    CFG = X.QwenConfig(layers=4, hidden=256, heads=4, kv_heads=2, head_dim=128, intermediate=512, vocab=2048,
                       eps=1e-6, max_pos=1024, rope_theta=1e6)


def _model():
    weights = S.random_weights(CFG, seed=3)
    cos, sin = R.t_spec(R.torch_inv_freq_bits(CFG.rope_theta, CFG.head_dim), CFG.max_pos)
    return weights, cos, sin


def _engine(weights, cos, sin, stage=None, device=0):
    return Qw.QwenEngine(CFG, weights, cos, sin, device=device, max_seqs=8, max_tokens=2048, max_batch=8,
                         stage=stage)


PROMPT_LENS = (600, 257, 130, 77)  # 1,064 rows: the prefill GEMMs run on CTA pairs
STEPS = 8


def _prompts():
    return [S.random_prompt(CFG.vocab, n, seed=70 + i, stream=f"pp{i}") for i, n in enumerate(PROMPT_LENS)]


@pytest.fixture(scope="module")
def unsplit():
    weights, cos, sin = _model()
    eng = _engine(weights, cos, sin)
    try:
        ids, logits = eng.greedy(_prompts(), STEPS, want_logits=True)
    finally:
        eng.close()
    return ids, logits


@pytest.mark.parametrize("split", [[(0, 2), (2, 4)], [(0, 1), (1, 3), (3, 4)]], ids=["2 stages", "3 stages"])
def test_split_forward_is_bit_identical(unsplit, split):
    weights, cos, sin = _model()
    stages = [_engine(weights, cos, sin, stage=s) for s in split]
    try:
        ids, logits = PL.LocalPipeline(stages, keep_history=False).greedy(_prompts(), STEPS, want_logits=True)
    finally:
        for s in stages:
            s.close()
    assert np.array_equal(ids, unsplit[0])
    assert np.array_equal(logits.view(np.uint32), unsplit[1].view(np.uint32))


def test_stages_load_their_weights_from_one_checkpoint(unsplit, tmp_path):
    from rosylnalive_b200 import safetensors as ST

    weights, cos, sin = _model()
    path = tmp_path / "model.safetensors"
    ST.write(str(path), {k: ("BF16", v) for k, v in weights.items()})
    stages = [_engine(str(path), cos, sin, stage=s) for s in [(0, 2), (2, 4)]]
    try:
        ids, logits = PL.LocalPipeline(stages, keep_history=False).greedy(_prompts(), STEPS, want_logits=True)
    finally:
        for s in stages:
            s.close()
    assert np.array_equal(ids, unsplit[0])
    assert np.array_equal(logits.view(np.uint32), unsplit[1].view(np.uint32))


def test_stage_rebuilt_by_exact_replay_continues_bit_identically(unsplit):
    weights, cos, sin = _model()
    stages = [_engine(weights, cos, sin, stage=s) for s in [(0, 2), (2, 4)]]
    pipe = PL.LocalPipeline(stages)
    fresh = None
    try:
        prompts = _prompts()
        slots = np.arange(len(prompts), dtype=np.int32)
        nxt, lg = pipe.prefill(slots, prompts, want_logits=True)
        ids, logs = [nxt.copy()], [lg]
        for step in range(1, STEPS):
            if step == 4:  # stage 1 loses its state: a fresh engine replays what it ran
                old = pipe.stages[1]
                fresh = _engine(weights, cos, sin, stage=(2, 4))
                old.close()
                pipe.rebuild(1, fresh)
            nxt, lg = pipe.decode(slots, nxt, want_logits=True)
            ids.append(nxt.copy())
            logs.append(lg)
    finally:
        for s in pipe.stages:
            s.close()
    assert np.array_equal(np.stack(ids, 1), unsplit[0])
    assert np.array_equal(np.stack(logs, 1).view(np.uint32), unsplit[1].view(np.uint32))


def test_stage_arguments_are_checked():
    weights, cos, sin = _model()
    for bad in [(2, 2), (3, 2), (0, 5), (-1, 2)]:
        with pytest.raises(ValueError):
            _engine(weights, cos, sin, stage=bad)
    last = _engine(weights, cos, sin, stage=(2, 4))
    try:
        assert (last.first, last.end, last.is_first, last.is_last) == (2, 4, False, True)
        assert tuple(last.residual().shape) == (2048, CFG.hidden)
        from rosylnalive_b200 import native as N

        slots, lens = np.zeros(1, np.int32), np.ones(1, np.int32)
        with pytest.raises(ValueError):  # the last stage needs somewhere to put the next ids
            N.check(N.lib().lrm_qwen_prefill(last._h, 1, Qw._p(slots, Qw.I32), Qw._p(lens, Qw.I32), None, None,
                                             None), None, "prefill")
    finally:
        last.close()


# ---- two GPUs: one process per stage, NCCL ----------------------------------------------------------------------------

def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _nccl_rank(rank, world, port, q):
    os.environ.update({"MASTER_ADDR": "127.0.0.1", "MASTER_PORT": str(port), "NCCL_NVLS_ENABLE": "0"})
    sys.path.insert(0, ROOT)
    import datetime

    import torch
    import torch.distributed as dist

    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120),
                            device_id=torch.device("cuda", rank))
    eng = None
    try:
        weights, cos, sin = _model()
        eng = _engine(weights, cos, sin, stage=PL.split_layers(CFG.layers, world)[rank], device=rank)
        ids = PL.DistPipeline(eng, rank, world, f"cuda:{rank}").greedy(_prompts(), STEPS, microbatches=2)
        q.put((rank, "ok", None if ids is None else ids.tolist()))
    except Exception as e:  # noqa: BLE001
        q.put((rank, "error", repr(e)))
    finally:
        if eng is not None:
            eng.close()
        dist.destroy_process_group()


@pytest.mark.skipif(not cuda_available() or __import__("torch").cuda.device_count() < 2, reason="needs two GPUs")
def test_dist_pipeline_on_two_gpus_equals_unsplit(unsplit):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_nccl_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    out, deadline = {}, time.time() + 300
    while len(out) < 2 and time.time() < deadline:
        try:
            r, status, val = q.get(timeout=1)
            out[r] = (status, val)
        except Exception:  # noqa: BLE001
            pass
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    assert out.get(0, ("missing",))[0] == "ok" and out.get(1, ("missing",))[0] == "ok", out
    assert np.array_equal(np.array(out[0][1]), unsplit[0])
