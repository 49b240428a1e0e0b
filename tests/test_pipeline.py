"""The pipeline stage split's host logic on CPU (rosylnalive_b200.pipeline): the layer split, and DistPipeline's
microbatched schedule over gloo ranks (world sizes 2 and 3), checked against the same stages run one after another
in one process. A stage here is a deterministic host stand-in with QwenEngine's stage interface and a per-slot state
that every call advances (as a KV cache does), so a schedule that reorders, drops or repeats a call gives other ids.
The CUDA stages are checked in tests/test_gpu_pipeline.py."""

import multiprocessing as mp
import os
import socket
import sys
import time

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

from rosylnalive_b200 import pipeline as PL  # noqa: E402

HIDDEN, VOCAB, LAYERS, SLOTS = 8, 97, 6, 8


class _Cfg:
    hidden, vocab, layers = HIDDEN, VOCAB, LAYERS


class FakeStage:
    """Layers [first, end) of a toy model with QwenEngine's stage interface (prefill_stage, decode, residual)."""

    def __init__(self, first, end):
        import torch

        self.cfg = _Cfg()
        self.first, self.end = first, end
        self.is_first, self.is_last = first == 0, end == LAYERS
        self.device = "cpu"
        self.x = torch.zeros((256, HIDDEN), dtype=torch.float32)
        self.state = np.zeros((LAYERS, SLOTS, HIDDEN), np.float32)  # per layer, as a KV cache
        self.calls = 0

    def residual(self, rows=None):
        return self.x if rows is None else self.x[:rows]

    def _layers(self, rows, row_slots):
        x = self.x[:rows].numpy().copy()
        f = np.float32
        for layer in range(self.first, self.end):
            st = self.state[layer]
            for r in range(rows):
                s = row_slots[r]
                st[s] = np.fmod(st[s] * f(0.5) + x[r] + f(layer), f(1000.0))
                x[r] = np.fmod(x[r] * f(1.25) + st[s] + f(0.125 * (layer + 1)), f(1000.0))
        self.x[:rows] = __import__("torch").from_numpy(x)

    def _embed(self, ids):
        import torch

        ids = np.asarray(ids, np.int64)
        e = (ids[:, None] * (np.arange(HIDDEN)[None, :] + 3)) % 13
        self.x[:len(ids)] = torch.from_numpy(e.astype(np.float32))

    def _head(self, rows, last_rows):
        x = self.x[:rows].numpy().astype(np.float64)
        return np.array([int(abs(x[r].sum()) * 7) % VOCAB for r in last_rows], np.uint32)  # order-fixed sum

    def prefill_stage(self, slots, lens, prompts=None, want_logits=False):
        self.calls += 1
        lens = np.asarray(lens)
        rows = int(lens.sum())
        row_slots = np.repeat(np.asarray(slots), lens)
        for s in slots:
            self.state[:, s] = 0.0
        if self.is_first:
            self._embed(np.concatenate([np.asarray(p) for p in prompts]))
        self._layers(rows, row_slots)
        if self.is_last:
            return self._head(rows, np.cumsum(lens) - 1), None
        return None, None

    def decode(self, slots, ids=None, want_logits=False):
        self.calls += 1
        if self.is_first:
            self._embed(ids)
        self._layers(len(slots), np.asarray(slots))
        if self.is_last:
            return self._head(len(slots), np.arange(len(slots))), None
        return None, None


def sequential(prompts, steps, stages):
    """The stages run one after another in one process: the reference for DistPipeline."""
    fakes = [FakeStage(a, b) for a, b in PL.split_layers(LAYERS, stages)]
    slots = np.arange(len(prompts))

    def through(kind, *args):
        out = None
        for i, f in enumerate(fakes):
            if i > 0:
                fakes[i].x[:] = fakes[i - 1].x
            out = f.prefill_stage(*args) if kind == "prefill" else f.decode(*args)
        return out[0]

    nxt = through("prefill", slots, [len(p) for p in prompts], prompts)
    ids = [nxt]
    for _ in range(1, steps):
        nxt = through("decode", slots, nxt)
        ids.append(nxt)
    return np.stack(ids, 1).astype(np.int64)


def free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


PROMPTS = [[(7 * i + 3 * k) % VOCAB for k in range(3 + i)] for i in range(6)]


class FailingStage(FakeStage):
    """A stage whose host raises on its `fail_at`-th call (a stage process that dies between ticks)."""

    def __init__(self, first, end, fail_at):
        super().__init__(first, end)
        self.fail_at = fail_at

    def _check(self):
        if self.calls + 1 == self.fail_at:
            raise RuntimeError(f"stage [{self.first}, {self.end}) failed at call {self.fail_at}")

    def prefill_stage(self, *args, **kw):
        self._check()
        return super().prefill_stage(*args, **kw)

    def decode(self, *args, **kw):
        self._check()
        return super().decode(*args, **kw)


def _rank_main(rank, world, port, steps, microbatches, q, fail=None):
    os.environ.update({"MASTER_ADDR": "127.0.0.1", "MASTER_PORT": str(port)})
    sys.path.insert(0, ROOT)
    import datetime

    import torch.distributed as dist

    timeout = datetime.timedelta(seconds=5 if fail else 60)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timeout)
    try:
        first, end = PL.split_layers(LAYERS, world)[rank]
        eng = FailingStage(first, end, fail[1]) if fail and fail[0] == rank else FakeStage(first, end)
        pipe = PL.DistPipeline(eng, rank, world, "cpu")
        ids = pipe.greedy(PROMPTS, steps, microbatches)
        q.put((rank, "ok", None if ids is None else ids.tolist(), eng.calls))
    except Exception as e:  # noqa: BLE001
        q.put((rank, "error", repr(e), 0))
    finally:
        dist.destroy_process_group()


def run_pipeline(world, steps, microbatches, timeout=120, fail=None):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, steps, microbatches, q, fail))
             for r in range(world)]
    for p in procs:
        p.start()
    out = {}
    deadline = time.time() + timeout
    while len(out) < world and time.time() < deadline:
        try:
            r, status, val, calls = q.get(timeout=1)
            out[r] = (status, val, calls)
        except Exception:  # noqa: BLE001
            pass
    for p in procs:
        p.join(timeout=30)
        if p.is_alive():
            p.kill()
    return out


def test_split_layers():
    assert PL.split_layers(28, 2) == [(0, 14), (14, 28)]
    assert PL.split_layers(28, 3) == [(0, 10), (10, 19), (19, 28)]
    assert PL.split_layers(5, 5) == [(i, i + 1) for i in range(5)]
    with pytest.raises(ValueError):
        PL.split_layers(4, 5)


def test_sequential_reference_depends_on_history():
    a = sequential(PROMPTS, 5, 2)
    b = sequential(PROMPTS, 5, 3)
    assert (a == b).all()  # the toy model does not depend on where it is split
    assert len({tuple(r) for r in a}) > 1


@pytest.mark.parametrize("world,microbatches", [(2, 1), (2, 2), (3, 2), (3, 3)])
def test_dist_pipeline_equals_sequential_stages(world, microbatches):
    steps = 5
    out = run_pipeline(world, steps, microbatches)
    assert sorted(out) == list(range(world)), out
    for r in range(world):
        assert out[r][0] == "ok", out[r]
    groups = len([g for g in np.array_split(np.arange(len(PROMPTS)), microbatches) if len(g)])
    for r in range(world):
        assert out[r][2] == groups * steps  # one call per microbatch and step on every stage
    assert np.array_equal(np.array(out[0][1]), sequential(PROMPTS, steps, world))
    for r in range(1, world):
        assert out[r][1] is None


def test_dist_pipeline_single_rank():
    import torch.distributed as dist

    eng = FakeStage(0, LAYERS)
    pipe = PL.DistPipeline(eng, 0, 1, "cpu")
    assert not dist.is_initialized()
    assert np.array_equal(pipe.greedy(PROMPTS, 4, 2), sequential(PROMPTS, 4, 1))


def test_dist_pipeline_rejects_a_stage_on_the_wrong_rank():
    with pytest.raises(ValueError):
        PL.DistPipeline(FakeStage(0, 3), 1, 2, "cpu")
    with pytest.raises(ValueError):
        PL.DistPipeline(FakeStage(3, LAYERS), 0, 2, "cpu")


@pytest.mark.parametrize("fail_rank", [0, 1])
def test_a_failing_stage_ends_the_other_ranks_with_an_error(fail_rank):
    """A stage that raises between ticks (its process then leaves) makes the other rank's next exchange fail on the
    host (peer gone, or the 5 s process-group timeout) instead of hanging; no rank returns ids."""
    t0 = time.time()
    out = run_pipeline(2, 5, 2, timeout=90, fail=(fail_rank, 3))
    assert time.time() - t0 < 90
    assert sorted(out) == [0, 1], out
    assert out[fail_rank][0] == "error" and "failed at call 3" in out[fail_rank][1], out
    other = 1 - fail_rank
    assert out[other][0] == "error", out
