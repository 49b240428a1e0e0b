"""The pipeline stage split of the forward (the reference's StagePipeline and QwenStageExecutor plan,
docs/dev-plan.md "C2a / C2b" and "StagePipeline": stage 0 runs embed plus layers 0-13, stage 1 layers 14-27 and the
head; the fp32 residual crosses the boundary; a stage that lost its KV cache rebuilds it by exact replay).

Two drivers over QwenEngine stages (QwenEngine(..., stage=(first, end))):

  * LocalPipeline: every stage in this process (on one GPU or several). Each call runs the stages in order and
    copies the residual rows between them (a peer copy over NVLink when the stages sit on different GPUs). It keeps
    each stage's input history, so rebuild(i, engine) replays it into a fresh engine: the same calls in the same
    order give the same KV cache bit for bit.
  * DistPipeline: one stage per rank of a torch.distributed group (one process per GPU, NCCL; gloo on CPU). Ranks
    pass the residual rows forward and the last stage's next ids back to rank 0 with point-to-point send/recv, and
    greedy() splits the sequences into microbatches so every stage works on one while the others work on the rest.

A split forward is bit-identical to the unsplit engine (the stages run the unsplit forward's kernels in its order),
which tests/test_gpu_pipeline.py checks for prefill, decode and the replayed rebuild.
"""

from __future__ import annotations

import numpy as np


def split_layers(layers: int, stages: int) -> list:
    """Contiguous layer ranges of near-equal size, earlier stages taking the extra layer: [(first, end), ...]. Two
    stages of Qwen3-0.6B's 28 layers give the reference's split, layers 0-13 and 14-27."""
    if not 1 <= stages <= layers:
        raise ValueError(f"{stages} stages for {layers} layers")
    base, extra = divmod(layers, stages)
    out, first = [], 0
    for i in range(stages):
        end = first + base + (1 if i < extra else 0)
        out.append((first, end))
        first = end
    return out


class LocalPipeline:
    """Stages in one process, run in order; see the module docstring."""

    def __init__(self, stages: list, keep_history: bool = True):
        if not stages or not stages[0].is_first or not stages[-1].is_last:
            raise ValueError("the stages must start with the first layer and end with the last")
        for a, b in zip(stages, stages[1:]):
            if a.end != b.first:
                raise ValueError(f"stage layers [{a.first}, {a.end}) and [{b.first}, {b.end}) do not meet")
        self.stages = list(stages)
        self.keep_history = keep_history
        # Per stage, the calls it ran: ("prefill", slots, lens, input) or ("decode", slots, input), where input is
        # the token ids (stage 0) or the residual rows it read (host copies).
        self.history = [[] for _ in stages]

    def _handoff(self, i: int, rows: int):
        """Copies the residual rows of stage i into stage i + 1 and returns the host copy kept for replay."""
        import torch

        src = self.stages[i].residual(rows)
        dst = self.stages[i + 1].residual(rows)
        torch.cuda.synchronize(src.device)
        dst.copy_(src)
        torch.cuda.synchronize(dst.device)
        return src.cpu() if self.keep_history else None

    def prefill(self, slots, prompts, want_logits=False):
        slots = np.asarray(slots, np.int32)
        lens = np.array([len(p) for p in prompts], np.int32)
        rows = int(lens.sum())
        inp = [np.asarray(p, np.uint32).copy() for p in prompts]
        out = (None, None)
        for i, st in enumerate(self.stages):
            if self.keep_history:
                self.history[i].append(("prefill", slots.copy(), lens.copy(), inp))
            out = st.prefill_stage(slots, lens, prompts if i == 0 else None, want_logits)
            if i + 1 < len(self.stages):
                inp = self._handoff(i, rows)
        return out

    def decode(self, slots, ids, want_logits=False):
        slots = np.asarray(slots, np.int32)
        inp = np.asarray(ids, np.uint32).copy()
        out = (None, None)
        for i, st in enumerate(self.stages):
            if self.keep_history:
                self.history[i].append(("decode", slots.copy(), inp))
            out = st.decode(slots, ids if i == 0 else None, want_logits)
            if i + 1 < len(self.stages):
                inp = self._handoff(i, len(slots))
        return out

    def greedy(self, prompts, steps: int, slots=None, want_logits=False):
        """QwenEngine.greedy through the stages."""
        n = len(prompts)
        slots = np.arange(n, dtype=np.int32) if slots is None else np.asarray(slots, np.int32)
        nxt, lg = self.prefill(slots, prompts, want_logits)
        ids, logs = [nxt.copy()], [lg]
        for _ in range(1, steps):
            nxt, lg = self.decode(slots, nxt, want_logits)
            ids.append(nxt.copy())
            logs.append(lg)
        ids = np.stack(ids, 1).astype(np.int64)
        return (ids, np.stack(logs, 1)) if want_logits else ids

    def rebuild(self, i: int, engine) -> None:
        """Replaces stage i with a fresh `engine` (same layers, weights loaded) and rebuilds its KV cache by exact
        replay of the calls stage i ran, fed with the inputs it read then."""
        import torch

        if not self.keep_history:
            raise RuntimeError("rebuild needs the pipeline's input history (keep_history=True)")
        old = self.stages[i]
        if (engine.first, engine.end) != (old.first, old.end):
            raise ValueError(f"the new engine holds layers [{engine.first}, {engine.end}), the stage [{old.first}, "
                             f"{old.end})")
        for call in self.history[i]:
            if call[0] == "prefill":
                _, slots, lens, inp = call
                if i > 0:
                    engine.residual(int(lens.sum())).copy_(inp.to(engine.residual(1).device))
                    torch.cuda.synchronize(engine.device)
                engine.prefill_stage(slots, lens, inp if i == 0 else None)
            else:
                _, slots, inp = call
                if i > 0:
                    engine.residual(len(slots)).copy_(inp.to(engine.residual(1).device))
                    torch.cuda.synchronize(engine.device)
                engine.decode(slots, inp if i == 0 else None)
        self.stages[i] = engine


class DistPipeline:
    """One stage per rank (rank r holds stage r of `world` stages); see the module docstring.

    `engine` is this rank's stage. Every rank calls greedy() with the same arguments; rank 0 returns the ids, the
    others None. Tensors travel with torch.distributed point-to-point calls on the default group (NCCL for CUDA
    engines, gloo for host ones); `device` is where the transfer buffers live.

    No order of the ranks' progress can deadlock: sends are non-blocking (isend); rank 0 takes a microbatch's ids
    from the last rank only right before it needs them for that microbatch's next step; and the residual rows
    (forward) and the ids (back) travel on two process groups. One communicator runs a rank's point-to-point calls
    in the order they were posted, so with a single group rank 0's queued residual sends would wait behind rank 1's
    ids send, which waits for rank 0's ids receive behind those sends, once a message is too large to go eagerly.
    Every rank constructs DistPipeline at the same point (the groups are created collectively)."""

    def __init__(self, engine, rank: int, world: int, device):
        self.engine, self.rank, self.world, self.device = engine, rank, world, device
        if engine.is_first != (rank == 0) or engine.is_last != (rank == world - 1):
            raise ValueError(f"rank {rank} of {world} holds layers [{engine.first}, {engine.end})")
        self._inflight = []
        self._fwd = self._back = None
        if world > 1:
            import torch.distributed as dist

            self._fwd = dist.new_group(list(range(world)))
            self._back = dist.new_group(list(range(world)))

    def _sync(self):
        import torch

        if str(self.device).startswith("cuda"):
            torch.cuda.synchronize(self.device)

    def _isend(self, t, dst, group):
        import torch.distributed as dist

        self._inflight = [(r, x) for r, x in self._inflight if not r.is_completed()]
        self._inflight.append((dist.isend(t, dst, group=group), t))  # the tensor stays alive until sent

    def _drain(self):
        for req, _ in self._inflight:
            req.wait()
        self._inflight.clear()

    def _run(self, kind, slots, lens, ids):
        """One call of this rank's stage on one microbatch: receive its residual rows (ranks after 0), run the stage,
        send the rows on (ranks before the last) or the next ids back to rank 0 (the last rank). Returns the next
        ids when this rank is both first and last."""
        import torch
        import torch.distributed as dist

        e = self.engine
        rows = int(np.sum(lens)) if kind == "prefill" else len(slots)
        if self.rank > 0:
            buf = torch.empty((rows, e.cfg.hidden), dtype=torch.float32, device=self.device)
            dist.recv(buf, self.rank - 1, group=self._fwd)
            self._sync()
            e.residual(rows).copy_(buf)
            self._sync()
        if kind == "prefill":
            nxt, _ = e.prefill_stage(slots, lens, ids if self.rank == 0 else None)
        else:
            nxt, _ = e.decode(slots, ids if self.rank == 0 else None)
        if not e.is_last:
            out = e.residual(rows).clone()
            self._sync()
            self._isend(out, self.rank + 1, self._fwd)
        elif self.world > 1:
            back = torch.from_numpy(nxt.astype(np.int64)).to(self.device)
            self._sync()
            self._isend(back, 0, self._back)
        return nxt

    def _ids_back(self, n):
        """Rank 0: the next ids of the oldest microbatch call whose ids it has not taken yet."""
        import torch
        import torch.distributed as dist

        buf = torch.empty(n, dtype=torch.int64, device=self.device)
        dist.recv(buf, self.world - 1, group=self._back)
        return buf.cpu().numpy().astype(np.uint32)

    @staticmethod
    def _groups(n, microbatches):
        return [g for g in np.array_split(np.arange(n, dtype=np.int32), max(1, microbatches)) if len(g)]

    def prefill(self, prompts, microbatches: int = 1):
        """Prefills `prompts` into slots 0..n-1 in `microbatches` groups (each stage runs group g while the next runs
        g-1). Rank 0 keeps each sequence's next id for decode_steps and returns them; the other ranks return None."""
        self._n = len(prompts)
        self._next = np.zeros(self._n, np.uint32)
        groups = self._groups(self._n, microbatches)
        for slots in groups:
            lens = np.array([len(prompts[s]) for s in slots], np.int32)
            toks = [np.asarray(prompts[s], np.uint32) for s in slots] if self.rank == 0 else None
            r = self._run("prefill", slots, lens, toks)
            if self.world == 1:
                self._next[slots] = r
        if self.rank == 0 and self.world > 1:
            for slots in groups:
                self._next[slots] = self._ids_back(len(slots))
        return self._next.copy() if self.rank == 0 else None

    def decode_steps(self, steps: int, microbatches: int = 2):
        """`steps` greedy decode steps of every prefilled sequence, in `microbatches` groups: rank 0 feeds group g's
        step s with the ids of its step s - 1 as soon as the last rank sends them, so the stages overlap. Returns ids
        [n, steps] on rank 0, None elsewhere."""
        groups = self._groups(self._n, microbatches)
        out = np.zeros((self._n, steps), np.int64) if self.rank == 0 else None
        for s in range(steps):
            for slots in groups:
                ids = None
                if self.rank == 0:
                    ids = self._next[slots] if (s == 0 or self.world == 1) else self._ids_back(len(slots))
                    if s > 0 and self.world > 1:
                        out[slots, s - 1] = ids
                        self._next[slots] = ids
                r = self._run("decode", slots, None, ids)
                if self.world == 1:
                    self._next[slots] = r
                    out[slots, s] = r
        if self.rank == 0 and self.world > 1 and steps > 0:
            for slots in groups:
                self._next[slots] = self._ids_back(len(slots))
                out[slots, steps - 1] = self._next[slots]
        self._drain()
        return out

    def greedy(self, prompts, steps: int, microbatches: int = 2):
        """QwenEngine.greedy through the pipeline: prefill, then steps - 1 decode steps, sequences in
        `microbatches` groups. Returns ids [n, steps] on rank 0, None elsewhere."""
        first = self.prefill(prompts, microbatches)
        rest = self.decode_steps(steps - 1, microbatches) if steps > 1 else None
        self._drain()
        if self.rank != 0:
            return None
        cols = [first.astype(np.int64)[:, None]] + ([rest] if rest is not None else [])
        return np.concatenate(cols, 1)
