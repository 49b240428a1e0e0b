"""The pipeline stage split of the forward (the reference's StagePipeline and QwenStageExecutor plan,
docs/dev-plan.md "C2a / C2b" and "StagePipeline": stage 0 runs embed plus layers 0-13, stage 1 layers 14-27 and the
head; the fp32 residual crosses the boundary; a stage that lost its KV cache rebuilds it by exact replay).

Two drivers over QwenEngine stages (QwenEngine(..., stage=(first, end))):

  * LocalPipeline: every stage in this process (on one GPU or several). Each call runs the stages in order and
    copies the residual rows between them (a peer copy over NVLink when the stages sit on different GPUs). It keeps
    each stage's input history, so rebuild(i, engine) replays it into a fresh engine: the same calls in the same
    order give the same KV cache bit for bit.
  * DistPipeline: one stage per rank of a torch.distributed group (one process per GPU, NCCL; gloo on CPU). Ranks
    pass the residual rows forward and the last stage's next ids back to rank 0 with point-to-point transfers
    between lockstep ticks, and the sequences run in microbatch groups so the stages work on different groups at
    once.

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

    `engine` is this rank's stage. Every rank makes the same calls with the same arguments; rank 0 returns the ids,
    the others None. Tensors travel with torch.distributed point-to-point calls on the default group (NCCL for CUDA
    engines, gloo for host ones); `device` is where the transfer buffers live.

    The ranks run in lockstep ticks: at tick t, stage r runs call k of sequence group g when
    t = k * max(M, W) + g + r (M groups, W stages), so a group's call moves one stage a tick and its next call
    starts on stage 0 after the last stage has returned the ids it needs. Between ticks every rank posts all its
    sends and receives of that exchange at once (batch_isend_irecv) and waits for them: residual rows to the next
    stage, and the last stage's next ids to rank 0. No transfer is in flight while a stage computes. This matters:
    a communication kernel waiting for its peer holds SMs, and the engine's persistent GEMMs size their grids to
    every SM, so a transfer left waiting across a compute call (the last stage's ids send, with rank 0 still busy
    prefilling) stalled that GPU's GEMM, and with it the peer's transfer: the two ranks hung."""

    def __init__(self, engine, rank: int, world: int, device):
        self.engine, self.rank, self.world, self.device = engine, rank, world, device
        if engine.is_first != (rank == 0) or engine.is_last != (rank == world - 1):
            raise ValueError(f"rank {rank} of {world} holds layers [{engine.first}, {engine.end})")
        self._n = 0
        self._next = np.zeros(0, np.uint32)
        self._captured = set()
        if world > 1:
            import torch.distributed as dist

            dist.barrier()  # every rank's communicator is up before the first point-to-point batch

    def _sync(self):
        import torch

        if str(self.device).startswith("cuda"):
            torch.cuda.synchronize(self.device)

    @staticmethod
    def _groups(n, microbatches):
        return [g for g in np.array_split(np.arange(n, dtype=np.int32), max(1, microbatches)) if len(g)]

    def _execute(self, groups, kinds, lens=None, toks=None):
        """Runs calls kinds[0], kinds[1], ... ("prefill" / "decode") for every sequence group through the stages in
        lockstep ticks. lens[g] are group g's prompt lengths and toks[g] its prompts (rank 0) for a prefill; a
        decode call of group g takes self._next[groups[g]] on rank 0. Rank 0 returns out[g][k], the next ids of
        group g's call k, and keeps the latest in self._next."""
        import torch
        import torch.distributed as dist

        W, M, C = self.world, len(groups), len(kinds)
        Mp = max(M, W)
        e = self.engine

        def task(r, t):
            u = t - r
            if r < 0 or r >= W or u < 0:
                return None
            k, g = divmod(u, Mp)
            return (g, k) if g < M and k < C else None

        def rows_of(g, k):
            return int(np.sum(lens[g])) if kinds[k] == "prefill" else len(groups[g])

        out = [[None] * C for _ in range(M)]
        inbox = None
        for t in range((C - 1) * Mp + (M - 1) + (W - 1) + 1):
            mine = task(self.rank, t)
            nxt = None
            if mine is not None:
                g, k = mine
                slots = groups[g]
                if self.rank > 0:
                    e.residual(inbox.shape[0]).copy_(inbox)
                    self._sync()
                if kinds[k] == "prefill":
                    nxt, _ = e.prefill_stage(slots, lens[g], toks[g] if self.rank == 0 else None)
                else:
                    nxt, _ = e.decode(slots, self._next[slots] if self.rank == 0 else None)
                if W == 1:
                    self._next[slots] = nxt
                    out[g][k] = nxt.copy()
            if W == 1:
                continue
            # the exchange after tick t: all of this rank's sends and receives, posted together
            ops, keep, idbuf, got = [], [], None, None
            if mine is not None and self.rank < W - 1:
                rows = e.residual(rows_of(*mine)).clone()
                keep.append(rows)
                ops.append(dist.P2POp(dist.isend, rows, self.rank + 1))
            if mine is not None and self.rank == W - 1:
                ids = torch.from_numpy(nxt.astype(np.int64)).to(self.device)
                keep.append(ids)
                ops.append(dist.P2POp(dist.isend, ids, 0))
            prev = task(self.rank - 1, t)
            if prev is not None:
                inbox = torch.empty((rows_of(*prev), e.cfg.hidden), dtype=torch.float32, device=self.device)
                ops.append(dist.P2POp(dist.irecv, inbox, self.rank - 1))
            if self.rank == 0:
                got = task(W - 1, t)
                if got is not None:
                    idbuf = torch.empty(len(groups[got[0]]), dtype=torch.int64, device=self.device)
                    ops.append(dist.P2POp(dist.irecv, idbuf, W - 1))
            if ops:
                self._sync()
                for req in dist.batch_isend_irecv(ops):
                    req.wait()
                self._sync()
            if got is not None:
                g, k = got
                ids = idbuf.cpu().numpy().astype(np.uint32)
                self._next[groups[g]] = ids
                out[g][k] = ids
        return out if self.rank == 0 else None

    def prefill(self, prompts, microbatches: int = 1):
        """Prefills `prompts` into slots 0..n-1 in `microbatches` groups (each stage runs group g while the next runs
        g-1). Rank 0 keeps each sequence's next id for decode_steps and returns them; the other ranks return None."""
        self._n = len(prompts)
        self._next = np.zeros(self._n, np.uint32)
        groups = self._groups(self._n, microbatches)
        lens = [np.array([len(prompts[s]) for s in slots], np.int32) for slots in groups]
        toks = [[np.asarray(prompts[s], np.uint32) for s in slots] for slots in groups] if self.rank == 0 else None
        self._execute(groups, ["prefill"], lens, toks)
        return self._next.copy() if self.rank == 0 else None

    def decode_steps(self, steps: int, microbatches: int = 2):
        """`steps` greedy decode steps of every prefilled sequence, in `microbatches` groups (the stages work on
        different groups at once once there are at least as many groups as stages). Returns ids [n, steps] on rank
        0, None elsewhere."""
        groups = self._groups(self._n, microbatches)
        if steps < 1:
            return np.zeros((self._n, 0), np.int64) if self.rank == 0 else None
        if hasattr(self.engine, "capture"):  # one decode graph per group, replayed by the engine's decode calls
            for slots in groups:
                key = tuple(int(x) for x in slots)
                if key not in self._captured:
                    self.engine.capture(slots)
                    self._captured.add(key)
        out = self._execute(groups, ["decode"] * steps)
        if self.rank != 0:
            return None
        ids = np.zeros((self._n, steps), np.int64)
        for g, slots in enumerate(groups):
            ids[slots] = np.stack(out[g], 1)
        return ids

    def greedy(self, prompts, steps: int, microbatches: int = 2):
        """QwenEngine.greedy through the pipeline: prefill, then steps - 1 decode steps, sequences in
        `microbatches` groups. Returns ids [n, steps] on rank 0, None elsewhere."""
        first = self.prefill(prompts, microbatches)
        rest = self.decode_steps(steps - 1, microbatches) if steps > 1 else None
        if self.rank != 0:
            return None
        cols = [first.astype(np.int64)[:, None]] + ([rest] if rest is not None else [])
        return np.concatenate(cols, 1)
