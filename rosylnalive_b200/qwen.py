"""The bf16 Qwen3 engine (liblrmcuda.so lrm_qwen_*), the fast path of the forward.

The reference plans this layer as Lrm.Gpu.Exec / Lrm.Models.Qwen (docs/dev-plan.md, "GpuForwardOps", "Greedy.run");
both are placeholders there. QwenEngine runs the same schedule as tests/Lrm.Tensor.Tests/TinyModel.fs:144-236 --
one prefill, then single-token greedy steps, argmax of the last row -- for many sequences at once, with bf16
weights/activations, an fp32 residual stream and a paged bf16 KV cache.
"""

from __future__ import annotations

import ctypes

import numpy as np

from . import native as N
from .executor import QwenConfig, weight_shapes

P, I32, U32, U64, F32 = ctypes.c_void_p, ctypes.c_int32, ctypes.c_uint32, ctypes.c_uint64, ctypes.c_float


class QwenConfigC(ctypes.Structure):
    _fields_ = [("layers", I32), ("hidden", I32), ("q_heads", I32), ("kv_heads", I32), ("head_dim", I32),
                ("intermediate", I32), ("vocab", I32), ("eps", F32), ("max_pos", I32), ("max_seqs", I32),
                ("kv_pages", I32), ("max_tokens", I32), ("max_batch", I32)]


PI32, PU32, PF32, PU16 = (ctypes.POINTER(t) for t in (I32, U32, F32, ctypes.c_uint16))

N.extra_signatures({
    "lrm_qwen_create": [I32, ctypes.POINTER(QwenConfigC), ctypes.POINTER(P)],
    "lrm_qwen_create_stage": [I32, ctypes.POINTER(QwenConfigC), I32, I32, ctypes.POINTER(P)],
    "lrm_qwen_stage": [P, PI32, PI32],
    "lrm_qwen_residual": [P, ctypes.POINTER(P), ctypes.POINTER(ctypes.c_int64)],
    "lrm_qwen_destroy": [P],
    "lrm_qwen_set_weight": [P, ctypes.c_char_p, PU16, U64],
    "lrm_qwen_set_rope": [P, PF32, PF32, I32, I32],
    "lrm_qwen_reset_seq": [P, I32],
    "lrm_qwen_reserve": [P, I32, I32],
    "lrm_qwen_prefill": [P, I32, PI32, PI32, PU32, PU32, PF32],
    "lrm_qwen_extend": [P, I32, PI32, PI32, PU32, PU32, PF32],
    "lrm_qwen_decode": [P, I32, PI32, PU32, PU32, PF32],
    "lrm_qwen_decode_graph": [P, I32, PI32, PU32, U32],
    "lrm_qwen_graph_kernels": [P, PI32],
    "lrm_qwen_attention_ms": [P, PF32],
    "lrm_qwen_truncate": [P, I32, I32],
    "lrm_qwen_decode_replay": [P, I32],
    "lrm_qwen_last_ids": [P, PU32],
    "lrm_qwen_sync": [P],
    "lrm_qwen_stream": [P, ctypes.POINTER(P)],
    "lrm_qwen_seq_len": [P, I32, PI32],
    "lrm_qwen_load_safetensors": [P, ctypes.c_char_p, PI32],
})


def _p(a: np.ndarray, t):
    return a.ctypes.data_as(ctypes.POINTER(t))


def stage_weight_names(cfg: QwenConfig, first: int, end: int) -> list:
    """The HF weight names a stage holding layers [first, end) loads: its layers' weights, the embedding on the first
    stage (gather table) and the last (tied head), the final norm on the last."""
    names = []
    for name in weight_shapes(cfg):
        if name.startswith("model.layers."):
            if first <= int(name.split(".")[2]) < end:
                names.append(name)
        elif name == "model.embed_tokens.weight":
            if first == 0 or end == cfg.layers:
                names.append(name)
        elif end == cfg.layers:
            names.append(name)
    return names


class _CudaArray:
    """A device buffer described by __cuda_array_interface__ (v3), so torch.as_tensor can view it without a copy."""

    def __init__(self, ptr: int, shape: tuple, typestr: str):
        self.__cuda_array_interface__ = {"shape": shape, "typestr": typestr, "data": (ptr, False), "version": 3,
                                         "strides": None, "stream": None}


class QwenEngine:
    """One device's Qwen3 engine. `weights` maps HF names to bf16 bit arrays (uint16), or is the path (or a list of
    paths) of safetensors checkpoint files holding every weight of the model once (BF16, or F32 narrowed to bf16),
    streamed to the device by the library's reader.

    `stage=(first, end)` makes it a pipeline stage holding layers [first, end) (the reference's StagePipeline split):
    only that stage's weights are loaded (others in `weights` are skipped), a stage after the first reads its input
    from `residual()` and a stage before the last leaves its output there; see prefill_stage and decode."""

    def __init__(self, cfg: QwenConfig, weights, rope_cos: np.ndarray, rope_sin: np.ndarray, device: int = 0,
                 max_seqs: int = 64, kv_pages: int | None = None, max_tokens: int = 4096, max_batch: int = 64,
                 max_pos: int | None = None, stage: tuple | None = None):
        self.cfg = cfg
        self.first, self.end = (0, cfg.layers) if stage is None else (int(stage[0]), int(stage[1]))
        self.is_first, self.is_last = self.first == 0, self.end == cfg.layers
        self.device = device
        max_pos = max_pos or cfg.max_pos
        pages_per_seq = (max_pos + 15) // 16
        kv_pages = kv_pages or max_seqs * pages_per_seq
        c = QwenConfigC(cfg.layers, cfg.hidden, cfg.heads, cfg.kv_heads, cfg.head_dim, cfg.intermediate, cfg.vocab,
                        cfg.eps, max_pos, max_seqs, kv_pages, max_tokens, max_batch)
        h = ctypes.c_void_p()
        N.check(N.lib().lrm_qwen_create_stage(device, ctypes.byref(c), self.first, self.end, ctypes.byref(h)), None,
                "lrm_qwen_create_stage")
        self._h = h
        self.max_seqs, self.max_tokens, self.max_batch, self.max_pos = max_seqs, max_tokens, max_batch, max_pos
        try:
            if isinstance(weights, dict):
                shapes = weight_shapes(cfg)
                for name in stage_weight_names(cfg, self.first, self.end):
                    shape = shapes[name]
                    w = np.ascontiguousarray(weights[name], np.uint16)
                    if w.shape != tuple(shape):
                        raise ValueError(f"{name} is {w.shape}, expected {shape}")
                    self._check(N.lib().lrm_qwen_set_weight(self._h, name.encode(), _p(w, ctypes.c_uint16), w.size),
                                "set_weight")
            else:
                self.load_checkpoint([weights] if isinstance(weights, (str, bytes)) or hasattr(weights, "__fspath__")
                                     else list(weights))
            cos = np.ascontiguousarray(rope_cos[:max_pos], np.float32)
            sin = np.ascontiguousarray(rope_sin[:max_pos], np.float32)
            if cos.shape[0] < max_pos:
                raise ValueError("the RoPE table has fewer rows than max_pos")
            self._check(N.lib().lrm_qwen_set_rope(self._h, _p(cos, F32), _p(sin, F32), cos.shape[0], cos.shape[1]),
                        "set_rope")
        except BaseException:
            self.close()  # a half-built engine frees its device memory
            raise

    def _check(self, status, what):
        if status != N.LRM_OK:
            N.check(status, None, what)

    def load_safetensors(self, path) -> int:
        """Streams every tensor of one safetensors file into the engine; returns how many it loaded."""
        n = I32()
        self._check(N.lib().lrm_qwen_load_safetensors(self._h, str(path).encode("utf-8"), ctypes.byref(n)),
                    "load_safetensors")
        return int(n.value)

    def load_checkpoint(self, paths) -> None:
        """Loads a checkpoint split over `paths`; every weight of the model must come exactly once (a stage takes
        its own and skips the rest)."""
        from .safetensors import SafetensorsFile

        want = set(weight_shapes(self.cfg))
        seen = set()
        for p in paths:
            with SafetensorsFile.open(p) as f:
                names = set(f.names)
            dup, extra = names & seen, names - want
            if dup or extra:
                raise ValueError(f"{p}: " + (f"tensors loaded twice: {sorted(dup)[:3]}" if dup else
                                             f"not weights of this model: {sorted(extra)[:3]}"))
            seen |= names
            if names & set(stage_weight_names(self.cfg, self.first, self.end)):
                self.load_safetensors(p)
        if seen != want:
            raise ValueError(f"the checkpoint misses {len(want - seen)} weights, e.g. {sorted(want - seen)[:3]}")

    def close(self):
        if self._h:
            N.lib().lrm_qwen_destroy(self._h)
            self._h = None

    def __enter__(self):
        return self

    def __exit__(self, *a):
        self.close()

    @property
    def stream(self) -> int:
        s = ctypes.c_void_p()
        self._check(N.lib().lrm_qwen_stream(self._h, ctypes.byref(s)), "stream")
        return s.value or 0

    def prefill(self, slots, prompts, want_logits=False):
        """Fresh prefill of prompts[i] into slots[i]; returns (next ids [n], last-row logits [n, vocab] or None)."""
        return self.prefill_stage(slots, [len(p) for p in prompts], prompts, want_logits)

    def extend(self, slots, chunks, want_logits=False):
        """Chunked prefill: chunks[i] (token ids) continue the tokens slots[i] already holds, attending to all of
        them; returns (next ids [n], last-row logits [n, vocab] or None). Prefill of a prompt's first chunk followed
        by extend of the rest equals one prefill of the whole prompt bit for bit."""
        return self.prefill_stage(slots, [len(c) for c in chunks], chunks, want_logits, extend=True)

    def prefill_stage(self, slots, lens, prompts=None, want_logits=False, extend=False):
        """Fresh prefill (or, with extend, a continuation) of sequences of `lens` tokens in `slots`. The first stage
        takes the token ids (`prompts`); a later stage reads the previous stage's residual rows (sequences packed in
        order) from residual(). Returns (next ids, logits or None) on the last stage, (None, None) on the others."""
        slots = np.ascontiguousarray(slots, np.int32)
        lens = np.ascontiguousarray(lens, np.int32)
        ids = None
        if self.is_first:
            ids = np.ascontiguousarray(np.concatenate([np.asarray(p, np.uint32) for p in prompts]), np.uint32)
        nxt = np.empty(len(slots), np.uint32) if self.is_last else None
        logits = np.empty((len(slots), self.cfg.vocab), np.float32) if want_logits and self.is_last else None
        fn = N.lib().lrm_qwen_extend if extend else N.lib().lrm_qwen_prefill
        self._check(fn(self._h, len(slots), _p(slots, I32), _p(lens, I32),
                       _p(ids, U32) if ids is not None else None,
                       _p(nxt, U32) if nxt is not None else None,
                       _p(logits, F32) if logits is not None else None), "extend" if extend else "prefill")
        return nxt, logits

    def decode(self, slots, ids=None, want_logits=False):
        """One decode step: ids[b] appended to slots[b] (the first stage; later stages read the residual rows).
        Returns (next ids, logits or None) on the last stage, (None, None) on the others."""
        slots = np.ascontiguousarray(slots, np.int32)
        ids = np.ascontiguousarray(ids, np.uint32) if self.is_first else None
        nxt = np.empty(len(slots), np.uint32) if self.is_last else None
        logits = np.empty((len(slots), self.cfg.vocab), np.float32) if want_logits and self.is_last else None
        self._check(N.lib().lrm_qwen_decode(self._h, len(slots), _p(slots, I32),
                                            _p(ids, U32) if ids is not None else None,
                                            _p(nxt, U32) if nxt is not None else None,
                                            _p(logits, F32) if logits is not None else None), "decode")
        return nxt, logits

    def residual(self, rows: int | None = None):
        """The fp32 residual x [rows, hidden] as a torch tensor viewing the engine's device buffer (no copy): the
        boundary a pipeline stage reads from and writes to. Work on it must be ordered with the engine's calls
        (synchronise, or use the engine's stream)."""
        import torch

        ptr, cap = P(), ctypes.c_int64()
        self._check(N.lib().lrm_qwen_residual(self._h, ctypes.byref(ptr), ctypes.byref(cap)), "residual")
        rows = int(cap.value) if rows is None else int(rows)
        if rows > cap.value:
            raise ValueError(f"the residual holds {cap.value} rows")
        with torch.cuda.device(self.device):
            return torch.as_tensor(_CudaArray(ptr.value, (rows, self.cfg.hidden), "<f4"), device=f"cuda:{self.device}")

    def capture(self, slots, first_ids=None, time_attention=False):
        """Captures the device-resident decode step for `slots` (inputs: the previous step's outputs)."""
        slots = np.ascontiguousarray(slots, np.int32)
        fid = None if first_ids is None else np.ascontiguousarray(first_ids, np.uint32)
        self._check(N.lib().lrm_qwen_decode_graph(self._h, len(slots), _p(slots, I32),
                                                  _p(fid, U32) if fid is not None else None,
                                                  1 if time_attention else 0), "decode_graph")
        self._graph_batch = len(slots)

    def graph_kernels(self) -> int:
        v = ctypes.c_int32()
        self._check(N.lib().lrm_qwen_graph_kernels(self._h, ctypes.byref(v)), "graph_kernels")
        return v.value

    def attention_ms(self) -> np.ndarray:
        out = np.empty(self.end - self.first, np.float32)
        self._check(N.lib().lrm_qwen_attention_ms(self._h, _p(out, F32)), "attention_ms")
        return out

    def truncate(self, slot: int, length: int):
        self._check(N.lib().lrm_qwen_truncate(self._h, slot, length), "truncate")

    def replay(self, steps: int):
        self._check(N.lib().lrm_qwen_decode_replay(self._h, steps), "decode_replay")

    def last_ids(self):
        out = np.empty(self._graph_batch, np.uint32)
        self._check(N.lib().lrm_qwen_last_ids(self._h, _p(out, U32)), "last_ids")
        return out

    def sync(self):
        self._check(N.lib().lrm_qwen_sync(self._h), "sync")

    def reserve(self, slot: int, tokens: int):
        self._check(N.lib().lrm_qwen_reserve(self._h, slot, tokens), "reserve")

    def seq_len(self, slot: int) -> int:
        v = ctypes.c_int32()
        self._check(N.lib().lrm_qwen_seq_len(self._h, slot, ctypes.byref(v)), "seq_len")
        return v.value

    def greedy(self, prompts, steps: int, slots=None, want_logits=False):
        """The canonical greedy schedule for each prompt: prefill, then steps - 1 single-token decode steps.
        Returns ids [n, steps] (and logits [n, steps, vocab] when asked)."""
        n = len(prompts)
        slots = np.arange(n, dtype=np.int32) if slots is None else np.asarray(slots, np.int32)
        nxt, lg = self.prefill(slots, prompts, want_logits)
        ids, logs = [nxt.copy()], [lg]
        for _ in range(1, steps):
            nxt, lg = self.decode(slots, nxt, want_logits)
            ids.append(nxt.copy())
            logs.append(lg)
        ids = np.stack(ids, 1).astype(np.int64)
        if want_logits:
            return ids, np.stack(logs, 1)
        return ids
