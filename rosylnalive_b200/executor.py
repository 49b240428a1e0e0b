"""The fp32 forward executor over the device contracts: the reference's planned X1 executor (docs/dev-plan.md
"GpuForwardOps", a two-pass static plan, HeapPlanner then a sealed table) written against the IGpuBackend interface
only, so it runs on any backend that implements it -- here the CUDA device.

It records the Qwen3 forward of tests/Lrm.Tensor.Tests/TinyModel.fs:144-204 as catalog dispatches (embed_gather_bf16,
rmsnorm_rows, matmul_bf16w, rope_apply, copy_rows, attention_gqa_causal, add, silu_mul, argmax_rows) with a barrier
between dependent dispatches, and the greedy schedule of TinyModel.fs:219-236. Activations and the KV cache are fp32,
as the catalog defines them. This is the fp32 parity path; the bf16 fast path is qwen.py.
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np

from . import gpu_core as G

HF = {
    "input_layernorm": "input_layernorm.weight",
    "q_proj": "self_attn.q_proj.weight",
    "k_proj": "self_attn.k_proj.weight",
    "v_proj": "self_attn.v_proj.weight",
    "o_proj": "self_attn.o_proj.weight",
    "q_norm": "self_attn.q_norm.weight",
    "k_norm": "self_attn.k_norm.weight",
    "post_attention_layernorm": "post_attention_layernorm.weight",
    "gate_proj": "mlp.gate_proj.weight",
    "up_proj": "mlp.up_proj.weight",
    "down_proj": "mlp.down_proj.weight",
}


@dataclass(frozen=True)
class QwenConfig:
    layers: int
    hidden: int
    heads: int
    kv_heads: int
    head_dim: int
    intermediate: int
    vocab: int
    eps: float
    max_pos: int
    rope_theta: float = 1e6

    @staticmethod
    def from_hf(cfg: dict) -> "QwenConfig":
        return QwenConfig(cfg["num_hidden_layers"], cfg["hidden_size"], cfg["num_attention_heads"],
                          cfg["num_key_value_heads"], cfg["head_dim"], cfg["intermediate_size"], cfg["vocab_size"],
                          float(cfg["rms_norm_eps"]), cfg["max_position_embeddings"],
                          float(cfg.get("rope_theta", 1e6)))


def weight_shapes(c: QwenConfig) -> dict:
    """HF name -> shape of every weight (TinyModel.fs:79-101; tied embeddings, no lm_head)."""
    s = {"model.embed_tokens.weight": (c.vocab, c.hidden), "model.norm.weight": (c.hidden,)}
    q, kv = c.heads * c.head_dim, c.kv_heads * c.head_dim
    per = {"input_layernorm": (c.hidden,), "q_proj": (q, c.hidden), "k_proj": (kv, c.hidden),
           "v_proj": (kv, c.hidden), "o_proj": (c.hidden, q), "q_norm": (c.head_dim,), "k_norm": (c.head_dim,),
           "post_attention_layernorm": (c.hidden,), "gate_proj": (c.intermediate, c.hidden),
           "up_proj": (c.intermediate, c.hidden), "down_proj": (c.hidden, c.intermediate)}
    for i in range(c.layers):
        for k, shp in per.items():
            s[f"model.layers.{i}.{HF[k]}"] = shp
    return s


def tap_shapes(c: QwenConfig, T: int) -> dict:
    """The forward's taps (the reference's tap names, goldens/tiny/g1 fwd_f32.*): name -> [rows, cols] for T rows."""
    q, kv, H, I = c.heads * c.head_dim, c.kv_heads * c.head_dim, c.hidden, c.intermediate
    per = {"input_layernorm.out": H, "attn.q_proj.out": q, "attn.k_proj.out": kv, "attn.v_proj.out": kv,
           "attn.q_norm.out": q, "attn.k_norm.out": kv, "attn.q_rope": q, "attn.k_rope": kv, "attn.v_cache": kv,
           "attn.o_proj.in": q, "attn.o_proj.out": H, "resid_mid": H, "post_attention_layernorm.out": H,
           "mlp.gate.out": I, "mlp.up.out": I, "mlp.down.in": I, "mlp.down.out": H, "out": H}
    s = {"embed.out": (T, H)}
    for i in range(c.layers):
        for k, cols in per.items():
            s[f"L{i}.{k}"] = (T, cols)
    s["final_norm.out"] = (T, H)
    s["logits"] = (T, c.vocab)
    return s


class Fp32Executor:
    """Plans, uploads and runs the fp32 Qwen3 forward on one backend.

    max_tokens bounds the rows of one forward (the longest prefill chunk); the KV cache holds max_pos positions.
    With taps, the plan adds a Taps arena (the reference's GpuExecutor plan: "taps copied into the Taps arena at
    record time") holding every intermediate of the forward under the reference's tap names: each is copied there by
    the command list right after the dispatch that produces it, before a later one overwrites its activation buffer.
    """

    def __init__(self, backend, config: QwenConfig, weights: dict, rope_cos: np.ndarray, rope_sin: np.ndarray,
                 max_tokens: int, page_bytes: int = G.MAX_PAGE_BYTES, taps: bool = False):
        self.b = backend
        self.c = c = config
        self.max_tokens = T = max_tokens
        if rope_cos.shape != (c.max_pos, c.head_dim // 2):
            raise ValueError("the RoPE table must be [max_pos, head_dim/2]")
        q, kv, H, I = c.heads * c.head_dim, c.kv_heads * c.head_dim, c.hidden, c.intermediate
        f32, bf16, u32 = G.DType.F32, G.DType.BF16, G.DType.U32

        # Pass one: placements.
        planner = G.HeapPlanner(page_bytes)
        specs = []  # (name, arena, dtype, dims, flags)
        for name, shp in weight_shapes(c).items():
            specs.append((name, G.ArenaKind.WEIGHTS, bf16, list(shp), G.TensorFlags.READ_ONLY))
        specs.append(("rope.cos", G.ArenaKind.ROPE, f32, [c.max_pos, c.head_dim // 2], G.TensorFlags.READ_ONLY))
        specs.append(("rope.sin", G.ArenaKind.ROPE, f32, [c.max_pos, c.head_dim // 2], G.TensorFlags.READ_ONLY))
        for i in range(c.layers):
            specs.append((f"L{i}.k_cache", G.ArenaKind.KV_CACHE, f32, [c.max_pos, kv], G.TensorFlags.NONE))
            specs.append((f"L{i}.v_cache", G.ArenaKind.KV_CACHE, f32, [c.max_pos, kv], G.TensorFlags.NONE))
        acts = {"ids": (u32, [T]), "x": (f32, [T, H]), "h": (f32, [T, H]), "q": (f32, [T, q]), "k": (f32, [T, kv]),
                "v": (f32, [T, kv]), "qn": (f32, [T, q]), "kn": (f32, [T, kv]), "qr": (f32, [T, q]),
                "kr": (f32, [T, kv]), "o": (f32, [T, q]), "oo": (f32, [T, H]), "r": (f32, [T, H]),
                "h2": (f32, [T, H]), "g": (f32, [T, I]), "u": (f32, [T, I]), "d": (f32, [T, I]),
                "dd": (f32, [T, H]), "f": (f32, [T, H]), "f_last": (f32, [1, H])}
        for name, (dt, dims) in acts.items():
            specs.append((name, G.ArenaKind.ACTIVATIONS, dt, dims, G.TensorFlags.NONE))
        specs.append(("logits", G.ArenaKind.LOGITS, f32, [T, c.vocab], G.TensorFlags.NONE))
        specs.append(("next", G.ArenaKind.LOGITS, u32, [T], G.TensorFlags.NONE))
        self.taps = tap_shapes(c, T) if taps else {}
        for name, dims in self.taps.items():
            specs.append(("tap:" + name, G.ArenaKind.TAPS, f32, list(dims), G.TensorFlags.NONE))
        placements = []
        for name, arena, dt, dims, flags in specs:
            n = 1
            for d in dims:
                n *= d
            placements.append(planner.allocate(arena, G.align_up(4, n * dt.size)))
        layout = planner.build()

        # Pass two: the table.
        table = G.TensorTable(layout)
        self.tok = {}
        self.place = {}
        for (name, arena, dt, dims, flags), pl in zip(specs, placements):
            self.tok[name] = table.add(name, pl, dt, dims, flags)
            self.place[name] = (layout.slot_of(pl.arena, pl.page), pl.offset)
        self.table = table.seal()

        self.heap = backend.create_heap(layout)
        if backend.kernels is None:
            backend.load_kernels()
        self.heap.write_table(self.table)
        for name, shp in weight_shapes(c).items():
            w = np.ascontiguousarray(weights[name], np.uint16)
            if w.shape != tuple(shp):
                raise ValueError(f"{name} is {w.shape}, expected {shp}")
            self._upload(name, w)
        self._upload("rope.cos", np.ascontiguousarray(rope_cos, np.float32))
        self._upload("rope.sin", np.ascontiguousarray(rope_sin, np.float32))
        self.scale = float(np.float32(c.head_dim ** -0.5))
        self.eps = float(np.float32(c.eps))

    def _upload(self, name, arr):
        slot, off = self.place[name]
        b = arr.view(np.uint8).reshape(-1)
        if b.nbytes % 4:
            b = np.concatenate([b, np.zeros(4 - b.nbytes % 4, np.uint8)])
        self.heap.upload(slot, off, b)

    def download(self, name, dtype, shape):
        slot, off = self.place[name]
        n = int(np.prod(shape))
        return self.heap.download_array(slot, off, dtype, n).reshape(shape)

    def reset_cache(self):
        kv = self.c.kv_heads * self.c.head_dim
        zero = np.zeros((self.c.max_pos, kv), np.float32)
        for i in range(self.c.layers):
            self._upload(f"L{i}.k_cache", zero)
            self._upload(f"L{i}.v_cache", zero)

    # -- recording ------------------------------------------------------------------------------------------------

    def _tap(self, cl, name: str, src: str, rows: int):
        """Copies rows [0, rows) of activation `src` to the Taps arena's tensor `name` (after a barrier, so the
        dispatch that wrote it has finished)."""
        if name not in self.taps:
            return
        cl.barrier()
        cols = self.taps[name][1]
        (ss, so), (ds, do) = self.place[src], self.place["tap:" + name]
        cl.copy(G.BufferRange(ss, so, rows * cols * 4), G.BufferRange(ds, do, rows * cols * 4))

    def record_forward(self, cl, T: int, pos0: int, logits_rows: str):
        c, t = self.c, self.tok
        q, kv, H, I = c.heads * c.head_dim, c.kv_heads * c.head_dim, c.hidden, c.intermediate
        d = cl.dispatch_named
        tap = lambda name, src: self._tap(cl, name, src, T)  # noqa: E731
        d("embed_gather_bf16", ids=t["ids"], table=t["model.embed_tokens.weight"], y=t["x"], rows=T, cols=H,
          vocab=c.vocab)
        tap("embed.out", "x")
        for i in range(c.layers):
            p, L = f"model.layers.{i}.", f"L{i}."
            cl.barrier()
            d("rmsnorm_rows", x=t["x"], w=t[p + HF["input_layernorm"]], y=t["h"], rows=T, cols=H, eps=self.eps)
            tap(L + "input_layernorm.out", "h")
            cl.barrier()
            d("matmul_bf16w", x=t["h"], w=t[p + HF["q_proj"]], y=t["q"], m=T, n=q, k=H)
            d("matmul_bf16w", x=t["h"], w=t[p + HF["k_proj"]], y=t["k"], m=T, n=kv, k=H)
            d("matmul_bf16w", x=t["h"], w=t[p + HF["v_proj"]], y=t["v"], m=T, n=kv, k=H)
            tap(L + "attn.q_proj.out", "q")
            tap(L + "attn.k_proj.out", "k")
            tap(L + "attn.v_proj.out", "v")
            cl.barrier()
            d("rmsnorm_rows", x=t["q"], w=t[p + HF["q_norm"]], y=t["qn"], rows=T * c.heads, cols=c.head_dim,
              eps=self.eps)
            d("rmsnorm_rows", x=t["k"], w=t[p + HF["k_norm"]], y=t["kn"], rows=T * c.kv_heads, cols=c.head_dim,
              eps=self.eps)
            tap(L + "attn.q_norm.out", "qn")
            tap(L + "attn.k_norm.out", "kn")
            cl.barrier()
            d("rope_apply", x=t["qn"], cos_table=t["rope.cos"], sin_table=t["rope.sin"], y=t["qr"],
              rows=T * c.heads, heads=c.heads, head_dim=c.head_dim, pos0=pos0)
            d("rope_apply", x=t["kn"], cos_table=t["rope.cos"], sin_table=t["rope.sin"], y=t["kr"],
              rows=T * c.kv_heads, heads=c.kv_heads, head_dim=c.head_dim, pos0=pos0)
            tap(L + "attn.q_rope", "qr")
            tap(L + "attn.k_rope", "kr")
            cl.barrier()
            d("copy_rows", src=t["kr"], dst=t[f"L{i}.k_cache"], rows=T, cols=kv, src_row0=0, dst_row0=pos0,
              src_stride=kv, dst_stride=kv)
            d("copy_rows", src=t["v"], dst=t[f"L{i}.v_cache"], rows=T, cols=kv, src_row0=0, dst_row0=pos0,
              src_stride=kv, dst_stride=kv)
            if L + "attn.v_cache" in self.taps:  # the rows just appended to the cache
                cl.barrier()
                (ss, so), (ds, do) = self.place[f"L{i}.v_cache"], self.place["tap:" + L + "attn.v_cache"]
                n = T * kv * 4
                cl.copy(G.BufferRange(ss, so + pos0 * kv * 4, n), G.BufferRange(ds, do, n))
            cl.barrier()
            d("attention_gqa_causal", q=t["qr"], k=t[f"L{i}.k_cache"], v=t[f"L{i}.v_cache"], y=t["o"], rows=T,
              q_row0=0, past=pos0, q_heads=c.heads, kv_heads=c.kv_heads, head_dim=c.head_dim, scale=self.scale)
            tap(L + "attn.o_proj.in", "o")
            cl.barrier()
            d("matmul_bf16w", x=t["o"], w=t[p + HF["o_proj"]], y=t["oo"], m=T, n=H, k=q)
            tap(L + "attn.o_proj.out", "oo")
            cl.barrier()
            d("add", a=t["x"], b=t["oo"], y=t["r"], n=T * H)
            tap(L + "resid_mid", "r")
            cl.barrier()
            d("rmsnorm_rows", x=t["r"], w=t[p + HF["post_attention_layernorm"]], y=t["h2"], rows=T, cols=H,
              eps=self.eps)
            tap(L + "post_attention_layernorm.out", "h2")
            cl.barrier()
            d("matmul_bf16w", x=t["h2"], w=t[p + HF["gate_proj"]], y=t["g"], m=T, n=I, k=H)
            d("matmul_bf16w", x=t["h2"], w=t[p + HF["up_proj"]], y=t["u"], m=T, n=I, k=H)
            tap(L + "mlp.gate.out", "g")
            tap(L + "mlp.up.out", "u")
            cl.barrier()
            d("silu_mul", gate=t["g"], up=t["u"], y=t["d"], n=T * I)
            tap(L + "mlp.down.in", "d")
            cl.barrier()
            d("matmul_bf16w", x=t["d"], w=t[p + HF["down_proj"]], y=t["dd"], m=T, n=H, k=I)
            tap(L + "mlp.down.out", "dd")
            cl.barrier()
            d("add", a=t["r"], b=t["dd"], y=t["x"], n=T * H)
            tap(L + "out", "x")
        cl.barrier()
        d("rmsnorm_rows", x=t["x"], w=t["model.norm.weight"], y=t["f"], rows=T, cols=H, eps=self.eps)
        tap("final_norm.out", "f")
        cl.barrier()
        if logits_rows == "last":
            d("copy_rows", src=t["f"], dst=t["f_last"], rows=1, cols=H, src_row0=T - 1, dst_row0=0, src_stride=H,
              dst_stride=H)
            cl.barrier()
            d("matmul_bf16w", x=t["f_last"], w=t["model.embed_tokens.weight"], y=t["logits"], m=1, n=c.vocab, k=H)
            rows = 1
        else:
            d("matmul_bf16w", x=t["f"], w=t["model.embed_tokens.weight"], y=t["logits"], m=T, n=c.vocab, k=H)
            rows = T
        self._tap(cl, "logits", "logits", rows)
        cl.barrier()
        d("argmax_rows", x=t["logits"], y=t["next"], rows=rows, cols=c.vocab)
        return rows

    def forward(self, pos0: int, ids, logits_rows: str = "all"):
        """One forward over ids at positions pos0..pos0+T-1; returns (logits [rows, vocab], argmax [rows])."""
        ids = np.ascontiguousarray(ids, np.uint32)
        T = len(ids)
        if T < 1 or T > self.max_tokens:
            raise ValueError(f"{T} tokens: 1..{self.max_tokens} per forward")
        if pos0 < 0 or pos0 + T > self.c.max_pos:
            raise ValueError("positions past max_pos")
        self._upload("ids", ids)
        cl = self.b.begin()
        rows = self.record_forward(cl, T, pos0, logits_rows)
        self.b.wait(self.b.submit(cl))
        logits = self.download("logits", np.float32, (rows, self.c.vocab))
        nxt = self.download("next", np.uint32, (rows,))
        self._last = (T, rows)
        return logits, nxt

    def read_taps(self) -> dict:
        """The taps of the last forward: name -> float32 [T, cols] ([rows, vocab] for the logits)."""
        if not self.taps:
            raise RuntimeError("the executor was built without taps")
        T, rows = self._last
        return {name: self.download("tap:" + name, np.float32, (rows if name == "logits" else T, cols))
                for name, (_, cols) in self.taps.items()}

    def greedy(self, prompt, steps: int, return_logits: bool = False):
        """TinyModel.greedy: prefill once, then single-token steps; argmax of each step's last row (a NaN row
        raises, as CpuRef.argmax does)."""
        self.reset_cache()
        logits, nxt = self.forward(0, prompt, "last")
        out_logits = [logits[-1].copy()]
        ids = [self._checked(nxt[-1])]
        for s in range(1, steps):
            logits, nxt = self.forward(len(prompt) + s - 1, [ids[-1]], "last")
            out_logits.append(logits[-1].copy())
            ids.append(self._checked(nxt[-1]))
        ids = np.array(ids, np.int64)
        return (ids, np.stack(out_logits)) if return_logits else ids

    @staticmethod
    def _checked(i):
        if int(i) == 0xFFFFFFFF:
            raise ValueError("argmax of a row that holds a NaN")
        return int(i)
