"""Catalog-kernel conformance on the CUDA device against the parity oracle (GPU tier).

Every case goes through the device contracts (CreateHeap, WriteTable, Upload, Dispatch, Submit, Wait, Download),
like the reference's conformance harness (tests/Lrm.Kernels.Conformance): outputs are poisoned first, each case runs
twice and must be bit-identical, and each kernel is judged by its KernelBounds kind
(docs/contracts/kernel-bounds.md): BitExact against CpuRef F32, or Relative:
relL2(gpu, CpuRef64) <= max(1e-6, 2 * relL2(CpuRef32, CpuRef64)).
"""

import ctypes

import numpy as np
import pytest

from oracle import oracle as O
from tests.conftest import cuda_available

pytestmark = pytest.mark.gpu

if cuda_available():
    from rosylnalive_b200 import cuda_backend as CB
    from rosylnalive_b200 import gpu_core as G
    from rosylnalive_b200 import native as N

POISON = 0x7FBADBAD


def rel_l2(a, ref):
    a = np.asarray(a, np.float64).reshape(-1)
    ref = np.asarray(ref, np.float64).reshape(-1)
    return float(np.linalg.norm(a - ref) / max(np.linalg.norm(ref), 1e-300))


def relative_ok(gpu, ref32, ref64):
    bound = max(1e-6, 2 * rel_l2(ref32, ref64))
    measured = rel_l2(gpu, ref64)
    assert not np.any(np.isnan(gpu))
    assert measured <= bound, f"relL2 {measured:.3e} > bound {bound:.3e}"
    return measured, bound


class Rig:
    """One backend with a planned heap of named tensors."""

    def __init__(self, tensors, time_dispatches=False):
        self.backend = CB.try_create(CB.DeviceOptions(time_dispatches=time_dispatches))
        planner = G.HeapPlanner(G.MAX_PAGE_BYTES)
        specs = []
        for name, (dtype, count) in tensors.items():
            arena = G.ArenaKind.WEIGHTS if name.startswith("w_") else G.ArenaKind.ACTIVATIONS
            specs.append((name, arena, dtype, count, planner.allocate(arena, G.align_up(4, count * dtype.size))))
        layout = planner.build()
        table = G.TensorTable(layout)
        self.tok, self.where, self.dtype = {}, {}, {}
        for name, arena, dtype, count, pl in sorted(specs, key=lambda s: (s[1], s[4].page, s[4].offset)):
            flags = G.TensorFlags.READ_ONLY if arena == G.ArenaKind.WEIGHTS else G.TensorFlags.NONE
            self.tok[name] = table.add(name, pl, dtype, [count], flags)
            self.where[name] = (layout.slot_of(pl.arena, pl.page), pl.offset, count)
            self.dtype[name] = dtype
        self.table = table.seal()
        self.heap = self.backend.create_heap(layout)
        self.kernels = self.backend.load_kernels()
        self.heap.write_table(self.table)

    def put(self, name, arr):
        slot, off, count = self.where[name]
        b = np.ascontiguousarray(arr).view(np.uint8).reshape(-1)
        if b.nbytes % 4:
            b = np.concatenate([b, np.zeros(4 - b.nbytes % 4, np.uint8)])
        self.heap.upload(slot, off, b)

    def poison(self, name):
        slot, off, count = self.where[name]
        nbytes = G.align_up(4, count * self.dtype[name].size)
        self.heap.upload(slot, off, np.full(nbytes // 4, POISON, np.uint32))

    def get(self, name, np_dtype, n=None):
        slot, off, count = self.where[name]
        return self.heap.download_array(slot, off, np_dtype, count if n is None else n)

    def run(self, kernel, outputs=(), **fields):
        """Poisons `outputs`, dispatches twice, and checks the two runs are bit-identical."""
        results = []
        for _ in range(2):
            for o in outputs:
                self.poison(o)
            cl = self.backend.begin()
            cl.dispatch_named(kernel, **{k: (self.tok[v] if isinstance(v, str) else v) for k, v in fields.items()})
            self.backend.wait(self.backend.submit(cl))
            results.append([self.get(o, np.uint32) for o in outputs])
        for a, b in zip(*results):
            assert np.array_equal(a, b), f"{kernel}: two runs differ"
        return results[0]

    def close(self):
        self.backend.dispose()


@pytest.fixture(scope="module")
def rng():
    return np.random.default_rng(0x4C524D2D45314341)


def f32(words):
    return words.view(np.float32)


def test_enumerate_and_class():
    cands = CB.CudaBackendProvider().enumerate()
    assert cands and cands[0].accepted, cands
    b = CB.try_create()
    b.load_kernels()
    ec = b.execution_class
    assert ec.backend == "cuda" and ec.device_id.startswith("pci:10de:") and len(ec.shader_set_hash) == 64
    assert b.fp32_denormals == "preserve"
    with pytest.raises(G.GpuContractException):
        b.load_kernels()
    b.dispose()


def test_selftests_scale_unpack_echo(rng):
    F, U, B = G.DType.F32, G.DType.U32, G.DType.BF16
    rig = Rig({"x": (F, 1000), "y": (F, 1000), "xb": (B, 999), "e": (U, 70000)})
    try:
        x = rng.standard_normal(1000).astype(np.float32)
        x[7] = np.nan
        rig.put("x", x)
        (y,) = rig.run("scale_f32", ["y"], x="x", y="y", n=1000, a=0.5)
        ref = x * np.float32(0.5)
        ok = np.isnan(ref) | (f32(y) == ref)
        assert ok.all() and np.isnan(f32(y)[7])
        xb = rng.integers(0, 65535, 999, dtype=np.uint16)
        rig.put("xb", xb)
        (y,) = rig.run("bf16_unpack", ["y"], x="xb", y="y", n=999)
        assert np.array_equal(y[:999], xb.astype(np.uint32) << 16)
        (e,) = rig.run("groups_echo", ["e"], y="e", groups=70000)  # folded to (35000, 2, 1)
        assert np.array_equal(e, np.arange(70000, dtype=np.uint32))
        fields = {f"v{i}": 1000 + i for i in range(2, 32)}
        (e,) = rig.run("args_echo", ["e"], y="e", **fields)
        assert e[0] == 1 and e[1] == rig.tok["e"] and list(e[2:32]) == [1000 + i for i in range(2, 32)]
        (e,) = rig.run("table_echo", ["e"], src=rig.tok["x"], y="e")
        assert list(e[:16]) == rig.table.row(rig.tok["x"]).w
        (e,) = rig.run("table_echo", ["e"], src=0, y="e")
        assert list(e[:16]) == [0] * 16
    finally:
        rig.close()


def test_embed_gather_bit_exact(rng):
    V, H, T = 300, 72, 9
    rig = Rig({"w_table": (G.DType.BF16, V * H), "ids": (G.DType.U32, T), "y": (G.DType.F32, T * H)})
    try:
        table = rng.integers(0, 65535, (V, H), dtype=np.uint16)
        ids = np.array([0, 5, 299, 300, 7, 1 << 31, 1, 2, 3], np.uint32)
        rig.put("w_table", table)
        rig.put("ids", ids)
        (y,) = rig.run("embed_gather_bf16", ["y"], ids="ids", table="w_table", y="y", rows=T, cols=H, vocab=V)
        ref = O.embed_gather(table, ids, "f32")
        assert np.array_equal(y, ref.view(np.uint32).reshape(-1))
    finally:
        rig.close()


@pytest.mark.parametrize("rows,cols", [(37, 1024), (13 * 16, 128), (3, 1), (2, 1000)])
def test_rmsnorm_relative(rng, rows, cols):
    rig = Rig({"x": (G.DType.F32, rows * cols), "w_w": (G.DType.BF16, cols), "y": (G.DType.F32, rows * cols)})
    try:
        x = rng.standard_normal((rows, cols)).astype(np.float32)
        w = O.narrow_rne((1 + 0.02 * rng.standard_normal(cols)).astype(np.float32))
        rig.put("x", x)
        rig.put("w_w", w)
        (y,) = rig.run("rmsnorm_rows", ["y"], x="x", w="w_w", y="y", rows=rows, cols=cols, eps=1e-6)
        relative_ok(f32(y), O.rmsnorm(x, w, 1e-6, "f32"), O.rmsnorm(x, w, 1e-6, "f64"))
        # in place (y aliases x, declared)
        (y2,) = rig.run("rmsnorm_rows", [], x="x", w="w_w", y="x", rows=rows, cols=cols, eps=1e-6) or [None]
    finally:
        rig.close()


def test_rope_matches_cpuref_bits(rng):
    from rosylnalive_b200 import rope as R
    cos, sin = R.t_spec(R.QWEN3_INV_FREQ_BITS, 4200)
    T, heads, hd, pos0 = 7, 16, 128, 4090
    rig = Rig({"x": (G.DType.F32, T * heads * hd), "cos": (G.DType.F32, cos.size), "sin": (G.DType.F32, sin.size),
               "y": (G.DType.F32, T * heads * hd)})
    try:
        x = rng.standard_normal((T, heads * hd)).astype(np.float32)
        rig.put("x", x)
        rig.put("cos", cos)
        rig.put("sin", sin)
        (y,) = rig.run("rope_apply", ["y"], x="x", cos_table="cos", sin_table="sin", y="y", rows=T * heads,
                       heads=heads, head_dim=hd, pos0=pos0)
        ref = O.rope_apply(x, cos, sin, heads, pos0, "f32")
        assert np.array_equal(y, ref.view(np.uint32).reshape(-1))
    finally:
        rig.close()


def test_silu_mul_and_add(rng):
    n = 3 * 3072 + 5
    F = G.DType.F32
    rig = Rig({"g": (F, n), "u": (F, n), "y": (F, n)})
    try:
        g = (4 * rng.standard_normal(n)).astype(np.float32)
        u = rng.standard_normal(n).astype(np.float32)
        rig.put("g", g)
        rig.put("u", u)
        (y,) = rig.run("silu_mul", ["y"], gate="g", up="u", y="y", n=n)
        relative_ok(f32(y), O.silu_mul(g, u, "f32"), O.silu_mul(g, u, "f64"))
        (y,) = rig.run("add", ["y"], a="g", b="u", y="y", n=n)
        assert np.array_equal(y, O.add(g, u, "f32").view(np.uint32))
    finally:
        rig.close()


def test_copy_rows_bit_exact(rng):
    U = G.DType.U32
    rig = Rig({"src": (U, 40 * 64), "dst": (U, 50 * 80)})
    try:
        src = rng.integers(0, 2 ** 32, 40 * 64, dtype=np.uint32)
        rig.put("src", src)
        rig.put("dst", np.zeros(50 * 80, np.uint32))
        cl = rig.backend.begin()
        cl.dispatch_named("copy_rows", src=rig.tok["src"], dst=rig.tok["dst"], rows=13, cols=60, src_row0=3,
                          dst_row0=31, src_stride=64, dst_stride=80)
        rig.backend.wait(rig.backend.submit(cl))
        dst = rig.get("dst", np.uint32).reshape(50, 80)
        ref = np.zeros((50, 80), np.uint32)
        ref[31:44, :60] = src.reshape(40, 64)[3:16, :60]
        assert np.array_equal(dst, ref)
    finally:
        rig.close()


def test_argmax_rows(rng):
    rows, cols = 6, 151936
    rig = Rig({"x": (G.DType.F32, rows * cols), "y": (G.DType.U32, rows)})
    try:
        x = rng.standard_normal((rows, cols)).astype(np.float32)
        x[1, 5] = x[1, 150000] = 100.0  # tie: lowest index
        x[2, :] = 0.0
        x[2, 3] = -0.0  # +0 and -0 tie
        x[3, 77777] = np.nan
        x[4, -1] = 50.0
        rig.put("x", x)
        (y,) = rig.run("argmax_rows", ["y"], x="x", y="y", rows=rows, cols=cols)
        assert np.array_equal(y, O.argmax_rows(x, "f32"))
        assert y[1] == 5 and y[2] == 0 and y[3] == 0xFFFFFFFF and y[4] == cols - 1
    finally:
        rig.close()


@pytest.mark.parametrize("m,n,k", [(37, 96, 256), (1, 2048, 1024), (65, 130, 1000), (5, 3072, 1024),
                                   (3, 1024, 3072)])
def test_matmul_bit_exact_to_cpuref_f32(rng, m, n, k):
    rig = Rig({"x": (G.DType.F32, m * k), "w_w": (G.DType.BF16, n * k), "y": (G.DType.F32, m * n)})
    try:
        x = rng.uniform(-1, 1, (m, k)).astype(np.float32)
        w = O.narrow_rne((0.02 * rng.standard_normal((n, k))).astype(np.float32))
        rig.put("x", x)
        rig.put("w_w", w)
        (y,) = rig.run("matmul_bf16w", ["y"], x="x", w="w_w", y="y", m=m, n=n, k=k)
        ref = O.matmul_bf16w(x, w, "f32")
        assert np.array_equal(y, ref.view(np.uint32).reshape(-1))
        # batch invariance: row 0 alone equals row 0 in the batch
        (y1,) = rig.run("matmul_bf16w", ["y"], x="x", w="w_w", y="y", m=1, n=n, k=k)
        assert np.array_equal(y1[:n], y[:n])
    finally:
        rig.close()


@pytest.mark.parametrize("qh,kvh,hd,past,rows", [(16, 8, 128, 0, 70), (16, 8, 128, 4095, 1), (16, 8, 128, 63, 2),
                                                  (4, 2, 32, 0, 13), (8, 1, 64, 100, 3), (6, 3, 200, 10, 5),
                                                  (3, 1, 3, 0, 9)])
def test_attention_relative_and_batch_invariant(rng, qh, kvh, hd, past, rows):
    keys = past + rows
    F = G.DType.F32
    rig = Rig({"q": (F, rows * qh * hd), "k": (F, keys * kvh * hd), "v": (F, keys * kvh * hd),
               "y": (F, rows * qh * hd)})
    try:
        q = rng.standard_normal((rows, qh * hd)).astype(np.float32)
        k = rng.standard_normal((keys, kvh * hd)).astype(np.float32)
        v = rng.standard_normal((keys, kvh * hd)).astype(np.float32)
        for nme, a in (("q", q), ("k", k), ("v", v)):
            rig.put(nme, a)
        scale = float(np.float32(hd ** -0.5))
        (y,) = rig.run("attention_gqa_causal", ["y"], q="q", k="k", v="v", y="y", rows=rows, q_row0=0, past=past,
                       q_heads=qh, kv_heads=kvh, head_dim=hd, scale=scale)
        ref32 = O.attention(q, k, v, qh, kvh, hd, past, scale, "f32")
        ref64 = O.attention(q, k, v, qh, kvh, hd, past, scale, "f64")
        relative_ok(f32(y), ref32, ref64)
        # the last query alone (a decode step at past + rows - 1) equals the same row of the prefill, bit for bit
        (y1,) = rig.run("attention_gqa_causal", ["y"], q="q", k="k", v="v", y="y", rows=1, q_row0=rows - 1,
                        past=past + rows - 1, q_heads=qh, kv_heads=kvh, head_dim=hd, scale=scale)
        last = slice((rows - 1) * qh * hd, rows * qh * hd)
        assert np.array_equal(y1[last], y[last])
    finally:
        rig.close()


def test_native_shim_refuses_bad_blocks():
    """The library checks the block again, so a block that skipped the host rules never reaches a kernel."""
    F = G.DType.F32
    rig = Rig({"x": (F, 64), "w_w": (G.DType.BF16, 64), "y": (F, 64)})
    try:
        cl = rig.backend.begin()
        mm = G.kernel("matmul_bf16w")
        bad = [
            mm.encode(x=rig.tok["x"], w=rig.tok["w_w"], y=rig.tok["y"], m=8, n=8, k=8),  # y needs 64, x needs 64: ok
        ]
        ok = G.prepare(rig.table, mm.id, bad[0])
        words = (ctypes.c_uint32 * 32)(*ok.args.words())
        assert N.lib().lrm_cuda_dispatch(cl._h, mm.id, words) == N.LRM_OK
        too_big = ok.args.with_word(4, 9)  # m = 9: x holds 64 < 72 elements
        too_big = too_big.with_groups_x(1)
        words = (ctypes.c_uint32 * 32)(*too_big.words())
        assert N.lib().lrm_cuda_dispatch(cl._h, mm.id, words) == N.LRM_ERR_CONTRACT
        assert "touches" in N.last_error(rig.backend._h)
        words = (ctypes.c_uint32 * 32)(*ok.args.with_word(2, rig.tok["y"]).words())  # w must be bf16
        assert N.lib().lrm_cuda_dispatch(cl._h, mm.id, words) == N.LRM_ERR_CONTRACT
        words = (ctypes.c_uint32 * 32)(*ok.args.with_word(3, rig.tok["w_w"]).words())  # writes a read-only weight
        assert N.lib().lrm_cuda_dispatch(cl._h, mm.id, words) == N.LRM_ERR_CONTRACT
        words = (ctypes.c_uint32 * 32)(*ok.args.with_groups_x(5).words())  # word 0 is not the physical x
        assert N.lib().lrm_cuda_dispatch(cl._h, mm.id, words) == N.LRM_ERR_CONTRACT
        with pytest.raises(G.GpuContractException):
            cl.dispatch_named("attention_gqa_causal", q=rig.tok["x"], k=rig.tok["x"], v=rig.tok["x"], y=rig.tok["y"],
                              rows=1, q_row0=0, past=0, q_heads=3, kv_heads=2, head_dim=8, scale=1.0)
    finally:
        rig.close()


def test_copy_timers_and_single_use_lists():
    F = G.DType.F32
    rig = Rig({"a": (F, 1 << 16), "b": (F, 1 << 16)}, time_dispatches=True)
    try:
        a = np.arange(1 << 16, dtype=np.float32)
        rig.put("a", a)
        cl = rig.backend.begin()
        t = cl.begin_timer("gpu.test", [("case", "copy")])
        sa, oa, _ = rig.where["a"]
        sb, ob, _ = rig.where["b"]
        cl.copy(G.BufferRange(sa, oa, 1 << 18), G.BufferRange(sb, ob, 1 << 18))
        cl.dispatch_named("scale_f32", x=rig.tok["b"], y=rig.tok["b"], n=1 << 16, a=2.0)
        cl.end_timer(t)
        fence = rig.backend.submit(cl)
        comp = rig.backend.wait(fence)
        assert comp.dispatches == 1 and [x.name for x in comp.timers] == ["gpu.test", "gpu.dispatch"]
        assert all(x.duration_ns >= 0 for x in comp.timers)
        assert np.array_equal(f32(rig.get("b", np.uint32)), a * 2)
        assert rig.backend.wait(fence) is comp
        with pytest.raises(G.GpuContractException):
            rig.backend.submit(cl)
        with pytest.raises(G.GpuContractException):
            cl.barrier()
        with pytest.raises(G.GpuContractException):
            rig.heap.write_table(rig.table)
    finally:
        rig.close()
