"""The host-side contract mirror against the reference's own vectors.

Vectors: kernel-abi.md "Vectors" (A1-A4, folding edge cases) and heap-and-tensor-table.md "Vectors" (T1, T2, the
null row, the table image). The dispatch-rule cases follow tests/Lrm.Gpu.Core.Tests/BackendTests.fs's list:
word 0, trailing words, tokens, dtypes, read-only, contiguity, aliasing, grid folding.
"""

import struct

import pytest

from rosylnalive_b200 import gpu_core as G


def words_hex(block):
    return " ".join(struct.pack("<I", w).hex() for w in block.words())


def layout_one_page():
    return G.HeapLayout.of_pages([(G.ArenaKind.ACTIVATIONS, 1 << 20)])


def test_vector_a1_scale_f32():
    k = G.kernel("scale_f32")
    table = fake_table(["f32", "f32"], base_token=5)
    b = k.encode(x=5, y=6, n=1000, a=0.5)
    p = G.prepare(table, k.id, b)
    assert words_hex(p.args).startswith("04000000 05000000 06000000 e8030000 0000003f")
    assert p.args.words()[5:] == [0] * 27
    assert p.physical == G.Grid(4, 1, 1)


def test_vector_a2_matmul():
    k = G.kernel("matmul_bf16w")
    b = k.encode(x=1, w=2, y=3, m=37, n=151936, k=1024)
    g = k.grid_of(b)
    p, err = G.physical(k.linear, g)
    assert err is None and p == G.Grid(2374, 1, 1)
    assert words_hex(b.with_groups_x(p.x)) .startswith(
        "46090000 01000000 02000000 03000000 25000000 80510200 00040000")


def test_vector_a3_add_folded():
    k = G.kernel("add")
    b = k.encode(a=1, b=2, y=3, n=8192 * 3072)
    g = k.grid_of(b)
    assert g.x == 98304
    p, err = G.physical(k.linear, g)
    assert p == G.Grid(49152, 2, 1)
    assert words_hex(b.with_groups_x(p.x)).startswith("00c00000 01000000 02000000 03000000 00008001")


def test_vector_a4_attention():
    k = G.kernel("attention_gqa_causal")
    b = k.encode(q=1, k=2, v=3, y=4, rows=7, q_row0=0, past=0, q_heads=16, kv_heads=8, head_dim=128,
                 scale=1 / 128 ** 0.5)
    p, err = G.physical(k.linear, k.grid_of(b))
    assert p == G.Grid(7, 16, 1)
    assert words_hex(b.with_groups_x(p.x)) == (
        "07000000 01000000 02000000 03000000 04000000 07000000 00000000 00000000 10000000 08000000 80000000 f304b53d"
        + " 00000000" * 20)


@pytest.mark.parametrize("x,expect", [(65535, (65535, 1, 1)), (65536, (32768, 2, 1)), (70000, (35000, 2, 1))])
def test_folding_edges(x, expect):
    p, err = G.physical(True, G.Grid(x, 1, 1))
    assert (p.x, p.y, p.z) == expect
    assert p.x * p.y - x < p.y


def test_folding_refused_for_non_linear_and_empty():
    assert G.physical(False, G.Grid(70000, 1, 1))[1] is not None
    assert G.physical(True, G.Grid(0, 1, 1))[1] is not None
    assert G.physical(True, G.Grid(1, 65536, 1))[1] is not None


def test_linear_kernels():
    assert {k.name for k in G.KERNELS if k.linear} == {
        "scale_f32", "table_echo", "args_echo", "groups_echo", "bf16_unpack", "rmsnorm_rows", "rope_apply",
        "silu_mul", "add", "copy_rows", "argmax_rows"}


def test_vector_t1_embedding_row():
    layout = G.HeapLayout.of_pages([(G.ArenaKind.WEIGHTS, 1 << 30)])
    row = G.TensorRow.create(1, 256, G.DType.BF16, [151936, 1024], G.TensorFlags.READ_ONLY,
                             G.debug_id_of("model.embed_tokens.weight"))
    assert row.to_bytes().hex() == (
        "01000000" "00010000" "02000000" "02000000" "80510200" "00040000" "01000000" "01000000"
        "00040000" "01000000" "00000000" "00000000" "00004609" "03000000" "fcd443ac" "00000000")
    assert row.validate(layout) == []


def test_vector_t2_view_row():
    row = G.TensorRow.create(4, 4096, G.DType.F32, [7, 16, 128], G.TensorFlags.VIEW, G.debug_id_of("L0.attn.q_rope"))
    assert row.to_bytes().hex() == (
        "04000000" "00100000" "01000000" "03000000" "07000000" "10000000" "80000000" "01000000"
        "00080000" "80000000" "01000000" "00000000" "00380000" "05000000" "d4fd8611" "00000000")


def test_table_image_layout():
    layout = layout_one_page()
    t = G.TensorTable(layout)
    pl = G.HeapPlanner(1 << 20)
    a = t.add("a", G.Placement(G.ArenaKind.ACTIVATIONS, 0, 0, 64), G.DType.F32, [16])
    b = t.add("b", G.Placement(G.ArenaKind.ACTIVATIONS, 0, 256, 64), G.DType.F32, [16])
    s = t.seal()
    assert (a, b) == (1, 2)
    assert s.image[:64] == bytes(64)
    assert s.image[64:128] == s.row(1).to_bytes()
    assert s.image[192:] == bytes(len(s.image) - 192)
    with pytest.raises(G.GpuContractException):
        t.seal()


def test_planner_places_and_rounds():
    p = G.HeapPlanner(1 << 20)
    a = p.allocate(G.ArenaKind.WEIGHTS, 100)
    b = p.allocate(G.ArenaKind.WEIGHTS, 100)
    c = p.allocate(G.ArenaKind.WEIGHTS, (1 << 20) - 100)
    d = p.allocate(G.ArenaKind.ROPE, 10)
    assert (a.offset, b.offset, c.page, c.offset) == (0, 256, 1, 0)
    lay = p.build()
    assert [(pg.arena, pg.bytes) for pg in lay.pages] == [(G.ArenaKind.WEIGHTS, 65536), (G.ArenaKind.WEIGHTS, 1 << 20),
                                                          (G.ArenaKind.ROPE, 65536)]
    with pytest.raises(G.GpuContractException):
        p.allocate(G.ArenaKind.WEIGHTS, 4)
    with pytest.raises(G.GpuContractException):
        G.HeapPlanner().allocate(G.ArenaKind.GRAD, 4)


def fake_table(dtypes, base_token=1, flags=None):
    """A table whose tokens base_token.. are 64-element tensors of the given dtypes, 256 bytes apart."""
    layout = layout_one_page()
    t = G.TensorTable(layout)
    for i in range(1, base_token):
        t.add(f"pad{i}", G.Placement(G.ArenaKind.ACTIVATIONS, 0, 0x10000 + 256 * i, 4), G.DType.F32, [1])
    for i, d in enumerate(dtypes):
        f = (flags or {}).get(i, G.TensorFlags.NONE)
        t.add(f"t{i}", G.Placement(G.ArenaKind.ACTIVATIONS, 0, 1024 * i, 256), G.dtype_of_name(d), [64], f)
    return t.seal()


def test_dispatch_rules():
    table = fake_table(["f32", "f32", "bf16"], flags={1: G.TensorFlags.READ_ONLY})
    k = G.kernel("scale_f32")
    G.prepare(table, k.id, k.encode(x=1, y=1, n=64, a=2.0))  # declared alias, same bytes: in place is fine
    bad = [
        k.encode(x=1, y=2, n=64, a=1.0),  # y is read only
        k.encode(x=3, y=1, n=64, a=1.0),  # bf16 where f32 is required
        k.encode(x=0, y=1, n=64, a=1.0),  # null token
        k.encode(x=9, y=1, n=64, a=1.0),  # unassigned token
        k.encode(x=1, y=1, n=0, a=1.0),  # empty grid
        k.encode(x=1, y=1, n=64, a=1.0).with_groups_x(1),  # word 0 must be 0
        k.encode(x=1, y=1, n=64, a=1.0).with_word(7, 1),  # trailing word
    ]
    for b in bad:
        with pytest.raises(G.GpuContractException):
            G.prepare(table, k.id, b)


def test_aliasing_rule():
    layout = layout_one_page()
    t = G.TensorTable(layout)
    a = t.add("a", G.Placement(G.ArenaKind.ACTIVATIONS, 0, 0, 256), G.DType.F32, [64])
    half = t.add_view("a.half", a, [32], 0)
    b = t.add("b", G.Placement(G.ArenaKind.ACTIVATIONS, 0, 1024, 256), G.DType.F32, [64])
    s = t.seal()
    add = G.kernel("add")
    G.prepare(s, add.id, add.encode(a=a, b=b, y=a, n=64))
    with pytest.raises(G.GpuContractException):  # overlapping but not the same bytes
        G.prepare(s, add.id, add.encode(a=a, b=b, y=half, n=32))
    mm = G.kernel("matmul_bf16w")
    with pytest.raises(G.GpuContractException):
        G.prepare(s, mm.id, mm.encode(x=a, w=a, y=a, m=1, n=1, k=1))


def test_copy_and_transfer_rules():
    layout = G.HeapLayout.of_pages([(G.ArenaKind.WEIGHTS, 65536), (G.ArenaKind.ACTIVATIONS, 65536)])
    G.check_copy(layout, G.BufferRange(1, 0, 64), G.BufferRange(2, 0, 64))
    for src, dst in [((1, 0, 64), (1, 32, 64)), ((0, 0, 4), (1, 0, 4)), ((1, 2, 4), (2, 0, 4)),
                     ((1, 0, 8), (2, 0, 4)), ((1, 65532, 8), (2, 0, 8))]:
        with pytest.raises(G.GpuContractException):
            G.check_copy(layout, G.BufferRange(*src), G.BufferRange(*dst))
    G.check_transfer(layout, True, 0, 0, G.TABLE_BYTES)
    with pytest.raises(G.GpuContractException):
        G.check_transfer(layout, False, 0, 0, 4)
    with pytest.raises(G.GpuContractException):
        G.check_transfer(layout, False, 1, 65532, 8)


def test_layout_rules():
    with pytest.raises(G.GpuContractException):
        G.HeapLayout.of_pages([(G.ArenaKind.ROPE, 65536), (G.ArenaKind.WEIGHTS, 65536)])
    with pytest.raises(G.GpuContractException):
        G.HeapLayout.of_pages([(G.ArenaKind.WEIGHTS, 1000)])
    with pytest.raises(G.GpuContractException):
        G.HeapLayout.of_pages([(G.ArenaKind.WEIGHTS, 65536)] * 64)
