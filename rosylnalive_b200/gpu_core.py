"""Host-side mirror of the reference's device/kernel contracts (src/Lrm.Gpu.Core), for the CUDA device.

The reference's F# host calls its shared rules (Dispatch.prepare and friends) before it hands a 128-byte argument
block to a backend. There is no .NET toolchain in this build, so this module restates those rules in Python, and the
CUDA device (cuda_backend.py over liblrmcuda.so) calls them exactly where the F# backends do. The C-ABI library
re-checks the parts a kernel's memory safety depends on (tokens, dtypes, bounds, element counts).

What is restated, with the reference file each part follows:
- ArgBlock, f32/i32 word bits, Grid folding above 65,535 groups ........ ArgBlock.fs:11-159
- the 14-kernel catalog (fields, threads, grids) ........................ Catalog/catalog.json (as data)
- HeapLayout / HeapPlanner / arenas ...................................... HeapLayout.fs
- TensorRow (64 bytes), TensorTable, SealedTable (1 MiB image) .......... TensorTable.fs:11-474
- Dispatch.prepare (token, aliasing and grid rules), checkCopy, checkTransfer ... Dispatch.fs:37-234
"""

from __future__ import annotations

import hashlib
import re
import struct
from dataclasses import dataclass, field
from enum import IntEnum, IntFlag


class GpuContractException(Exception):
    """A broken device/kernel contract rule (reference: src/Lrm.Gpu.Core/Errors.fs, Fail.contract)."""


def fail(msg: str, *args):
    raise GpuContractException(msg % args if args else msg)


# ---------------------------------------------------------------------------------------------------------------
# DType codes (Lrm.Core DType; heap-and-tensor-table.md "TensorRow" word 2).


class DType(IntEnum):
    F32 = 1
    BF16 = 2
    F16 = 3
    I32 = 4
    U32 = 5
    U8 = 6
    F64 = 7
    I64 = 8

    @property
    def size(self) -> int:
        return {1: 4, 2: 2, 3: 2, 4: 4, 5: 4, 6: 1, 7: 8, 8: 8}[int(self)]

    @property
    def label(self) -> str:
        return self.name.lower()


def dtype_of_name(name: str) -> DType:
    return DType[name.upper()]


# ---------------------------------------------------------------------------------------------------------------
# ArgBlock (ArgBlock.fs:11-92).


def f32_bits(x: float) -> int:
    return struct.unpack("<I", struct.pack("<f", x))[0]


def i32_bits(x: int) -> int:
    return x & 0xFFFFFFFF


class ArgBlock:
    """32 little-endian u32 words. Word 0 is lrm_groups_x (written by Dispatch); fields follow from word 1."""

    WORD_COUNT = 32
    BYTE_COUNT = 128

    def __init__(self, words=None):
        w = [0] * 32 if words is None else [int(x) & 0xFFFFFFFF for x in words]
        if len(w) != 32:
            fail("an argument block is 32 words")
        self._w = w

    @staticmethod
    def of_bytes(b: bytes) -> "ArgBlock":
        if len(b) != 128:
            fail("an argument block is 128 bytes, got %d", len(b))
        return ArgBlock(struct.unpack("<32I", b))

    def __getitem__(self, i):
        return self._w[i]

    @property
    def groups_x(self):
        return self._w[0]

    def with_word(self, i, v) -> "ArgBlock":
        w = list(self._w)
        w[i] = int(v) & 0xFFFFFFFF
        return ArgBlock(w)

    def with_groups_x(self, gx) -> "ArgBlock":
        return self.with_word(0, gx)

    def words(self):
        return list(self._w)

    def to_bytes(self) -> bytes:
        return struct.pack("<32I", *self._w)

    def __eq__(self, o):
        return isinstance(o, ArgBlock) and o._w == self._w

    def __repr__(self):
        return "ArgBlock(" + " ".join("%08x" % x for x in self._w) + ")"


# ---------------------------------------------------------------------------------------------------------------
# Grids (ArgBlock.fs:95-159).

MAX_DIMENSION = 65535


@dataclass(frozen=True)
class Grid:
    x: int
    y: int
    z: int


def ceildiv(a: int, b: int) -> int:
    if b < 1:
        fail("ceildiv by %d", b)
    if a < 0:
        fail("ceildiv of negative %d", a)
    return (a + b - 1) // b


def physical(linear: bool, g: Grid):
    """The dispatched grid for a logical one; returns (Grid, None) or (None, error)."""
    if g.x < 1 or g.y < 1 or g.z < 1:
        return None, "empty grid %dx%dx%d (every dimension must be at least 1)" % (g.x, g.y, g.z)
    if g.y > MAX_DIMENSION or g.z > MAX_DIMENSION:
        return None, "grid %dx%dx%d: y and z must be at most 65535" % (g.x, g.y, g.z)
    if g.x <= MAX_DIMENSION:
        return Grid(g.x, g.y, g.z), None
    if not linear:
        return None, "grid x of %d exceeds 65535 and the kernel's grid is not linear, so it cannot be folded" % g.x
    if g.x > MAX_DIMENSION * MAX_DIMENSION:
        return None, "grid x of %d exceeds 65535 * 65535" % g.x
    y = ceildiv(g.x, MAX_DIMENSION)
    x = ceildiv(g.x, y)
    return Grid(x, y, 1), None


# ---------------------------------------------------------------------------------------------------------------
# The kernel catalog (Catalog/catalog.json; kernel-abi.md "The catalog at contracts-v1"). KernelId i is KERNELS[i].


class Access(IntEnum):
    READ = 1
    WRITE = 2
    READWRITE = 3
    META = 4

    @property
    def writes(self):
        return self in (Access.WRITE, Access.READWRITE)


@dataclass(frozen=True)
class FieldSpec:
    name: str
    kind: str  # "token" | "u32" | "i32" | "f32"
    access: Access | None = None
    dtypes: tuple = ()
    alias: tuple = ()


@dataclass(frozen=True)
class KernelSpec:
    id: int
    name: str
    family: str
    threads: tuple
    grid_text: tuple
    fields: tuple

    @property
    def linear(self) -> bool:
        return self.grid_text[1] == "1" and self.grid_text[2] == "1"

    def field_index(self, name: str) -> int:
        for i, f in enumerate(self.fields):
            if f.name == name:
                return i
        raise KeyError(name)

    def grid_of(self, args: ArgBlock) -> Grid:
        env = {f.name: args[i + 1] for i, f in enumerate(self.fields) if f.kind == "u32"}
        return Grid(*(eval_grid(t, env) for t in self.grid_text))

    def encode(self, **values) -> ArgBlock:
        """A block from field values by name (tokens and u32 as ints, i32 as ints, f32 as floats); word 0 left 0."""
        w = [0] * 32
        for i, f in enumerate(self.fields):
            if f.name not in values:
                raise KeyError(f"{self.name}: missing field {f.name}")
            v = values.pop(f.name)
            if f.kind == "f32":
                w[i + 1] = f32_bits(float(v))
            elif f.kind == "i32":
                w[i + 1] = i32_bits(int(v))
            else:
                w[i + 1] = int(v) & 0xFFFFFFFF
        if values:
            raise KeyError(f"{self.name}: unknown fields {sorted(values)}")
        return ArgBlock(w)


_TOKEN_RE = re.compile(r"\s*(ceildiv\(|\(|\)|,|\+|\*|[a-z_][a-z0-9_]*|[0-9]+)")


def eval_grid(text: str, env: dict) -> int:
    """Evaluates a catalog grid formula (kernel-abi.md "Grids and folding" grammar) in Python integers."""
    toks = []
    pos = 0
    while pos < len(text):
        m = _TOKEN_RE.match(text, pos)
        if not m:
            raise ValueError(f"bad grid formula {text!r}")
        toks.append(m.group(1))
        pos = m.end()
        while pos < len(text) and text[pos] == " ":
            pos += 1
    it = iter(toks + [None])
    cur = [next(it)]

    def take():
        t = cur[0]
        cur[0] = next(it)
        return t

    def expr():
        v = term()
        while cur[0] == "+":
            take()
            v += term()
        return v

    def term():
        v = atom()
        while cur[0] == "*":
            take()
            v *= atom()
        return v

    def atom():
        t = take()
        if t == "ceildiv(":
            a = expr()
            assert take() == ","
            b = expr()
            assert take() == ")"
            return ceildiv(a, b)
        if t == "(":
            v = expr()
            assert take() == ")"
            return v
        if t.isdigit():
            return int(t)
        return int(env[t])

    return expr()


def _tok(name, access, dtypes, alias=()):
    return FieldSpec(name, "token", access, tuple(dtype_of_name(d) for d in dtypes), tuple(alias))


def _u(name):
    return FieldSpec(name, "u32")


def _f(name):
    return FieldSpec(name, "f32")


R, W, M = Access.READ, Access.WRITE, Access.META

KERNELS = (
    KernelSpec(0, "scale_f32", "selftest", (256, 1, 1), ("ceildiv(n, 256)", "1", "1"),
               (_tok("x", R, ["f32"]), _tok("y", W, ["f32"], ["x"]), _u("n"), _f("a"))),
    KernelSpec(1, "table_echo", "selftest", (16, 1, 1), ("1", "1", "1"),
               (FieldSpec("src", "token", M), _tok("y", W, ["u32"]))),
    KernelSpec(2, "args_echo", "selftest", (32, 1, 1), ("1", "1", "1"),
               (_tok("y", W, ["u32"]),) + tuple(_u(f"v{i}") for i in range(2, 32))),
    KernelSpec(3, "groups_echo", "selftest", (1, 1, 1), ("groups", "1", "1"), (_tok("y", W, ["u32"]), _u("groups"))),
    KernelSpec(4, "bf16_unpack", "selftest", (256, 1, 1), ("ceildiv(n, 256)", "1", "1"),
               (_tok("x", R, ["bf16"]), _tok("y", W, ["f32"]), _u("n"))),
    KernelSpec(5, "embed_gather_bf16", "basic", (256, 1, 1), ("ceildiv(cols, 256)", "rows", "1"),
               (_tok("ids", R, ["u32"]), _tok("table", R, ["bf16"]), _tok("y", W, ["f32"]), _u("rows"), _u("cols"),
                _u("vocab"))),
    KernelSpec(6, "rmsnorm_rows", "basic", (256, 1, 1), ("rows", "1", "1"),
               (_tok("x", R, ["f32"]), _tok("w", R, ["bf16"]), _tok("y", W, ["f32"], ["x"]), _u("rows"), _u("cols"),
                _f("eps"))),
    KernelSpec(7, "rope_apply", "basic", (64, 1, 1), ("rows", "1", "1"),
               (_tok("x", R, ["f32"]), _tok("cos_table", R, ["f32"]), _tok("sin_table", R, ["f32"]),
                _tok("y", W, ["f32"], ["x"]), _u("rows"), _u("heads"), _u("head_dim"), _u("pos0"))),
    KernelSpec(8, "silu_mul", "basic", (256, 1, 1), ("ceildiv(n, 256)", "1", "1"),
               (_tok("gate", R, ["f32"]), _tok("up", R, ["f32"]), _tok("y", W, ["f32"], ["gate", "up"]), _u("n"))),
    KernelSpec(9, "add", "basic", (256, 1, 1), ("ceildiv(n, 256)", "1", "1"),
               (_tok("a", R, ["f32"]), _tok("b", R, ["f32"]), _tok("y", W, ["f32"], ["a", "b"]), _u("n"))),
    KernelSpec(10, "copy_rows", "basic", (256, 1, 1), ("ceildiv(rows * cols, 256)", "1", "1"),
               (_tok("src", R, ["f32", "u32", "i32"]), _tok("dst", W, ["f32", "u32", "i32"]), _u("rows"), _u("cols"),
                _u("src_row0"), _u("dst_row0"), _u("src_stride"), _u("dst_stride"))),
    KernelSpec(11, "argmax_rows", "basic", (256, 1, 1), ("rows", "1", "1"),
               (_tok("x", R, ["f32"]), _tok("y", W, ["u32"]), _u("rows"), _u("cols"))),
    KernelSpec(12, "matmul_bf16w", "matmul", (16, 16, 1), ("ceildiv(n, 64)", "ceildiv(m, 64)", "1"),
               (_tok("x", R, ["f32"]), _tok("w", R, ["bf16"]), _tok("y", W, ["f32"]), _u("m"), _u("n"), _u("k"))),
    KernelSpec(13, "attention_gqa_causal", "attention", (64, 1, 1), ("rows", "q_heads", "1"),
               (_tok("q", R, ["f32"]), _tok("k", R, ["f32"]), _tok("v", R, ["f32"]), _tok("y", W, ["f32"]),
                _u("rows"), _u("q_row0"), _u("past"), _u("q_heads"), _u("kv_heads"), _u("head_dim"), _f("scale"))),
)

KERNEL_BY_NAME = {k.name: k for k in KERNELS}


def kernel(name_or_id) -> KernelSpec:
    if isinstance(name_or_id, int):
        if name_or_id < 0 or name_or_id >= len(KERNELS):
            fail("kernel %d is not in the catalog (%d kernels)", name_or_id, len(KERNELS))
        return KERNELS[name_or_id]
    return KERNEL_BY_NAME[name_or_id]


# ---------------------------------------------------------------------------------------------------------------
# Heap, arenas and layout (HeapLayout.fs; heap-and-tensor-table.md "The heap", "Arenas", "HeapLayout").

SLOT_COUNT = 64
TABLE_SLOT = 0
TABLE_ROWS = 16384
ROW_BYTES = 64
TABLE_BYTES = TABLE_ROWS * ROW_BYTES
MAX_PAGE_BYTES = 1 << 30
PAGE_GRANULARITY = 64 << 10
ALLOCATION_ALIGNMENT = 256


class ArenaKind(IntEnum):
    WEIGHTS = 1
    ROPE = 2
    KV_CACHE = 3
    ACTIVATIONS = 4
    SCRATCH = 5
    LOGITS = 6
    TAPS = 7
    MASTER = 8
    GRAD = 9
    ADAM_M = 10
    ADAM_V = 11
    ROSLYN_IN = 12
    ROSLYN_OUT = 13

    @property
    def reserved(self):
        return self >= ArenaKind.MASTER


def align_up(a: int, v: int) -> int:
    return (v + a - 1) // a * a


@dataclass(frozen=True)
class Page:
    slot: int
    arena: ArenaKind
    index: int
    bytes: int


class HeapLayout:
    """Pages in slots 1..N in contract arena order; slot 0 is the table."""

    def __init__(self, pages):
        self.pages = tuple(pages)

    @staticmethod
    def of_pages(pages) -> "HeapLayout":
        pages = [(ArenaKind(k), int(b)) for k, b in pages]
        if len(pages) > SLOT_COUNT - 1:
            fail("%d pages: at most 63", len(pages))
        last = 0
        out = []
        counts = {}
        for i, (kind, b) in enumerate(pages):
            if b < PAGE_GRANULARITY or b > MAX_PAGE_BYTES or b % PAGE_GRANULARITY:
                fail("page %d: %d bytes is not a multiple of 64 KiB from 64 KiB to 1 GiB", i, b)
            if kind.reserved:
                fail("arena %s is reserved until contracts-v2", kind.name.lower())
            if kind < last:
                fail("arenas must appear in contract order (%s after a later kind)", kind.name.lower())
            last = kind
            idx = counts.get(kind, 0)
            counts[kind] = idx + 1
            out.append(Page(i + 1, kind, idx, b))
        return HeapLayout(out)

    @property
    def page_count(self):
        return len(self.pages)

    def page(self, slot: int) -> Page:
        if slot < 1 or slot > len(self.pages):
            fail("slot %d holds no page", slot)
        return self.pages[slot - 1]

    def try_page(self, slot: int):
        return self.pages[slot - 1] if 1 <= slot <= len(self.pages) else None

    def slot_of(self, arena: ArenaKind, index: int) -> int:
        for p in self.pages:
            if p.arena == arena and p.index == index:
                return p.slot
        fail("no page %d in arena %s", index, ArenaKind(arena).name.lower())

    def arena_bytes(self, arena: ArenaKind) -> int:
        return sum(p.bytes for p in self.pages if p.arena == arena)

    @property
    def total_bytes(self):
        return TABLE_BYTES + sum(p.bytes for p in self.pages)

    def __eq__(self, o):
        return isinstance(o, HeapLayout) and o.pages == self.pages


@dataclass(frozen=True)
class Placement:
    arena: ArenaKind
    page: int
    offset: int
    bytes: int


class HeapPlanner:
    """Pass one of a static plan (heap-and-tensor-table.md "HeapPlanner"): allocations at the end of the arena's last
    page, 256-byte aligned, else at offset 0 of a new page; never straddling pages."""

    def __init__(self, page_bytes: int = MAX_PAGE_BYTES):
        if page_bytes < PAGE_GRANULARITY or page_bytes > MAX_PAGE_BYTES or page_bytes % PAGE_GRANULARITY:
            fail("page size %d", page_bytes)
        self.page_bytes = page_bytes
        self._fill = {}  # arena -> list of used bytes per page
        self._built = False

    def allocate(self, arena: ArenaKind, nbytes: int) -> Placement:
        if self._built:
            fail("the planner is built")
        arena = ArenaKind(arena)
        if arena.reserved:
            fail("arena %s is reserved until contracts-v2", arena.name.lower())
        if nbytes < 1 or nbytes > self.page_bytes:
            fail("an allocation of %d bytes does not fit one page of %d", nbytes, self.page_bytes)
        pages = self._fill.setdefault(arena, [])
        if pages:
            off = align_up(ALLOCATION_ALIGNMENT, pages[-1])
            if off + nbytes <= self.page_bytes:
                pages[-1] = off + nbytes
                return Placement(arena, len(pages) - 1, off, nbytes)
        pages.append(nbytes)
        return Placement(arena, len(pages) - 1, 0, nbytes)

    def build(self) -> HeapLayout:
        self._built = True
        out = []
        for arena in sorted(self._fill):
            for used in self._fill[arena]:
                out.append((arena, max(PAGE_GRANULARITY, align_up(PAGE_GRANULARITY, used))))
        return HeapLayout.of_pages(out)


# ---------------------------------------------------------------------------------------------------------------
# Tensor rows and the table (TensorTable.fs).


class TensorFlags(IntFlag):
    NONE = 0
    CONTIGUOUS = 1
    READ_ONLY = 2
    VIEW = 4


def debug_id_of(name: str) -> int:
    if not name:
        return 0
    return struct.unpack("<I", hashlib.sha256(name.encode("utf-8")).digest()[:4])[0]


def packed_strides(dims):
    out = []
    acc = 1
    for d in reversed(dims):
        out.append(acc)
        acc *= d
    return list(reversed(out))


class TensorRow:
    """One 64-byte row of 16 little-endian u32 words (TensorTable.fs:45-118)."""

    def __init__(self, words):
        if len(words) != 16:
            fail("a tensor row is 16 words")
        self.w = [int(x) & 0xFFFFFFFF for x in words]

    ZERO_WORDS = [0] * 16

    @staticmethod
    def zero():
        return TensorRow([0] * 16)

    @staticmethod
    def create(slot, byte_offset, dtype: DType, dims, flags=TensorFlags.NONE, debug_id=0, strides=None):
        rank = len(dims)
        if rank < 1 or rank > 4:
            fail("tensor rank %d is outside 1..4", rank)
        strides = packed_strides(dims) if strides is None else list(strides)
        if len(strides) != rank:
            fail("%d strides for rank %d", len(strides), rank)
        if any(d < 1 or d > 0xFFFFFFFF for d in dims):
            fail("tensor dims %s must each be 1..2^32-1", dims)
        if any(s < 0 or s > 0xFFFFFFFF for s in strides):
            fail("tensor strides %s must each be 0..2^32-1", strides)
        if byte_offset < 0 or byte_offset > 0xFFFFFFFF:
            fail("byte offset %d does not fit in u32", byte_offset)
        count = 1
        for d in dims:
            count *= d
        if count > 0xFFFFFFFF:
            fail("tensor of %d elements does not fit a u32 count", count)
        contiguous = TensorFlags.CONTIGUOUS if strides == packed_strides(dims) else TensorFlags.NONE
        w = [0] * 16
        w[0] = slot
        w[1] = byte_offset
        w[2] = int(dtype)
        w[3] = rank
        for i in range(4):
            w[4 + i] = dims[i] if i < rank else 1
            w[8 + i] = strides[i] if i < rank else 0
        w[12] = count
        w[13] = int((TensorFlags(flags) & ~TensorFlags.CONTIGUOUS) | contiguous)
        w[14] = debug_id
        return TensorRow(w)

    slot = property(lambda s: s.w[0])
    byte_offset = property(lambda s: s.w[1])
    dtype_code = property(lambda s: s.w[2])
    rank = property(lambda s: s.w[3])
    count = property(lambda s: s.w[12])
    flags = property(lambda s: TensorFlags(s.w[13] & 7))
    debug_id = property(lambda s: s.w[14])

    @property
    def dtype(self):
        try:
            return DType(self.w[2])
        except ValueError:
            return None

    def dims(self):
        return self.w[4:4 + self.rank]

    def strides(self):
        return self.w[8:8 + self.rank]

    @property
    def is_zero(self):
        return all(x == 0 for x in self.w)

    def to_bytes(self):
        return struct.pack("<16I", *self.w)

    def span_elements(self):
        return 1 + sum((self.w[4 + i] - 1) * self.w[8 + i] for i in range(self.rank))

    def extent_bytes(self):
        dt = self.dtype
        return align_up(4, self.span_elements() * dt.size) if dt else 0

    def validate(self, layout: HeapLayout):
        problems = []
        if self.slot < 1 or self.slot >= SLOT_COUNT:
            problems.append("slot %d is outside 1..63" % self.slot)
        elif layout.try_page(self.slot) is None:
            problems.append("slot %d holds no page in the layout" % self.slot)
        dt = self.dtype
        if dt is None:
            problems.append("dtype code %d is not a DType" % self.dtype_code)
        elif self.byte_offset % max(4, dt.size):
            problems.append("byte offset %d is not a multiple of %d" % (self.byte_offset, max(4, dt.size)))
        if self.rank < 1 or self.rank > 4:
            problems.append("rank %d is outside 1..4" % self.rank)
        else:
            for i in range(4):
                if i < self.rank and self.w[4 + i] < 1:
                    problems.append("dims[%d] is 0" % i)
                if i >= self.rank and (self.w[4 + i] != 1 or self.w[8 + i] != 0):
                    problems.append("unused dims[%d] must be 1 with stride 0" % i)
            prod = 1
            for d in self.dims():
                prod *= d
            if prod != self.count:
                problems.append("element count %d is not the product of the dims (%d)" % (self.count, prod))
            if bool(self.w[13] & 1) != (packed_strides(self.dims()) == self.strides()):
                problems.append("the Contiguous flag must be set exactly when the strides are packed row-major")
        if self.w[13] & ~7:
            problems.append("flags 0x%x use reserved bits" % self.w[13])
        if self.w[15] != 0:
            problems.append("word 15 is reserved and must be 0")
        if not problems:
            page = layout.page(self.slot)
            end = self.byte_offset + self.extent_bytes()
            if end > page.bytes:
                problems.append("extent ends at byte %d, past the %d-byte page in slot %d" % (end, page.bytes,
                                                                                               self.slot))
        return problems


class SealedTable:
    def __init__(self, layout, rows, names):
        self.layout = layout
        self._rows = rows
        self._names = names
        img = bytearray(TABLE_BYTES)
        for i, r in enumerate(rows):
            img[i * ROW_BYTES:(i + 1) * ROW_BYTES] = r.to_bytes()
        self.image = bytes(img)
        self.id = hashlib.sha256(self.image).hexdigest()
        self._by_name = {n: i for i, n in enumerate(names) if i > 0}

    @property
    def count(self):
        return len(self._rows) - 1

    def row(self, token: int) -> TensorRow:
        if token >= TABLE_ROWS or token < 0:
            fail("token %d is outside 0..%d", token, TABLE_ROWS - 1)
        return self._rows[token] if token < len(self._rows) else TensorRow.zero()

    def is_assigned(self, token: int) -> bool:
        return 1 <= token < len(self._rows)

    def name(self, token: int) -> str:
        return self._names[token] if token < len(self._names) else ""

    def find(self, name: str):
        return self._by_name.get(name)


class TensorTable:
    """Pass two of a static plan: rows under unique names, tokens 1, 2, ...; sealed once."""

    def __init__(self, layout: HeapLayout):
        self.layout = layout
        self._rows = [TensorRow.zero()]
        self._names = [""]
        self._sealed = None

    @property
    def count(self):
        return len(self._rows) - 1

    def row(self, token):
        if token < len(self._rows):
            return self._rows[token]
        fail("token %d has not been added", token)

    def add_row(self, name: str, row: TensorRow) -> int:
        if self._sealed is not None:
            fail("the tensor table is sealed")
        if not name:
            fail("a tensor needs a name")
        if name in self._names:
            fail("tensor name '%s' is already in the table", name)
        if len(self._rows) >= TABLE_ROWS:
            fail("the tensor table is full (%d rows)", TABLE_ROWS - 1)
        problems = row.validate(self.layout)
        if problems:
            fail("tensor '%s': %s", name, "; ".join(problems))
        self._rows.append(row)
        self._names.append(name)
        return len(self._rows) - 1

    def add(self, name: str, placement: Placement, dtype: DType, dims, flags=TensorFlags.NONE) -> int:
        slot = self.layout.slot_of(placement.arena, placement.page)
        row = TensorRow.create(slot, placement.offset, dtype, list(dims), flags, debug_id_of(name))
        if row.extent_bytes() > align_up(4, placement.bytes):
            fail("tensor '%s' needs %d bytes but its placement has %d", name, row.extent_bytes(), placement.bytes)
        return self.add_row(name, row)

    def add_view(self, name: str, source: int, dims, element_offset: int) -> int:
        src = self.row(source)
        if src.is_zero:
            fail("cannot view the null token")
        dt = src.dtype
        offset = src.byte_offset + element_offset * dt.size
        row = TensorRow.create(src.slot, offset, dt, list(dims), TensorFlags.VIEW | (src.flags & TensorFlags.READ_ONLY),
                               debug_id_of(name))
        if element_offset < 0 or offset + row.extent_bytes() > src.byte_offset + src.extent_bytes():
            fail("view '%s' does not lie inside its source t%d", name, source)
        return self.add_row(name, row)

    def seal(self) -> SealedTable:
        if self._sealed is not None:
            fail("the tensor table is sealed")
        self._sealed = SealedTable(self.layout, list(self._rows), list(self._names))
        return self._sealed


# ---------------------------------------------------------------------------------------------------------------
# Dispatch rules (Dispatch.fs).


@dataclass
class TokenUse:
    field: str
    access: Access
    token: int
    row: TensorRow
    slot: int
    start: int
    end: int


@dataclass
class PreparedDispatch:
    kernel: KernelSpec
    grid: Grid
    physical: Grid
    args: ArgBlock
    tokens: list


def resolve_tokens(table: SealedTable, k: KernelSpec, args: ArgBlock):
    uses = []
    for i, f in enumerate(k.fields):
        if f.kind != "token":
            continue
        token = args[i + 1]
        row = table.row(token)
        if f.access == Access.META:
            if token != 0 and not table.is_assigned(token):
                fail("%s.%s: token %d is not in the table", k.name, f.name, token)
        else:
            if token == 0:
                fail("%s.%s: the null token is not allowed here", k.name, f.name)
            if not table.is_assigned(token):
                fail("%s.%s: token %d is not in the table", k.name, f.name, token)
            if row.dtype not in f.dtypes:
                fail("%s.%s: tensor '%s' is %s, the kernel accepts %s", k.name, f.name, table.name(token),
                     row.dtype.label if row.dtype else "invalid", ", ".join(d.label for d in f.dtypes))
            if not (row.flags & TensorFlags.CONTIGUOUS):
                fail("%s.%s: tensor '%s' is not contiguous", k.name, f.name, table.name(token))
            if f.access.writes and (row.flags & TensorFlags.READ_ONLY):
                fail("%s.%s: tensor '%s' is read only", k.name, f.name, table.name(token))
        start = row.byte_offset
        uses.append(TokenUse(f.name, f.access, token, row, row.slot, start, start + row.extent_bytes()))
    return uses


def check_aliasing(k: KernelSpec, uses):
    data = [u for u in uses if u.access != Access.META]

    def alias_of(fname):
        for f in k.fields:
            if f.name == fname:
                return f.alias
        return ()

    for i in range(len(data)):
        for j in range(i + 1, len(data)):
            a, b = data[i], data[j]
            overlap = a.slot == b.slot and a.start < b.end and b.start < a.end
            if overlap and (a.access.writes or b.access.writes):
                same = a.start == b.start and a.end == b.end
                declared = (a.access.writes and not b.access.writes and b.field in alias_of(a.field)) or \
                           (b.access.writes and not a.access.writes and a.field in alias_of(b.field))
                if not (declared and same):
                    fail("%s: %s and %s overlap in slot %d, and %s", k.name, a.field, b.field, a.slot,
                         "a declared alias must span exactly the same bytes" if declared
                         else "the catalog does not let them alias")


def prepare(table: SealedTable, kernel_id: int, args: ArgBlock) -> PreparedDispatch:
    """Dispatch.prepare (Dispatch.fs:149-173): word rules, token rules, aliasing, grid with word 0 written."""
    k = kernel(kernel_id)
    if args[0] != 0:
        fail("%s: argument word 0 is lrm_groups_x, which Dispatch writes; pass 0", k.name)
    for w in range(len(k.fields) + 1, 32):
        if args[w] != 0:
            fail("%s: argument word %d is past the last field and must be 0", k.name, w)
    uses = resolve_tokens(table, k, args)
    check_aliasing(k, uses)
    g = k.grid_of(args)
    p, err = physical(k.linear, g)
    if err:
        fail("%s: %s", k.name, err)
    return PreparedDispatch(k, g, p, args.with_groups_x(p.x), uses)


@dataclass(frozen=True)
class BufferRange:
    slot: int
    offset: int
    bytes: int


def check_copy(layout: HeapLayout, src: BufferRange, dst: BufferRange):
    for what, r in (("source", src), ("destination", dst)):
        if r.slot < 1 or r.slot >= SLOT_COUNT:
            fail("copy %s: slot %d is not a page slot (1..63)", what, r.slot)
        page = layout.page(r.slot)
        if r.offset < 0 or r.bytes <= 0 or r.offset % 4 or r.bytes % 4:
            fail("copy %s: offset %d and size %d must be multiples of 4, size > 0", what, r.offset, r.bytes)
        if r.offset + r.bytes > page.bytes:
            fail("copy %s: bytes %d..%d are past the %d-byte page", what, r.offset, r.offset + r.bytes, page.bytes)
    if src.bytes != dst.bytes:
        fail("copy: source has %d bytes, destination %d", src.bytes, dst.bytes)
    if src.slot == dst.slot and src.offset < dst.offset + dst.bytes and dst.offset < src.offset + src.bytes:
        fail("copy: source and destination overlap in slot %d", src.slot)


def check_transfer(layout: HeapLayout, allow_table: bool, slot: int, offset: int, nbytes: int):
    if slot == TABLE_SLOT and allow_table:
        size = TABLE_BYTES
    elif slot == TABLE_SLOT:
        fail("slot 0 holds the tensor table; write it with WriteTable")
    elif slot < 1 or slot >= SLOT_COUNT:
        fail("slot %d is outside 0..63", slot)
    else:
        size = layout.page(slot).bytes
    if offset < 0 or nbytes < 0 or offset % 4 or nbytes % 4:
        fail("transfer in slot %d: offset %d and size %d must be non-negative multiples of 4", slot, offset, nbytes)
    if offset + nbytes > size:
        fail("transfer in slot %d: bytes %d..%d are past the %d-byte buffer", slot, offset, offset + nbytes, size)
