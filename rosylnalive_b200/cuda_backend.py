"""The CUDA device as an IGpuBackendProvider / IGpuBackend (reference: src/Lrm.Gpu.Core/Backend.fs:96-161,
docs/contracts/gpu-backend.md), over liblrmcuda.so.

This is the Python twin of the planned F# ``Lrm.Gpu.Cuda`` project: the same members with the same meaning and the
same errors. Contract violations raise ``GpuContractException`` from the shared rules (gpu_core.prepare,
check_copy, check_transfer) before the native call; the native library re-checks the safety-relevant parts.
"""

from __future__ import annotations

import ctypes
import hashlib
import io
import platform
from dataclasses import dataclass, field

import numpy as np

from . import gpu_core as G
from . import native as N

BACKEND = "cuda"

# Fp32Denormals.probeInputs (Backend.fs:472-481) and the two expected result sets (Preserve, Flush).
PROBE_INPUTS = [0x3F800000, 0x01000000, 0x00800000, 0x80800000, 0x00000002, 0x807FFFFE, 0x00400000]
PROBE_PRESERVE = [0x3F000000, 0x00800000, 0x00400000, 0x80400000, 0x00000001, 0x803FFFFF, 0x00200000]
PROBE_FLUSH = [0x3F000000, 0x00800000, 0x00000000, 0x80000000, 0x00000000, 0x80000000, 0x00000000]


def classify_denormals(results) -> str:
    """Fp32Denormals.classify (Backend.fs:497-512)."""
    r = [int(x) for x in results]
    if len(r) != 7:
        G.fail("the fp32 denormal probe needs 7 results")
    if r[0] != PROBE_PRESERVE[0] or r[1] != PROBE_PRESERVE[1]:
        G.fail("the fp32 denormal probe's normal controls are wrong: scale_f32 itself failed")
    if r == PROBE_PRESERVE:
        return "preserve"
    if r == PROBE_FLUSH:
        return "flush"
    return "mixed"


@dataclass
class DeviceInfo:
    backend: str
    index: int
    name: str
    vendor_id: int
    pci_device_id: int
    driver: str
    memory_bytes: int
    details: list = field(default_factory=list)


@dataclass
class DeviceCandidate:
    info: DeviceInfo
    rejections: list

    @property
    def accepted(self):
        return not self.rejections


@dataclass
class DeviceOptions:
    backend: str = BACKEND
    index: int | None = None
    debug: bool = False
    time_dispatches: bool = False


@dataclass
class ExecutionClass:
    backend: str
    device_id: str
    driver: str
    shader_set_hash: str | None
    arch: str


@dataclass
class TimerResult:
    name: str
    attrs: list
    gpu_start_ns: int
    duration_ns: int


@dataclass
class Completion:
    submission: int
    dispatches: int
    timers: list


class KernelSet:
    """IKernelSet (Backend.fs:96-100)."""

    def __init__(self, backend, set_hash: bytes):
        self._backend = backend
        self.shader_set_hash = set_hash.hex()

    def contains(self, kernel_id: int) -> bool:
        present = ctypes.c_int32(0)
        N.check(N.lib().lrm_cuda_kernel_present(self._backend._h, int(kernel_id), ctypes.byref(present)),
                self._backend._h)
        return bool(present.value)


class CudaHeap:
    """IGpuHeap (Backend.fs:102-116)."""

    UPLOAD_CHUNK = 64 << 20

    def __init__(self, backend, layout: G.HeapLayout):
        self._b = backend
        self.layout = layout
        self.table: G.SealedTable | None = None

    def write_table(self, table: G.SealedTable):
        if self.table is not None:
            G.fail("WriteTable is called exactly once")
        if table.layout != self.layout:
            G.fail("the table was built against another layout")
        img = np.frombuffer(table.image, np.uint8)
        N.check(N.lib().lrm_cuda_write_table(self._b._h, N.ptr(img), len(table.image)), self._b._h, "WriteTable")
        self.table = table

    def upload(self, slot: int, offset: int, data):
        buf = np.ascontiguousarray(np.frombuffer(memoryview(data).cast("B"), np.uint8))
        G.check_transfer(self.layout, False, slot, offset, buf.nbytes)
        N.check(N.lib().lrm_cuda_upload(self._b._h, slot, offset, N.ptr(buf), buf.nbytes), self._b._h, "Upload")

    def upload_array(self, slot: int, offset: int, arr: np.ndarray):
        arr = np.ascontiguousarray(arr)
        self.upload(slot, offset, arr.view(np.uint8).reshape(-1))

    def upload_from(self, slot: int, offset: int, source: io.RawIOBase, length: int):
        """UploadFrom: `length` bytes of a stream, staged in chunks of at most 64 MiB."""
        G.check_transfer(self.layout, False, slot, offset, length)
        done = 0
        while done < length:
            n = min(self.UPLOAD_CHUNK, length - done)
            chunk = source.read(n)
            if len(chunk) != n:
                G.fail("UploadFrom: the stream ended after %d of %d bytes", done + len(chunk), length)
            self.upload(slot, offset + done, chunk)
            done += n

    def download(self, slot: int, offset: int, nbytes: int) -> bytes:
        G.check_transfer(self.layout, True, slot, offset, nbytes)
        out = np.empty(nbytes, np.uint8)
        N.check(N.lib().lrm_cuda_download(self._b._h, slot, offset, N.ptr(out), nbytes), self._b._h, "Download")
        return out.tobytes()

    def download_array(self, slot: int, offset: int, dtype, count: int) -> np.ndarray:
        nb = np.dtype(dtype).itemsize * count
        return np.frombuffer(self.download(slot, offset, G.align_up(4, nb))[:nb], dtype).copy()


class CudaCommandList:
    """ICommandList (Backend.fs:118-134). Single use: Submit closes it."""

    def __init__(self, backend):
        self._b = backend
        h = ctypes.c_void_p()
        N.check(N.lib().lrm_cuda_begin(backend._h, ctypes.byref(h)), backend._h, "Begin")
        self._h = h
        self.closed = False
        self.dispatch_count = 0
        self._timers = []  # (id, name, attrs)
        self._open = []
        self.prepared = []

    def _open_check(self):
        if self.closed:
            G.fail("the command list was submitted; record into a new one")

    def dispatch(self, kernel_id: int, args: G.ArgBlock) -> G.PreparedDispatch:
        self._open_check()
        heap = self._b.heap
        if heap is None or heap.table is None:
            G.fail("a dispatch needs the heap and its written table")
        if self._b.kernels is None or not self._b.kernels.contains(kernel_id):
            G.fail("kernel %s is not in the loaded set", kernel_id)
        p = G.prepare(heap.table, kernel_id, args)
        words = (ctypes.c_uint32 * 32)(*p.args.words())
        N.check(N.lib().lrm_cuda_dispatch(self._h, int(kernel_id), words), self._b._h, p.kernel.name)
        self.dispatch_count += 1
        self.prepared.append(p)
        return p

    def dispatch_named(self, name: str, **fields) -> G.PreparedDispatch:
        k = G.kernel(name)
        return self.dispatch(k.id, k.encode(**fields))

    def barrier(self):
        self._open_check()
        N.check(N.lib().lrm_cuda_barrier(self._h), self._b._h, "Barrier")

    def copy(self, source: G.BufferRange, destination: G.BufferRange):
        self._open_check()
        G.check_copy(self._b.heap.layout, source, destination)
        N.check(N.lib().lrm_cuda_copy(self._h, source.slot, source.offset, destination.slot, destination.offset,
                                      source.bytes), self._b._h, "Copy")

    def begin_timer(self, name: str, attrs=None) -> int:
        self._open_check()
        tid = ctypes.c_uint32()
        N.check(N.lib().lrm_cuda_timer_begin(self._h, ctypes.byref(tid)), self._b._h, "BeginTimer")
        self._timers.append((tid.value, name, list(attrs or [])))
        self._open.append(tid.value)
        return tid.value

    def end_timer(self, timer: int):
        self._open_check()
        if not self._open or self._open[-1] != timer:
            G.fail("timers close in reverse order of opening")
        N.check(N.lib().lrm_cuda_timer_end(self._h, timer), self._b._h, "EndTimer")
        self._open.pop()


class CudaBackend:
    """IGpuBackend (Backend.fs:136-150). Calls come from one thread at a time."""

    def __init__(self, info: DeviceInfo, options: DeviceOptions):
        flags = (N.LRM_CUDA_DEBUG if options.debug else 0) | (N.LRM_CUDA_TIME_DISPATCHES if options.time_dispatches
                                                              else 0)
        h = ctypes.c_void_p()
        N.check(N.lib().lrm_cuda_create(info.index, flags, ctypes.byref(h)), None, "Create")
        self._h = h
        self.info = info
        self.options = options
        self.heap: CudaHeap | None = None
        self.kernels: KernelSet | None = None
        self.fp32_denormals: str | None = None
        self._lists = {}
        self._completions = {}

    # IDisposable
    def dispose(self):
        if self._h:
            N.lib().lrm_cuda_destroy(self._h)
            self._h = None

    close = dispose

    def __enter__(self):
        return self

    def __exit__(self, *a):
        self.dispose()

    @property
    def execution_class(self) -> ExecutionClass:
        if self.kernels is None:
            G.fail("the execution class is known once LoadKernels has run")
        return ExecutionClass(BACKEND, "pci:%04x:%04x" % (self.info.vendor_id, self.info.pci_device_id),
                              self.info.driver, self.kernels.shader_set_hash, host_arch())

    def create_heap(self, layout: G.HeapLayout) -> CudaHeap:
        if self.heap is not None:
            G.fail("CreateHeap is called once per backend")
        arenas = (ctypes.c_uint32 * max(1, layout.page_count))(*[int(p.arena) for p in layout.pages])
        sizes = (ctypes.c_uint64 * max(1, layout.page_count))(*[p.bytes for p in layout.pages])
        N.check(N.lib().lrm_cuda_create_heap(self._h, layout.page_count, arenas, sizes), self._h, "CreateHeap")
        self.heap = CudaHeap(self, layout)
        return self.heap

    def load_kernels(self) -> KernelSet:
        """LoadKernels: the catalog kernels are built into liblrmcuda.so for sm_100a. Runs the denormal probe."""
        if self.kernels is not None:
            G.fail("LoadKernels is called once per backend")
        digest = ctypes.create_string_buffer(32)
        N.check(N.lib().lrm_cuda_load_kernels(self._h, digest), self._h, "LoadKernels")
        self.kernels = KernelSet(self, digest.raw)
        ins = (ctypes.c_uint32 * 7)(*PROBE_INPUTS)
        outs = (ctypes.c_uint32 * 7)()
        N.check(N.lib().lrm_cuda_denormal_probe(self._h, ins, outs), self._h, "denormal probe")
        self.fp32_denormals = classify_denormals(list(outs))
        return self.kernels

    def begin(self) -> CudaCommandList:
        return CudaCommandList(self)

    def submit(self, commands: CudaCommandList) -> int:
        if not isinstance(commands, CudaCommandList) or commands._b is not self:
            G.fail("the command list belongs to another backend")
        if commands.closed:
            G.fail("a command list is submitted once")
        if commands._open:
            G.fail("a timer is still open")
        fence = ctypes.c_uint64()
        N.check(N.lib().lrm_cuda_submit(commands._h, ctypes.byref(fence)), self._h, "Submit")
        commands.closed = True
        self._lists[fence.value] = commands
        return fence.value

    def wait(self, submission: int, timeout_ms: int = 30000) -> Completion:
        if submission in self._completions:
            return self._completions[submission]
        c = N.CompletionC()
        N.check(N.lib().lrm_cuda_wait(self._h, submission, timeout_ms, ctypes.byref(c)), self._h, "Wait")
        lst = self._lists.pop(submission, None)
        names = {t[0]: (t[1], t[2]) for t in (lst._timers if lst else [])}
        timers = []
        for i in range(c.timer_count):
            tid, st, du = ctypes.c_uint32(), ctypes.c_int64(), ctypes.c_int64()
            N.check(N.lib().lrm_cuda_timer_result(self._h, submission, i, ctypes.byref(tid), ctypes.byref(st),
                                                  ctypes.byref(du)), self._h, "timer")
            if tid.value & 0x80000000:
                kname = G.kernel(tid.value & 0x7FFFFFFF).name
                timers.append(TimerResult("gpu.dispatch", [("backend", BACKEND), ("kernel", kname)], st.value,
                                          du.value))
            else:
                name, attrs = names.get(tid.value, ("gpu.timer", []))
                timers.append(TimerResult(name, attrs, st.value, du.value))
        if lst is not None:
            N.lib().lrm_cuda_list_free(lst._h)
        comp = Completion(submission, c.dispatches, timers)
        self._completions[submission] = comp
        return comp


def host_arch() -> str:
    m = platform.machine().lower()
    return "linux-" + {"x86_64": "x64", "amd64": "x64", "aarch64": "arm64"}.get(m, m)


class CudaBackendProvider:
    """IGpuBackendProvider (Backend.fs:154-161)."""

    backend = BACKEND

    def enumerate(self) -> list:
        n = ctypes.c_int32()
        N.check(N.lib().lrm_cuda_device_count(ctypes.byref(n)))
        out = []
        for i in range(n.value):
            d = N.DeviceInfoC()
            N.check(N.lib().lrm_cuda_device_info(i, ctypes.byref(d)))
            info = DeviceInfo(BACKEND, d.index, d.name.decode(), d.vendor_id, d.pci_device_id, d.driver.decode(),
                              d.memory_bytes, [("sm_count", str(d.sm_count)),
                                               ("compute_capability", f"{d.cc_major}.{d.cc_minor}")])
            out.append(DeviceCandidate(info, [] if d.accepted else [d.rejection.decode()]))
        return out

    def create(self, device: DeviceInfo, options: DeviceOptions | None = None) -> CudaBackend:
        return CudaBackend(device, options or DeviceOptions())


def try_create(options: DeviceOptions | None = None) -> CudaBackend:
    """Backend.tryCreate for the CUDA provider: device `index` (must be accepted) or the first accepted device."""
    options = options or DeviceOptions()
    cands = CudaBackendProvider().enumerate()
    chosen = None
    if options.index is not None:
        chosen = next((c for c in cands if c.info.index == options.index), None)
    else:
        chosen = next((c for c in cands if c.accepted), None)
    if chosen is None or not chosen.accepted:
        why = "; ".join(f"{c.info.index} {c.info.name}: {'; '.join(c.rejections)}" for c in cands) or "no devices"
        raise LookupError(f"no accepted cuda device ({why})")
    return CudaBackendProvider().create(chosen.info, options)
