// device.cu -- the CUDA device behind the reference's IGpuBackend / IGpuHeap / ICommandList contracts
// (src/Lrm.Gpu.Core/Backend.fs:96-161, docs/contracts/gpu-backend.md), exported through include/lrm_cuda.h.
//
// Design (CUDA-first, not a translation of the D3D12 backend):
//  - one CUDA stream per device; command lists are recorded on the host and enqueued in order at Submit, so a
//    Barrier needs no GPU work (the stream is in order) and a Copy is one cudaMemcpyAsync;
//  - a fence is a CUDA event recorded after the list; Wait polls it with a time limit, so a slow or stuck
//    submission returns LRM_ERR_TIMEOUT instead of blocking forever, and the context stays usable;
//  - the heap is 63 page allocations plus the 1 MiB table; tokens are resolved to device pointers once, at
//    Dispatch, from the host copy of the sealed table (the table never changes after WriteTable);
//  - every dispatch is re-checked here before it is recorded (token rows, dtypes, flags, aliasing, the catalog grid
//    and the minimum element counts of kernel-abi.md), so no block a caller gets wrong can reach a kernel.
#include <cuda_runtime.h>
#include <stdarg.h>
#include <stdio.h>
#include <string.h>
#include <time.h>

#include <memory>
#include <mutex>
#include <string>
#include <vector>

#include "../../include/lrm_cuda.h"
#include "internal.h"

namespace lrm {

static thread_local std::string g_thread_error;
void set_thread_error(const std::string &m) { g_thread_error = m; }
std::string thread_error() { return g_thread_error; }

static thread_local bool g_pdl = false;
bool pdl_enabled() { return g_pdl; }
void set_pdl(bool on) { g_pdl = on; }

static std::string fmt(const char *f, ...) {
    char buf[1024];
    va_list ap;
    va_start(ap, f);
    vsnprintf(buf, sizeof buf, f, ap);
    va_end(ap);
    return buf;
}

// ---- catalog facts the shim needs (kernel-abi.md "The catalog at contracts-v1") -------------------------------

enum Kind : uint8_t { TOK_R, TOK_W, TOK_M, U32, F32 };
// dtype codes (heap-and-tensor-table.md): F32 1, BF16 2, U32 5, I32 4.
struct FieldInfo {
    Kind kind;
    uint8_t dtypes;  // bit per accepted dtype code
    uint8_t alias;   // bit per field index this written field may alias (read fields)
};
struct KernelInfo {
    const char *name;
    int nfields;
    FieldInfo f[31];
    bool linear;
};

#define DT(c) (uint8_t)(1u << (c))
static const uint8_t DF32 = DT(1), DBF16 = DT(2), DU32 = DT(5), DI32 = DT(4);

static KernelInfo make_args_echo() {
    KernelInfo k{"args_echo", 31, {}, true};
    k.f[0] = {TOK_W, DU32, 0};
    for (int i = 1; i < 31; ++i) k.f[i] = {U32, 0, 0};
    return k;
}

static const KernelInfo KERNELS[LRM_CATALOG_KERNELS] = {
    {"scale_f32", 4, {{TOK_R, DF32, 0}, {TOK_W, DF32, 1u << 0}, {U32, 0, 0}, {F32, 0, 0}}, true},
    {"table_echo", 2, {{TOK_M, 0, 0}, {TOK_W, DU32, 0}}, true},
    make_args_echo(),
    {"groups_echo", 2, {{TOK_W, DU32, 0}, {U32, 0, 0}}, true},
    {"bf16_unpack", 3, {{TOK_R, DBF16, 0}, {TOK_W, DF32, 0}, {U32, 0, 0}}, true},
    {"embed_gather_bf16",
     6,
     {{TOK_R, DU32, 0}, {TOK_R, DBF16, 0}, {TOK_W, DF32, 0}, {U32, 0, 0}, {U32, 0, 0}, {U32, 0, 0}},
     false},
    {"rmsnorm_rows",
     6,
     {{TOK_R, DF32, 0}, {TOK_R, DBF16, 0}, {TOK_W, DF32, 1u << 0}, {U32, 0, 0}, {U32, 0, 0}, {F32, 0, 0}},
     true},
    {"rope_apply",
     8,
     {{TOK_R, DF32, 0},
      {TOK_R, DF32, 0},
      {TOK_R, DF32, 0},
      {TOK_W, DF32, 1u << 0},
      {U32, 0, 0},
      {U32, 0, 0},
      {U32, 0, 0},
      {U32, 0, 0}},
     true},
    {"silu_mul", 4, {{TOK_R, DF32, 0}, {TOK_R, DF32, 0}, {TOK_W, DF32, (1u << 0) | (1u << 1)}, {U32, 0, 0}}, true},
    {"add", 4, {{TOK_R, DF32, 0}, {TOK_R, DF32, 0}, {TOK_W, DF32, (1u << 0) | (1u << 1)}, {U32, 0, 0}}, true},
    {"copy_rows",
     8,
     {{TOK_R, (uint8_t)(DF32 | DU32 | DI32), 0},
      {TOK_W, (uint8_t)(DF32 | DU32 | DI32), 0},
      {U32, 0, 0},
      {U32, 0, 0},
      {U32, 0, 0},
      {U32, 0, 0},
      {U32, 0, 0},
      {U32, 0, 0}},
     true},
    {"argmax_rows", 4, {{TOK_R, DF32, 0}, {TOK_W, DU32, 0}, {U32, 0, 0}, {U32, 0, 0}}, true},
    {"matmul_bf16w",
     6,
     {{TOK_R, DF32, 0}, {TOK_R, DBF16, 0}, {TOK_W, DF32, 0}, {U32, 0, 0}, {U32, 0, 0}, {U32, 0, 0}},
     false},
    {"attention_gqa_causal",
     11,
     {{TOK_R, DF32, 0},
      {TOK_R, DF32, 0},
      {TOK_R, DF32, 0},
      {TOK_W, DF32, 0},
      {U32, 0, 0},
      {U32, 0, 0},
      {U32, 0, 0},
      {U32, 0, 0},
      {U32, 0, 0},
      {U32, 0, 0},
      {F32, 0, 0}},
     false},
};

static int64_t cdiv(int64_t a, int64_t b) { return (a + b - 1) / b; }

// The catalog grid formulas, evaluated in int64 (kernel-abi.md "Grids and folding").
static void logical_grid(uint32_t k, const uint32_t *w, int64_t g[3]) {
    g[1] = g[2] = 1;
    switch (k) {
        case 0: case 4: g[0] = cdiv(w[3], 256); break;
        case 1: case 2: g[0] = 1; break;
        case 3: g[0] = w[2]; break;
        case 5: g[0] = cdiv(w[5], 256); g[1] = w[4]; break;
        case 6: g[0] = w[4]; break;
        case 7: g[0] = w[5]; break;
        case 8: case 9: g[0] = cdiv(w[4], 256); break;
        case 10: g[0] = cdiv((int64_t)w[3] * w[4], 256); break;
        case 11: g[0] = w[3]; break;
        case 12: g[0] = cdiv(w[5], 64); g[1] = cdiv(w[4], 64); break;
        case 13: g[0] = w[5]; g[1] = w[8]; break;
    }
}

// ---- objects --------------------------------------------------------------------------------------------------

struct Command {
    enum Type { DISPATCH, COPY, TIMER_BEGIN, TIMER_END } type;
    CatalogLaunch launch;
    void *dst, *src;
    uint64_t bytes;
    uint32_t timer;
};

struct TimerRec {
    uint32_t id;
    cudaEvent_t begin, end;
};

struct Submission {
    uint64_t fence;
    cudaEvent_t done;
    uint32_t dispatches;
    std::vector<TimerRec> timers;
    bool completed = false;
};

}  // namespace lrm

struct lrm_cmdlist_s {
    lrm_device dev;
    std::vector<lrm::Command> cmds;
    std::vector<uint32_t> open_timers;
    uint32_t next_timer = 1;
    uint32_t dispatches = 0;
    bool closed = false;
};

struct lrm_device_s {
    int index;
    uint32_t flags;
    cudaStream_t stream = nullptr;
    cudaEvent_t base = nullptr;
    std::mutex mu;
    std::string error;
    bool heap = false, table_written = false, kernels_loaded = false;
    std::vector<void *> pages;      // index = slot (0 = table)
    std::vector<uint64_t> page_bytes;
    std::vector<uint32_t> table;    // host copy, 16384 x 16 words
    uint64_t next_fence = 1;
    std::vector<std::unique_ptr<lrm::Submission>> subs;
    std::vector<lrm_cmdlist> lists;
};

using namespace lrm;

static lrm_status dev_fail(lrm_device d, lrm_status s, const std::string &m) {
    if (d)
        d->error = m;
    else
        set_thread_error(m);
    return s;
}

static lrm_status cuda_fail(lrm_device d, cudaError_t e, const char *what) {
    return dev_fail(d, LRM_ERR_CUDA, fmt("%s: %s (%s)", what, cudaGetErrorName(e), cudaGetErrorString(e)));
}

#define CUDA_TRY(d, call, what)                          \
    do {                                                  \
        cudaError_t e_ = (call);                          \
        if (e_ != cudaSuccess) return cuda_fail(d, e_, what); \
    } while (0)

extern "C" {

int32_t lrm_cuda_abi_version(void) { return LRM_CUDA_ABI_VERSION; }

size_t lrm_cuda_last_error(lrm_device dev, char *buf, size_t n) {
    std::string m = dev ? dev->error : thread_error();
    if (buf && n) {
        size_t c = m.size() < n - 1 ? m.size() : n - 1;
        memcpy(buf, m.data(), c);
        buf[c] = 0;
    }
    return m.size();
}

lrm_status lrm_cuda_device_count(int32_t *count) {
    if (!count) return dev_fail(nullptr, LRM_ERR_ARGUMENT, "count is null");
    int n = 0;
    cudaError_t e = cudaGetDeviceCount(&n);
    if (e == cudaErrorNoDevice || e == cudaErrorInsufficientDriver) {
        *count = 0;
        return LRM_OK;
    }
    if (e != cudaSuccess) return cuda_fail(nullptr, e, "cudaGetDeviceCount");
    *count = n;
    return LRM_OK;
}

static void read_text(const char *path, char *out, size_t n) {
    out[0] = 0;
    FILE *f = fopen(path, "r");
    if (!f) return;
    size_t r = fread(out, 1, n - 1, f);
    out[r] = 0;
    fclose(f);
}

lrm_status lrm_cuda_device_info(int32_t index, lrm_device_info *out) {
    if (!out) return dev_fail(nullptr, LRM_ERR_ARGUMENT, "out is null");
    int32_t n = 0;
    lrm_status s = lrm_cuda_device_count(&n);
    if (s != LRM_OK) return s;
    if (index < 0 || index >= n) return dev_fail(nullptr, LRM_ERR_NO_DEVICE, fmt("no CUDA device %d", index));
    cudaDeviceProp p;
    cudaError_t e = cudaGetDeviceProperties(&p, index);
    if (e != cudaSuccess) return cuda_fail(nullptr, e, "cudaGetDeviceProperties");
    memset(out, 0, sizeof *out);
    out->index = index;
    snprintf(out->name, sizeof out->name, "%s", p.name);
    out->vendor_id = 0x10de;
    char path[256], txt[512];
    snprintf(path, sizeof path, "/sys/bus/pci/devices/%04x:%02x:%02x.0/device", p.pciDomainID, p.pciBusID,
             p.pciDeviceID);
    read_text(path, txt, sizeof txt);
    out->pci_device_id = (uint32_t)strtoul(txt, nullptr, 16);
    read_text("/proc/driver/nvidia/version", txt, sizeof txt);
    const char *k = strstr(txt, "Kernel Module");
    if (k) {
        k += strlen("Kernel Module");
        while (*k == ' ' || *k == '\t') ++k;
        size_t i = 0;
        while (k[i] && k[i] != ' ' && k[i] != '\n' && i < sizeof out->driver - 1) {
            out->driver[i] = k[i];
            ++i;
        }
    } else {
        int dv = 0;
        cudaDriverGetVersion(&dv);
        snprintf(out->driver, sizeof out->driver, "cuda-%d.%d", dv / 1000, (dv % 1000) / 10);
    }
    out->memory_bytes = (int64_t)p.totalGlobalMem;
    out->sm_count = p.multiProcessorCount;
    out->cc_major = p.major;
    out->cc_minor = p.minor;
    out->accepted = p.major == 10 && p.minor == 0;
    if (!out->accepted)
        snprintf(out->rejection, sizeof out->rejection, "requires compute capability 10.0 (sm_100a), found %d.%d",
                 p.major, p.minor);
    return LRM_OK;
}

lrm_status lrm_cuda_create(int32_t index, uint32_t flags, lrm_device *out) {
    if (!out) return dev_fail(nullptr, LRM_ERR_ARGUMENT, "out is null");
    *out = nullptr;
    lrm_device_info info;
    lrm_status s = lrm_cuda_device_info(index, &info);
    if (s != LRM_OK) return s;
    if (!info.accepted) return dev_fail(nullptr, LRM_ERR_NO_DEVICE, info.rejection);
    cudaError_t e = cudaSetDevice(index);
    if (e != cudaSuccess) return cuda_fail(nullptr, e, "cudaSetDevice");
    std::unique_ptr<lrm_device_s> d(new lrm_device_s());
    d->index = index;
    d->flags = flags;
    e = cudaStreamCreateWithFlags(&d->stream, cudaStreamNonBlocking);
    if (e != cudaSuccess) return cuda_fail(nullptr, e, "cudaStreamCreate");
    e = cudaEventCreate(&d->base);
    if (e != cudaSuccess) return cuda_fail(nullptr, e, "cudaEventCreate");
    e = cudaEventRecord(d->base, d->stream);
    if (e != cudaSuccess) return cuda_fail(nullptr, e, "cudaEventRecord");
    *out = d.release();
    return LRM_OK;
}

lrm_status lrm_cuda_destroy(lrm_device d) {
    if (!d) return dev_fail(nullptr, LRM_ERR_ARGUMENT, "device is null");
    cudaSetDevice(d->index);
    cudaStreamSynchronize(d->stream);
    for (auto &sub : d->subs) {
        cudaEventDestroy(sub->done);
        for (auto &t : sub->timers) {
            cudaEventDestroy(t.begin);
            cudaEventDestroy(t.end);
        }
    }
    for (lrm_cmdlist l : d->lists) delete l;
    for (void *p : d->pages)
        if (p) cudaFree(p);
    if (d->base) cudaEventDestroy(d->base);
    if (d->stream) cudaStreamDestroy(d->stream);
    delete d;
    return LRM_OK;
}

lrm_status lrm_cuda_create_heap(lrm_device d, int32_t n, const uint32_t *arenas, const uint64_t *bytes) {
    if (!d || (n > 0 && (!arenas || !bytes))) return dev_fail(d, LRM_ERR_ARGUMENT, "null argument");
    std::lock_guard<std::mutex> g(d->mu);
    if (d->heap) return dev_fail(d, LRM_ERR_CONTRACT, "CreateHeap is called once per backend");
    if (n < 0 || n > 63) return dev_fail(d, LRM_ERR_CONTRACT, fmt("%d pages: at most 63", n));
    uint32_t last = 0;
    for (int i = 0; i < n; ++i) {
        if (bytes[i] < (64u << 10) || bytes[i] > (1ull << 30) || bytes[i] % (64u << 10))
            return dev_fail(d, LRM_ERR_CONTRACT, fmt("page %d: %llu bytes is not a multiple of 64 KiB in 64 KiB..1 GiB",
                                                     i, (unsigned long long)bytes[i]));
        if (arenas[i] < 1 || arenas[i] > 7)
            return dev_fail(d, LRM_ERR_CONTRACT, fmt("page %d: arena code %u is not a v1 arena", i, arenas[i]));
        if (arenas[i] < last) return dev_fail(d, LRM_ERR_CONTRACT, "arenas must appear in contract order");
        last = arenas[i];
    }
    cudaSetDevice(d->index);
    d->pages.assign(n + 1, nullptr);
    d->page_bytes.assign(n + 1, 0);
    d->page_bytes[0] = 1u << 20;
    for (int s = 0; s <= n; ++s) {
        uint64_t b = s == 0 ? (1u << 20) : bytes[s - 1];
        cudaError_t e = cudaMalloc(&d->pages[s], b);
        if (e != cudaSuccess) {
            for (void *p : d->pages)
                if (p) cudaFree(p);
            d->pages.clear();
            return dev_fail(d, LRM_ERR_OUT_OF_MEMORY, fmt("page %d of %llu bytes: %s", s, (unsigned long long)b,
                                                          cudaGetErrorString(e)));
        }
        d->page_bytes[s] = b;
        cudaMemsetAsync(d->pages[s], 0, b, d->stream);
    }
    CUDA_TRY(d, cudaStreamSynchronize(d->stream), "CreateHeap");
    d->table.assign(16384 * 16, 0);
    d->heap = true;
    return LRM_OK;
}

lrm_status lrm_cuda_load_kernels(lrm_device d, uint8_t set_hash[32]) {
    if (!d || !set_hash) return dev_fail(d, LRM_ERR_ARGUMENT, "null argument");
    std::lock_guard<std::mutex> g(d->mu);
    if (d->kernels_loaded) return dev_fail(d, LRM_ERR_CONTRACT, "LoadKernels is called once per backend");
    // The set hash identifies the compiled kernel set; the build writes it into lrm_kernel_set_hash.
    extern const uint8_t lrm_kernel_set_hash[32];
    memcpy(set_hash, lrm_kernel_set_hash, 32);
    d->kernels_loaded = true;
    return LRM_OK;
}

lrm_status lrm_cuda_kernel_present(lrm_device d, uint32_t kernel_id, int32_t *present) {
    if (!d || !present) return dev_fail(d, LRM_ERR_ARGUMENT, "null argument");
    *present = d->kernels_loaded && catalog_kernel_present(kernel_id);
    return LRM_OK;
}

lrm_status lrm_cuda_denormal_probe(lrm_device d, const uint32_t inputs[7], uint32_t results[7]) {
    if (!d || !inputs || !results) return dev_fail(d, LRM_ERR_ARGUMENT, "null argument");
    std::lock_guard<std::mutex> g(d->mu);
    cudaSetDevice(d->index);
    void *buf = nullptr;
    CUDA_TRY(d, cudaMalloc(&buf, 64), "denormal probe");
    CatalogLaunch L;
    memset(&L, 0, sizeof L);
    L.kernel = 0;  // scale_f32
    L.w[3] = 7;
    float half = 0.5f;
    memcpy(&L.w[4], &half, 4);
    L.ptr[1] = buf;
    L.ptr[2] = (char *)buf + 32;
    cudaError_t e = cudaMemcpy(buf, inputs, 28, cudaMemcpyHostToDevice);
    if (e == cudaSuccess) e = launch_catalog(L, d->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(d->stream);
    if (e == cudaSuccess) e = cudaMemcpy(results, (char *)buf + 32, 28, cudaMemcpyDeviceToHost);
    cudaFree(buf);
    if (e != cudaSuccess) return cuda_fail(d, e, "denormal probe");
    return LRM_OK;
}

static lrm_status check_transfer(lrm_device d, bool allow_table, int32_t slot, uint64_t offset, uint64_t n) {
    if (!d->heap) return dev_fail(d, LRM_ERR_CONTRACT, "no heap: call CreateHeap first");
    if (slot == 0 && !allow_table)
        return dev_fail(d, LRM_ERR_CONTRACT, "slot 0 holds the tensor table; write it with WriteTable");
    if (slot < 0 || slot >= (int32_t)d->pages.size())
        return dev_fail(d, LRM_ERR_CONTRACT, fmt("slot %d holds no page", slot));
    if (offset % 4 || n % 4)
        return dev_fail(d, LRM_ERR_CONTRACT,
                        fmt("transfer in slot %d: offset %llu and size %llu must be multiples of 4", slot,
                            (unsigned long long)offset, (unsigned long long)n));
    if (offset + n > d->page_bytes[slot] || offset + n < offset)
        return dev_fail(d, LRM_ERR_CONTRACT,
                        fmt("transfer in slot %d: bytes %llu..%llu are past the %llu-byte buffer", slot,
                            (unsigned long long)offset, (unsigned long long)(offset + n),
                            (unsigned long long)d->page_bytes[slot]));
    return LRM_OK;
}

lrm_status lrm_cuda_write_table(lrm_device d, const void *image, uint64_t bytes) {
    if (!d || !image) return dev_fail(d, LRM_ERR_ARGUMENT, "null argument");
    std::lock_guard<std::mutex> g(d->mu);
    if (!d->heap) return dev_fail(d, LRM_ERR_CONTRACT, "no heap: call CreateHeap first");
    if (d->table_written) return dev_fail(d, LRM_ERR_CONTRACT, "WriteTable is called exactly once");
    if (bytes != (1u << 20)) return dev_fail(d, LRM_ERR_CONTRACT, "the table image is 1 MiB");
    memcpy(d->table.data(), image, bytes);
    // Rows must name real pages with their extent inside (TensorRow.validate); checked again at each dispatch.
    cudaSetDevice(d->index);
    CUDA_TRY(d, cudaStreamSynchronize(d->stream), "WriteTable");
    CUDA_TRY(d, cudaMemcpy(d->pages[0], image, bytes, cudaMemcpyHostToDevice), "WriteTable");
    d->table_written = true;
    return LRM_OK;
}

lrm_status lrm_cuda_upload(lrm_device d, int32_t slot, uint64_t offset, const void *src, uint64_t n) {
    if (!d || (!src && n)) return dev_fail(d, LRM_ERR_ARGUMENT, "null argument");
    std::lock_guard<std::mutex> g(d->mu);
    lrm_status s = check_transfer(d, false, slot, offset, n);
    if (s != LRM_OK) return s;
    cudaSetDevice(d->index);
    CUDA_TRY(d, cudaStreamSynchronize(d->stream), "Upload (waiting for submitted work)");
    if (n) CUDA_TRY(d, cudaMemcpy((char *)d->pages[slot] + offset, src, n, cudaMemcpyHostToDevice), "Upload");
    return LRM_OK;
}

lrm_status lrm_cuda_download(lrm_device d, int32_t slot, uint64_t offset, void *dst, uint64_t n) {
    if (!d || (!dst && n)) return dev_fail(d, LRM_ERR_ARGUMENT, "null argument");
    std::lock_guard<std::mutex> g(d->mu);
    lrm_status s = check_transfer(d, true, slot, offset, n);
    if (s != LRM_OK) return s;
    cudaSetDevice(d->index);
    CUDA_TRY(d, cudaStreamSynchronize(d->stream), "Download (waiting for submitted work)");
    if (n) CUDA_TRY(d, cudaMemcpy(dst, (char *)d->pages[slot] + offset, n, cudaMemcpyDeviceToHost), "Download");
    return LRM_OK;
}

lrm_status lrm_cuda_begin(lrm_device d, lrm_cmdlist *out) {
    if (!d || !out) return dev_fail(d, LRM_ERR_ARGUMENT, "null argument");
    std::lock_guard<std::mutex> g(d->mu);
    lrm_cmdlist l = new lrm_cmdlist_s();
    l->dev = d;
    d->lists.push_back(l);
    *out = l;
    return LRM_OK;
}

lrm_status lrm_cuda_list_free(lrm_cmdlist l) {
    if (!l) return dev_fail(nullptr, LRM_ERR_ARGUMENT, "list is null");
    lrm_device d = l->dev;
    std::lock_guard<std::mutex> g(d->mu);
    for (size_t i = 0; i < d->lists.size(); ++i)
        if (d->lists[i] == l) {
            d->lists.erase(d->lists.begin() + i);
            delete l;
            return LRM_OK;
        }
    return dev_fail(d, LRM_ERR_ARGUMENT, "unknown list");
}

// ---- Dispatch: the shared rules again, on the native side ---------------------------------------------------

struct Resolved {
    bool data;
    bool writes;
    uint32_t slot, dtype, count;
    uint64_t start, end;
    int field;
};

static const uint32_t *row_of(lrm_device d, uint32_t token) { return &d->table[(size_t)token * 16]; }
static uint32_t dtype_size(uint32_t code) {
    switch (code) {
        case 1: case 4: case 5: return 4;
        case 2: case 3: return 2;
        case 6: return 1;
        case 7: case 8: return 8;
    }
    return 0;
}

static lrm_status min_counts(lrm_device d, uint32_t k, const uint32_t *w, const Resolved *r) {
    // r[i] is field i (word i + 1). Every count is int64 arithmetic over u32 fields (kernel-abi.md table).
    auto need = [&](int field, int64_t elems, const char *what) -> bool {
        if (!r[field].data) return true;
        if ((int64_t)r[field].count < elems) {
            d->error = fmt("%s.%s: the token holds %u elements but the dispatch touches %lld", KERNELS[k].name, what,
                           r[field].count, (long long)elems);
            return false;
        }
        return true;
    };
    auto rule = [&](bool ok, const char *msg) -> bool {
        if (!ok) d->error = fmt("%s: %s", KERNELS[k].name, msg);
        return ok;
    };
    bool ok = true;
    switch (k) {
        case 0: ok = need(0, w[3], "x") && need(1, w[3], "y"); break;
        case 1: ok = need(1, 16, "y"); break;
        case 2: ok = need(0, 32, "y"); break;
        case 3: ok = need(0, w[2], "y"); break;
        case 4: ok = need(0, w[3], "x") && need(1, w[3], "y"); break;
        case 5:
            ok = need(0, w[4], "ids") && need(1, (int64_t)w[6] * w[5], "table") &&
                 need(2, (int64_t)w[4] * w[5], "y");
            break;
        case 6:
            ok = rule(w[5] >= 1, "cols >= 1") && need(0, (int64_t)w[4] * w[5], "x") && need(1, w[5], "w") &&
                 need(2, (int64_t)w[4] * w[5], "y");
            break;
        case 7: {
            uint32_t rows = w[5], heads = w[6], hd = w[7], pos0 = w[8];
            ok = rule(heads >= 1 && rows % heads == 0, "heads >= 1 and divides rows") &&
                 rule(hd >= 2 && hd % 2 == 0, "head_dim even and at least 2") &&
                 need(0, (int64_t)rows * hd, "x") && need(3, (int64_t)rows * hd, "y") &&
                 need(1, ((int64_t)pos0 + rows / heads) * (hd / 2), "cos_table") &&
                 need(2, ((int64_t)pos0 + rows / heads) * (hd / 2), "sin_table");
            break;
        }
        case 8: case 9: ok = need(0, w[4], "a") && need(1, w[4], "b") && need(2, w[4], "y"); break;
        case 10: {
            int64_t rows = w[3], cols = w[4];
            ok = rule(r[0].dtype == r[1].dtype, "src and dst have the same dtype") &&
                 rule(rows <= 1 || cols <= w[8], "cols <= dst_stride when rows > 1") &&
                 need(0, ((int64_t)w[5] + rows - 1) * w[7] + cols, "src") &&
                 need(1, ((int64_t)w[6] + rows - 1) * w[8] + cols, "dst");
            break;
        }
        case 11:
            ok = rule(w[4] >= 1, "cols >= 1") && need(0, (int64_t)w[3] * w[4], "x") && need(1, w[3], "y");
            break;
        case 12:
            ok = need(0, (int64_t)w[4] * w[6], "x") && need(1, (int64_t)w[5] * w[6], "w") &&
                 need(2, (int64_t)w[4] * w[5], "y");
            break;
        case 13: {
            int64_t qcols = (int64_t)w[8] * w[10], kvcols = (int64_t)w[9] * w[10];
            ok = rule(w[9] >= 1 && w[8] % w[9] == 0, "kv_heads >= 1 and divides q_heads") &&
                 rule(w[10] >= 1, "head_dim >= 1") &&
                 rule(w[10] <= 16384, "head_dim above 16,384 is beyond this device's shared-memory staging") &&
                 need(0, ((int64_t)w[6] + w[5]) * qcols, "q") && need(3, ((int64_t)w[6] + w[5]) * qcols, "y") &&
                 need(1, ((int64_t)w[7] + w[5]) * kvcols, "k") && need(2, ((int64_t)w[7] + w[5]) * kvcols, "v");
            break;
        }
    }
    return ok ? LRM_OK : LRM_ERR_CONTRACT;
}

lrm_status lrm_cuda_dispatch(lrm_cmdlist l, uint32_t kernel_id, const uint32_t words[32]) {
    if (!l || !words) return dev_fail(l ? l->dev : nullptr, LRM_ERR_ARGUMENT, "null argument");
    lrm_device d = l->dev;
    std::lock_guard<std::mutex> g(d->mu);
    if (l->closed) return dev_fail(d, LRM_ERR_CONTRACT, "the command list was submitted; record into a new one");
    if (!d->kernels_loaded) return dev_fail(d, LRM_ERR_CONTRACT, "no kernels: call LoadKernels first");
    if (!d->table_written) return dev_fail(d, LRM_ERR_CONTRACT, "the table is not written: a dispatch needs it");
    if (kernel_id >= LRM_CATALOG_KERNELS || !catalog_kernel_present(kernel_id))
        return dev_fail(d, LRM_ERR_CONTRACT, fmt("kernel %u is not in the loaded set", kernel_id));
    const KernelInfo &K = KERNELS[kernel_id];
    for (int i = K.nfields + 1; i < 32; ++i)
        if (words[i]) return dev_fail(d, LRM_ERR_CONTRACT, fmt("%s: argument word %d is past the last field and must be 0", K.name, i));
    Resolved r[31];
    CatalogLaunch L;
    memset(&L, 0, sizeof L);
    L.kernel = kernel_id;
    memcpy(L.w, words, sizeof L.w);
    L.table = (const uint32_t *)d->pages[0];
    for (int i = 0; i < K.nfields; ++i) {
        r[i] = Resolved{false, false, 0, 0, 0, 0, 0, i};
        Kind kind = K.f[i].kind;
        if (kind != TOK_R && kind != TOK_W && kind != TOK_M) continue;
        uint32_t tok = words[i + 1];
        if (tok >= 16384) return dev_fail(d, LRM_ERR_CONTRACT, fmt("%s: token %u is outside 0..16383", K.name, tok));
        const uint32_t *row = row_of(d, tok);
        if (kind == TOK_M) continue;  // meta: only the row is read, by table_echo
        if (tok == 0) return dev_fail(d, LRM_ERR_CONTRACT, fmt("%s field %d: the null token is not allowed here", K.name, i));
        uint32_t slot = row[0], off = row[1], dt = row[2], count = row[12], flags = row[13];
        if (slot < 1 || slot >= d->pages.size())
            return dev_fail(d, LRM_ERR_CONTRACT, fmt("%s field %d: token %u is not in the table", K.name, i, tok));
        if (dt > 7 || !(K.f[i].dtypes & (1u << dt)))
            return dev_fail(d, LRM_ERR_CONTRACT, fmt("%s field %d: tensor dtype %u is not accepted", K.name, i, dt));
        if (!(flags & 1)) return dev_fail(d, LRM_ERR_CONTRACT, fmt("%s field %d: tensor is not contiguous", K.name, i));
        if (kind == TOK_W && (flags & 2))
            return dev_fail(d, LRM_ERR_CONTRACT, fmt("%s field %d: tensor is read only", K.name, i));
        uint64_t sz = dtype_size(dt);
        uint64_t extent = ((uint64_t)count * sz + 3) / 4 * 4;
        if (off % (sz < 4 ? 4 : sz) || (uint64_t)off + extent > d->page_bytes[slot])
            return dev_fail(d, LRM_ERR_CONTRACT, fmt("%s field %d: tensor lies outside its page", K.name, i));
        r[i] = Resolved{true, kind == TOK_W, slot, dt, count, off, off + extent, i};
        L.ptr[i + 1] = (char *)d->pages[slot] + off;
    }
    // Aliasing (Dispatch.fs:107-143).
    for (int a = 0; a < K.nfields; ++a)
        for (int b = a + 1; b < K.nfields; ++b) {
            if (!r[a].data || !r[b].data || r[a].slot != r[b].slot) continue;
            if (!(r[a].start < r[b].end && r[b].start < r[a].end)) continue;
            if (!r[a].writes && !r[b].writes) continue;
            bool same = r[a].start == r[b].start && r[a].end == r[b].end;
            bool declared = (r[a].writes && !r[b].writes && (K.f[a].alias & (1u << b))) ||
                            (r[b].writes && !r[a].writes && (K.f[b].alias & (1u << a)));
            if (!(declared && same))
                return dev_fail(d, LRM_ERR_CONTRACT, fmt("%s: fields %d and %d overlap in slot %u and may not alias",
                                                         K.name, a, b, r[a].slot));
        }
    // Grid (catalog formula, folded): word 0 must be the physical x.
    int64_t gr[3];
    logical_grid(kernel_id, words, gr);
    if (gr[0] < 1 || gr[1] < 1 || gr[2] < 1) return dev_fail(d, LRM_ERR_CONTRACT, fmt("%s: empty grid", K.name));
    if (gr[1] > 65535 || gr[2] > 65535) return dev_fail(d, LRM_ERR_CONTRACT, fmt("%s: y and z must be at most 65535", K.name));
    int64_t px = gr[0];
    if (gr[0] > 65535) {
        if (!K.linear) return dev_fail(d, LRM_ERR_CONTRACT, fmt("%s: grid x above 65535 is not foldable", K.name));
        if (gr[0] > 65535ll * 65535ll) return dev_fail(d, LRM_ERR_CONTRACT, fmt("%s: grid x exceeds 65535 * 65535", K.name));
        int64_t y = cdiv(gr[0], 65535);
        px = cdiv(gr[0], y);
    }
    if (words[0] != (uint32_t)px)
        return dev_fail(d, LRM_ERR_CONTRACT, fmt("%s: word 0 is %u but the physical grid x is %lld (Dispatch.prepare writes it)",
                                                 K.name, words[0], (long long)px));
    lrm_status s = min_counts(d, kernel_id, words, r);
    if (s != LRM_OK) return s;
    Command c;
    memset(&c, 0, sizeof c);
    c.type = Command::DISPATCH;
    c.launch = L;
    l->cmds.push_back(c);
    l->dispatches++;
    return LRM_OK;
}

lrm_status lrm_cuda_barrier(lrm_cmdlist l) {
    if (!l) return dev_fail(nullptr, LRM_ERR_ARGUMENT, "list is null");
    if (l->closed) return dev_fail(l->dev, LRM_ERR_CONTRACT, "the command list was submitted");
    return LRM_OK;  // one in-order stream: every earlier command completes before a later one starts
}

lrm_status lrm_cuda_copy(lrm_cmdlist l, int32_t ss, uint64_t so, int32_t ds, uint64_t dof, uint64_t n) {
    if (!l) return dev_fail(nullptr, LRM_ERR_ARGUMENT, "list is null");
    lrm_device d = l->dev;
    std::lock_guard<std::mutex> g(d->mu);
    if (l->closed) return dev_fail(d, LRM_ERR_CONTRACT, "the command list was submitted");
    if (ss == 0 || ds == 0) return dev_fail(d, LRM_ERR_CONTRACT, "copy: slot 0 is the table, not a page");
    lrm_status s = check_transfer(d, false, ss, so, n);
    if (s == LRM_OK) s = check_transfer(d, false, ds, dof, n);
    if (s != LRM_OK) return s;
    if (n == 0) return dev_fail(d, LRM_ERR_CONTRACT, "copy: size must be positive");
    if (ss == ds && so < dof + n && dof < so + n) return dev_fail(d, LRM_ERR_CONTRACT, "copy: source and destination overlap");
    Command c;
    memset(&c, 0, sizeof c);
    c.type = Command::COPY;
    c.src = (char *)d->pages[ss] + so;
    c.dst = (char *)d->pages[ds] + dof;
    c.bytes = n;
    l->cmds.push_back(c);
    return LRM_OK;
}

lrm_status lrm_cuda_timer_begin(lrm_cmdlist l, uint32_t *id) {
    if (!l || !id) return dev_fail(nullptr, LRM_ERR_ARGUMENT, "null argument");
    if (l->closed) return dev_fail(l->dev, LRM_ERR_CONTRACT, "the command list was submitted");
    Command c;
    memset(&c, 0, sizeof c);
    c.type = Command::TIMER_BEGIN;
    c.timer = l->next_timer++;
    l->open_timers.push_back(c.timer);
    l->cmds.push_back(c);
    *id = c.timer;
    return LRM_OK;
}

lrm_status lrm_cuda_timer_end(lrm_cmdlist l, uint32_t id) {
    if (!l) return dev_fail(nullptr, LRM_ERR_ARGUMENT, "list is null");
    if (l->closed) return dev_fail(l->dev, LRM_ERR_CONTRACT, "the command list was submitted");
    if (l->open_timers.empty() || l->open_timers.back() != id)
        return dev_fail(l->dev, LRM_ERR_CONTRACT, "timers close in reverse order of opening");
    l->open_timers.pop_back();
    Command c;
    memset(&c, 0, sizeof c);
    c.type = Command::TIMER_END;
    c.timer = id;
    l->cmds.push_back(c);
    return LRM_OK;
}

lrm_status lrm_cuda_submit(lrm_cmdlist l, uint64_t *fence) {
    if (!l || !fence) return dev_fail(nullptr, LRM_ERR_ARGUMENT, "null argument");
    lrm_device d = l->dev;
    std::lock_guard<std::mutex> g(d->mu);
    if (l->closed) return dev_fail(d, LRM_ERR_CONTRACT, "a command list is submitted once");
    if (!l->open_timers.empty()) return dev_fail(d, LRM_ERR_CONTRACT, "a timer is still open");
    l->closed = true;
    cudaSetDevice(d->index);
    std::unique_ptr<Submission> sub(new Submission());
    sub->fence = d->next_fence++;
    sub->dispatches = l->dispatches;
    std::vector<TimerRec> dispatch_timers;
    std::vector<size_t> open;  // indices into sub->timers
    for (Command &c : l->cmds) {
        switch (c.type) {
            case Command::DISPATCH: {
                TimerRec tr{0x80000000u | c.launch.kernel, nullptr, nullptr};
                bool timed = d->flags & LRM_CUDA_TIME_DISPATCHES;
                if (timed) {
                    cudaEventCreate(&tr.begin);
                    cudaEventCreate(&tr.end);
                    cudaEventRecord(tr.begin, d->stream);
                }
                cudaError_t e = launch_catalog(c.launch, d->stream);
                if (e != cudaSuccess) return cuda_fail(d, e, KERNELS[c.launch.kernel].name);
                if (timed) {
                    cudaEventRecord(tr.end, d->stream);
                    dispatch_timers.push_back(tr);
                }
                if (d->flags & LRM_CUDA_DEBUG) CUDA_TRY(d, cudaStreamSynchronize(d->stream), KERNELS[c.launch.kernel].name);
                break;
            }
            case Command::COPY:
                CUDA_TRY(d, cudaMemcpyAsync(c.dst, c.src, c.bytes, cudaMemcpyDeviceToDevice, d->stream), "Copy");
                break;
            case Command::TIMER_BEGIN: {
                TimerRec tr{c.timer, nullptr, nullptr};
                CUDA_TRY(d, cudaEventCreate(&tr.begin), "cudaEventCreate");
                CUDA_TRY(d, cudaEventCreate(&tr.end), "cudaEventCreate");
                CUDA_TRY(d, cudaEventRecord(tr.begin, d->stream), "cudaEventRecord");
                open.push_back(sub->timers.size());
                sub->timers.push_back(tr);
                break;
            }
            case Command::TIMER_END: {
                size_t i = open.back();
                open.pop_back();
                CUDA_TRY(d, cudaEventRecord(sub->timers[i].end, d->stream), "cudaEventRecord");
                break;
            }
        }
    }
    for (auto &t : dispatch_timers) sub->timers.push_back(t);
    CUDA_TRY(d, cudaEventCreateWithFlags(&sub->done, cudaEventDisableTiming), "cudaEventCreate");
    CUDA_TRY(d, cudaEventRecord(sub->done, d->stream), "cudaEventRecord");
    *fence = sub->fence;
    d->subs.push_back(std::move(sub));
    return LRM_OK;
}

static Submission *find_sub(lrm_device d, uint64_t fence) {
    for (auto &s : d->subs)
        if (s->fence == fence) return s.get();
    return nullptr;
}

lrm_status lrm_cuda_wait(lrm_device d, uint64_t fence, uint32_t timeout_ms, lrm_completion *out) {
    if (!d || !out) return dev_fail(d, LRM_ERR_ARGUMENT, "null argument");
    Submission *s;
    {
        std::lock_guard<std::mutex> g(d->mu);
        s = find_sub(d, fence);
    }
    if (!s) return dev_fail(d, LRM_ERR_CONTRACT, fmt("fence %llu was never submitted", (unsigned long long)fence));
    cudaSetDevice(d->index);
    struct timespec t0, t;
    clock_gettime(CLOCK_MONOTONIC, &t0);
    while (!s->completed) {
        cudaError_t e = cudaEventQuery(s->done);
        if (e == cudaSuccess) {
            s->completed = true;
            break;
        }
        if (e != cudaErrorNotReady) return cuda_fail(d, e, "Wait");
        clock_gettime(CLOCK_MONOTONIC, &t);
        double ms = (t.tv_sec - t0.tv_sec) * 1e3 + (t.tv_nsec - t0.tv_nsec) / 1e6;
        if (ms > timeout_ms)
            return dev_fail(d, LRM_ERR_TIMEOUT, fmt("Wait: fence %llu not done after %u ms", (unsigned long long)fence, timeout_ms));
        struct timespec nap = {0, 20000};
        nanosleep(&nap, nullptr);
    }
    out->fence = fence;
    out->dispatches = s->dispatches;
    out->timer_count = (uint32_t)s->timers.size();
    return LRM_OK;
}

lrm_status lrm_cuda_timer_result(lrm_device d, uint64_t fence, uint32_t index, uint32_t *id, int64_t *start_ns,
                                 int64_t *dur_ns) {
    if (!d || !id || !start_ns || !dur_ns) return dev_fail(d, LRM_ERR_ARGUMENT, "null argument");
    Submission *s = find_sub(d, fence);
    if (!s || !s->completed) return dev_fail(d, LRM_ERR_CONTRACT, "timer results need a completed Wait");
    if (index >= s->timers.size()) return dev_fail(d, LRM_ERR_ARGUMENT, "timer index out of range");
    TimerRec &t = s->timers[index];
    float a = 0, b = 0;
    CUDA_TRY(d, cudaEventElapsedTime(&a, d->base, t.begin), "cudaEventElapsedTime");
    CUDA_TRY(d, cudaEventElapsedTime(&b, t.begin, t.end), "cudaEventElapsedTime");
    *id = t.id;
    *start_ns = (int64_t)(a * 1e6);
    *dur_ns = (int64_t)(b * 1e6);
    return LRM_OK;
}

}  // extern "C"
