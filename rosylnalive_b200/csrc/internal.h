// internal.h -- shared declarations inside liblrmcuda.so (not part of the ABI).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <mutex>
#include <string>

namespace lrm {

// One catalog dispatch, resolved: the 32 argument words and, for each token field i (word i + 1), its device
// pointer (nullptr for non-token fields and the null token). `table` is the device copy of the tensor table.
struct CatalogLaunch {
    uint32_t kernel;
    uint32_t w[32];
    void *ptr[32];
    const uint32_t *table;
};

// Launches one catalog kernel on `stream`; returns the launch error (cudaSuccess when queued).
cudaError_t launch_catalog(const CatalogLaunch &l, cudaStream_t stream);

// True when the catalog kernel is compiled into this library.
bool catalog_kernel_present(uint32_t kernel);

// Thread-local error message for calls that have no device yet.
void set_thread_error(const std::string &msg);
std::string thread_error();

// Whether launches on this thread use programmatic dependent launch (the engine turns it on around its own
// sequences; every kernel that can be launched this way calls griddepcontrol.wait before it touches data that the
// previous kernel writes).
bool pdl_enabled();
void set_pdl(bool on);

// A kernel's dynamic shared-memory opt-in, made once per device. The library's entry points may be called from
// several host threads (one per device, or several on one device), so each call site keeps one of these as a
// function-local static and the flag is read and set under its lock.
struct SmemOptIn {
    std::mutex mu;
    bool done[64] = {};
    // With big_clusters, the kernel also opts into clusters above the portable 8 CTAs.
    cudaError_t set(const void *kernel, int bytes, bool big_clusters = false) {
        int dev = 0;
        cudaError_t e = cudaGetDevice(&dev);
        if (e != cudaSuccess) return e;
        if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
        std::lock_guard<std::mutex> g(mu);
        if (!done[dev]) {
            e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
            if (e == cudaSuccess && big_clusters)
                e = cudaFuncSetAttribute(kernel, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
            if (e != cudaSuccess) return e;
            done[dev] = true;
        }
        return cudaSuccess;
    }
};

// Launches `kernel` with programmatic stream serialization when pdl_enabled().
template <typename... KArgs, typename... Args>
cudaError_t launch_kernel(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                          Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl_enabled() ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kernel, ((KArgs)args)...);
}

}  // namespace lrm

#define LRM_CATALOG_KERNELS 14
