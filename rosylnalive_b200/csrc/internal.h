// internal.h -- shared declarations inside liblrmcuda.so (not part of the ABI).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

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

}  // namespace lrm

#define LRM_CATALOG_KERNELS 14
