// decode_attn_static.cu -- decode attention for callers that cannot allocate device memory.
//
// Who needs it: a host that sizes all of its device memory once up front and never allocates per call, a serving
// loop whose memory budget is fixed after warm-up, code running inside a stream capture or a host callback (where
// cudaMalloc is not allowed).
// Such a caller can pass the inputs and the output but has no way to provide the split-K scratch that
// lrm_op_decode_attention takes as `workspace`. This entry point runs the same kernels with that scratch in a
// fixed array inside this library:
//   - the array is LRM_DECODE_ATTN_STATIC_SCRATCH_BYTES (16 MiB) of file-scope __device__ memory, so every GPU that
//     loads the library holds it until the process exits; a call whose scratch would not fit is refused
//     (LRM_ERR_ARGUMENT) before anything is launched;
//   - host code cannot use the array's name as a device address (on the host it names a stand-in object), so the
//     first call on each device, with that device current, asks the runtime for the address with
//     cudaGetSymbolAddress and caches it per device for the life of the process; make that first call before any
//     stream capture. A device reset (cudaDeviceReset) makes the cached address stale, so a process that resets a
//     device must not call this entry point on it again;
//   - nothing in the scratch has to start at zero: the combine kernel reads only the split states that the attention
//     kernel of the same call has just written;
//   - every call on a device shares the one array and it keeps the last call's contents, so calls that overlap on
//     the GPU (two streams, or a call still running when the next starts on another stream) race on it.
// No cudaMalloc, cudaFree or allocating library routine is called.
#include <cuda_runtime.h>
#include <string.h>

#include <mutex>
#include <string>

#include "../../include/lrm_cuda.h"
#include "internal.h"

namespace {

static __device__ __align__(256) unsigned char g_decode_attn_scratch[LRM_DECODE_ATTN_STATIC_SCRATCH_BYTES];

void *g_scratch_addr[64];
std::mutex g_scratch_mu;

}  // namespace

extern "C" lrm_status lrm_op_decode_attention_static(void *stream, const lrm_decode_attn_desc *desc) {
    if (!desc) {
        lrm::set_thread_error("decode attention (static scratch): descriptor is null");
        return LRM_ERR_ARGUMENT;
    }
    if (desc->workspace) {
        lrm::set_thread_error("decode attention (static scratch): workspace must be 0; the scratch is built in");
        return LRM_ERR_ARGUMENT;
    }
    const uint64_t need =
        lrm_op_decode_attention_workspace(desc->batch, desc->kv_heads, desc->pages_per_seq, desc->pages_per_split);
    if (need == 0 || need > LRM_DECODE_ATTN_STATIC_SCRATCH_BYTES) {
        lrm::set_thread_error("decode attention (static scratch): this call needs " + std::to_string(need) +
                              " bytes of scratch, above the built-in " +
                              std::to_string((unsigned long long)LRM_DECODE_ATTN_STATIC_SCRATCH_BYTES) +
                              " (use fewer rows or more pages per split, or lrm_op_decode_attention)");
        return LRM_ERR_ARGUMENT;
    }
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess || dev < 0 || dev >= 64) {
        lrm::set_thread_error("decode attention (static scratch): no usable current device");
        return LRM_ERR_CUDA;
    }
    void *scratch;
    {
        std::lock_guard<std::mutex> g(g_scratch_mu);
        if (!g_scratch_addr[dev]) {
            void *p = nullptr;
            e = cudaGetSymbolAddress(&p, g_decode_attn_scratch);
            if (e != cudaSuccess || !p) {
                lrm::set_thread_error(std::string("decode attention (static scratch): cudaGetSymbolAddress: ") +
                                      cudaGetErrorString(e));
                return LRM_ERR_CUDA;
            }
            g_scratch_addr[dev] = p;
        }
        scratch = g_scratch_addr[dev];
    }
    lrm_decode_attn_desc d = *desc;
    d.workspace = (uint64_t)(uintptr_t)scratch;
    return lrm_op_decode_attention(stream, &d);
}
