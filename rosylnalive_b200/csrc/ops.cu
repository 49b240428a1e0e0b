// ops.cu -- the fast-path operators on device memory (include/lrm_cuda.h, "fast-path operators"): argument checks,
// the per-device error word that bounded in-kernel waits report to, and launches on a caller's stream.
#include <cuda_runtime.h>
#include <stdio.h>
#include <string.h>

#include <mutex>
#include <string>

#include "../../include/lrm_cuda.h"
#include "gemm.h"
#include "internal.h"

namespace lrm {

// One error word per device; kernels write a nonzero code here when a bounded wait gives up.
__device__ uint32_t g_error_word;

namespace {
struct DeviceState {
    bool init = false;
    uint32_t *err = nullptr;  // device address of g_error_word, from cudaGetSymbolAddress
    int sms = 0;
};
DeviceState g_dev[64];
std::mutex g_mu;
}  // namespace

// Returns the device state of the current device (initialising it once), or nullptr with the thread error set.
static DeviceState *device_state() {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
        set_thread_error("no current CUDA device");
        return nullptr;
    }
    std::lock_guard<std::mutex> g(g_mu);
    DeviceState &s = g_dev[dev];
    if (!s.init) {
        void *p = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&p, g_error_word);
        if (e != cudaSuccess) {
            set_thread_error(std::string("cudaGetSymbolAddress(error word): ") + cudaGetErrorString(e));
            return nullptr;
        }
        s.err = (uint32_t *)p;
        cudaDeviceGetAttribute(&s.sms, cudaDevAttrMultiProcessorCount, dev);
        s.init = true;
    }
    return &s;
}

uint32_t *device_error_word() {
    DeviceState *s = device_state();
    return s ? s->err : nullptr;
}

int device_sms() {
    DeviceState *s = device_state();
    return s ? s->sms : 148;
}

lrm_status op_fail(lrm_status s, const std::string &m) {
    set_thread_error(m);
    return s;
}

lrm_status op_cuda(cudaError_t e, const char *what) {
    if (e == cudaSuccess) return LRM_OK;
    return op_fail(LRM_ERR_CUDA, std::string(what) + ": " + cudaGetErrorName(e) + " (" + cudaGetErrorString(e) + ")");
}

}  // namespace lrm

using namespace lrm;

extern "C" {

lrm_status lrm_op_set_device(int32_t device) {
    cudaError_t e = cudaSetDevice(device);
    if (e != cudaSuccess) return op_cuda(e, "cudaSetDevice");
    return device_state() ? LRM_OK : LRM_ERR_CUDA;
}

lrm_status lrm_op_error_word(uint32_t *code, int32_t clear) {
    if (!code) return op_fail(LRM_ERR_ARGUMENT, "code is null");
    uint32_t *p = device_error_word();
    if (!p) return LRM_ERR_CUDA;
    cudaError_t e = cudaMemcpy(code, p, 4, cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) return op_cuda(e, "reading the error word");
    if (clear) {
        e = cudaMemset(p, 0, 4);
        if (e != cudaSuccess) return op_cuda(e, "clearing the error word");
    }
    return LRM_OK;
}

lrm_status lrm_op_gemm_bf16(void *stream, const lrm_gemm_desc *d) {
    if (!d) return op_fail(LRM_ERR_ARGUMENT, "descriptor is null");
    GemmArgs a;
    memset(&a, 0, sizeof a);
    a.M = d->m;
    a.N = d->n;
    a.K = d->k;
    a.A = (const void *)d->a;
    a.B = (const void *)d->b;
    a.epi = d->epilogue;
    a.bn = d->bn ? d->bn : (d->n >= 256 ? 256 : (d->n >= 128 ? 128 : 64));
    a.splits = d->splits < 1 ? 1 : d->splits;
    int nkb = (d->k + 63) / 64;
    a.kb_per_split = (nkb + a.splits - 1) / a.splits;
    if (d->epilogue == EPI_SWIGLU || d->epilogue == EPI_BF16)
        a.out_bf16 = (__nv_bfloat16 *)d->out;
    else if (d->epilogue == EPI_PARTIAL)
        a.partial = (float *)d->out;
    else
        a.out_f32 = (float *)d->out;
    a.ldo = d->ldo;
    a.resid = (const float *)d->resid;
    a.ldr = d->ldr;
    a.split_stride = d->split_stride;
    a.err = device_error_word();
    if (!a.err) return LRM_ERR_CUDA;
    if (d->epilogue < 0 || d->epilogue > 4) return op_fail(LRM_ERR_ARGUMENT, "unknown epilogue");
    if (const char *why = gemm_check(a)) return op_fail(LRM_ERR_ARGUMENT, std::string("gemm: ") + why);
    return op_cuda(gemm_launch(a, device_sms(), (cudaStream_t)stream), "gemm");
}

}  // extern "C"
