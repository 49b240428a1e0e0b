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
#include "ptx.cuh"
#include "qwen.h"

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

namespace {
// The bounded wait every kernel of this library uses (ptx::mbar_wait), on an mbarrier that nothing ever arrives on:
// the wait gives up after `polls` polls, records `code` in the error word and the kernel returns. No copy is issued,
// so nothing is in flight when it returns.
__global__ void wait_probe_kernel(uint32_t polls, uint32_t code, uint32_t *err) {
    __shared__ __align__(8) uint64_t bar;
    if (threadIdx.x == 0) {
        ptx::mbar_init(&bar, 1);
        ptx::fence_barrier_init();
    }
    __syncthreads();
    if (threadIdx.x == 0) ptx::mbar_wait(&bar, 0, err, code, polls);
}
}  // namespace

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
    if (d->m < 1 || d->n < 1 || d->k < 1 || d->m > (1 << 30) || d->n > (1 << 30) || d->k > (1 << 30))
        return op_fail(LRM_ERR_ARGUMENT, "gemm: M, N and K must be 1 .. 2^30");
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
    a.cta_pair = d->cta_pair;
    a.err = device_error_word();
    if (!a.err) return LRM_ERR_CUDA;
    if (d->epilogue < 0 || d->epilogue > 4) return op_fail(LRM_ERR_ARGUMENT, "unknown epilogue");
    if (const char *why = gemm_check(a)) return op_fail(LRM_ERR_ARGUMENT, std::string("gemm: ") + why);
    return op_cuda(gemm_launch(a, device_sms(), (cudaStream_t)stream), "gemm");
}

lrm_status lrm_op_prefill_attention(void *stream, const lrm_prefill_attn_desc *d) {
    if (!d) return op_fail(LRM_ERR_ARGUMENT, "descriptor is null");
    if (d->head_dim != kHeadDim) return op_fail(LRM_ERR_ARGUMENT, "prefill attention needs head_dim 128");
    if (d->nseq < 1 || d->nseq > 65535 || d->max_len < 1 || d->q_heads < 1 || d->q_heads > 65535 ||
        d->kv_heads < 1 || d->q_heads % d->kv_heads)
        return op_fail(LRM_ERR_ARGUMENT, "prefill attention: bad sizes (kv_heads must divide q_heads)");
    if (!d->q || !d->k || !d->v || !d->out || !d->cu_seqlens || ((d->q | d->k | d->v | d->out) & 15))
        return op_fail(LRM_ERR_ARGUMENT, "prefill attention: pointers must be non-null and 16-byte aligned");
    if (d->total_tokens < 1) return op_fail(LRM_ERR_ARGUMENT, "prefill attention: total_tokens must be positive");
    if (d->max_len > 65535 * 128)  // one grid z index per 128-row query tile
        return op_fail(LRM_ERR_ARGUMENT, "prefill attention: max_len must be at most 65535 * 128");
    uint32_t *err = device_error_word();
    if (!err) return LRM_ERR_CUDA;
    PrefillAttnArgs a;
    a.q = (const __nv_bfloat16 *)d->q;
    a.k = (const __nv_bfloat16 *)d->k;
    a.v = (const __nv_bfloat16 *)d->v;
    a.out = (__nv_bfloat16 *)d->out;
    a.cu_seqlens = (const int32_t *)d->cu_seqlens;
    a.nseq = d->nseq;
    a.max_len = d->max_len;
    a.q_heads = d->q_heads;
    a.kv_heads = d->kv_heads;
    a.scale_log2 = d->scale * 1.4426950408889634f;
    return op_cuda(launch_prefill_attention_tc(a, d->total_tokens, err, (cudaStream_t)stream), "prefill attention");
}

// Page counts above 2^20 (16M tokens a sequence) are refused, so split counts and scratch sizes stay far from
// overflow in every integer type they pass through.
static constexpr int32_t kMaxDecodePages = 1 << 20;

lrm_status lrm_op_wait_probe(void *stream, uint32_t polls, uint32_t code) {
    if (polls < 1 || polls > ptx::kWaitLimit) return op_fail(LRM_ERR_ARGUMENT, "wait probe: polls must be 1 .. 2^24");
    if (code == 0) return op_fail(LRM_ERR_ARGUMENT, "wait probe: the code must be nonzero");
    uint32_t *err = device_error_word();
    if (!err) return LRM_ERR_CUDA;
    wait_probe_kernel<<<1, 32, 0, (cudaStream_t)stream>>>(polls, code, err);
    return op_cuda(cudaGetLastError(), "wait probe");
}

lrm_status lrm_op_argmax_rows(void *stream, const float *logits, int32_t rows, int32_t vocab, uint32_t *out) {
    if (!logits || !out) return op_fail(LRM_ERR_ARGUMENT, "argmax: null pointer");
    if (rows < 1 || rows > 65535) return op_fail(LRM_ERR_ARGUMENT, "argmax: rows must be 1 .. 65535");
    // the kernel's column arithmetic (chunk rounding, strides of 1024) is int32: a bound well below INT_MAX
    if (vocab < 1 || vocab > (1 << 30)) return op_fail(LRM_ERR_ARGUMENT, "argmax: vocab must be 1 .. 2^30");
    if (vocab % 4 == 0 && ((uintptr_t)logits & 15))
        return op_fail(LRM_ERR_ARGUMENT, "argmax: logits must be 16-byte aligned when vocab is a multiple of 4");
    return op_cuda(launch_argmax(logits, rows, vocab, out, (cudaStream_t)stream), "argmax");
}

uint64_t lrm_op_decode_attention_workspace(int32_t batch, int32_t kv_heads, int32_t pages_per_seq,
                                           int32_t pages_per_split) {
    if (batch < 1 || kv_heads < 1 || pages_per_seq < 1 || pages_per_split < 1) return 0;
    if (pages_per_seq > kMaxDecodePages || pages_per_split > kMaxDecodePages) return 0;
    const uint64_t splits = ((uint64_t)pages_per_seq + (uint64_t)pages_per_split - 1) / (uint64_t)pages_per_split;
    const uint64_t states = (uint64_t)batch * kv_heads * splits * 2;
    return states * (128 + 2) * sizeof(float);
}

// Fills the launch arguments shared by both decode-attention entry points; nullptr or the reason it refuses.
static const char *decode_attn_args(const lrm_decode_attn_desc *d, DecodeAttnArgs &a) {
    if (d->head_dim != kHeadDim) return "decode attention needs head_dim 128";
    if (d->batch < 1 || d->batch > 65535 || d->kv_heads < 1 || d->kv_heads > 65535 || d->q_heads != 2 * d->kv_heads)
        return "decode attention: bad sizes (q_heads must be 2 * kv_heads)";
    if (d->pages_per_seq < 1 || d->pages_per_split < 1) return "decode attention: page counts must be positive";
    if (d->pages_per_seq > kMaxDecodePages || d->pages_per_split > kMaxDecodePages)
        return "decode attention: pages_per_seq and pages_per_split must be at most 2^20";
    if (!d->q || !d->pool || !d->page_table || !d->seq_len || !d->slots || !d->out)
        return "decode attention: null pointer";
    if ((d->q | d->pool | d->out) & 15) return "decode attention: q, pool and out must be 16-byte aligned";
    a.q = (const __nv_bfloat16 *)d->q;
    a.kv = KvLayout{(__nv_bfloat16 *)d->pool, (const int32_t *)d->page_table, d->pages_per_seq, d->kv_heads};
    a.slots = (const int32_t *)d->slots;
    a.seq_len = (const int32_t *)d->seq_len;
    a.B = d->batch;
    a.q_heads = d->q_heads;
    a.pages_per_split = d->pages_per_split;
    a.max_splits = (int32_t)(((int64_t)d->pages_per_seq + d->pages_per_split - 1) / d->pages_per_split);
    a.scale_log2 = d->scale * 1.4426950408889634f;
    a.out = (__nv_bfloat16 *)d->out;
    return nullptr;
}

lrm_status lrm_op_decode_attention(void *stream, const lrm_decode_attn_desc *d) {
    if (!d) return op_fail(LRM_ERR_ARGUMENT, "descriptor is null");
    DecodeAttnArgs a;
    if (const char *why = decode_attn_args(d, a)) return op_fail(LRM_ERR_ARGUMENT, why);
    if (!d->workspace || (d->workspace & 15))
        return op_fail(LRM_ERR_ARGUMENT, "decode attention: the workspace must be non-null and 16-byte aligned");
    const size_t states = (size_t)a.B * d->kv_heads * a.max_splits * 2;
    a.part_o = (float *)d->workspace;
    a.part_ml = a.part_o + states * 128;
    a.err = device_error_word();
    if (!a.err) return LRM_ERR_CUDA;
    return op_cuda(launch_decode_attention(a, (cudaStream_t)stream), "decode attention");
}

}  // extern "C"
