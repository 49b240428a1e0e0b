// gemm.h -- the tcgen05 GEMM's arguments (internal).
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace lrm {

enum GemmEpi : int { EPI_F32 = 0, EPI_RESID = 1, EPI_SWIGLU = 2, EPI_PARTIAL = 3, EPI_BF16 = 4, EPI_QKV = 5 };

// The q/k/v epilogue (EPI_QKV): the output columns are head rows of 128 (q heads, then k heads, then v heads); each
// thread owns one token row of one head, applies the per-head RMSNorm (q_norm / k_norm) and NeoX RoPE to q and k at
// the token's position, and writes bf16 q to q_out [T][q_heads][128], k and v into the paged cache (pool
// [pages][kv_heads][2][16][128], page table [slots][pages_per_seq]) and, when k_out / v_out are not null, to
// contiguous copies [T][kv_heads][128].
struct QkvEpilogue {
    __nv_bfloat16 *q_out, *k_out, *v_out, *pool;
    const int32_t *pages;
    int pages_per_seq;
    int q_heads, kv_heads;
    const __nv_bfloat16 *q_norm, *k_norm;
    float eps;
    const float *cos_t, *sin_t;  // [max_pos][64]
    const int32_t *tok_slot, *tok_pos;
};

struct GemmArgs {
    int M, N, K;
    const void *A;  // bf16 [M, K]
    const void *B;  // bf16 [N, K]
    int epi;
    int bn;            // 64, 128 or 256
    int splits;        // split-K count (EPI_PARTIAL only)
    int kb_per_split;  // 64-wide k blocks per split
    float *out_f32;
    __nv_bfloat16 *out_bf16;
    int ldo;  // leading dimension of the output (elements); for EPI_PARTIAL the token stride (= M)
    const float *resid;
    int ldr;
    float *partial;
    size_t split_stride;  // elements between split slices of `partial`
    uint32_t *err;        // device error word: bounded waits write a code here
    // Which operand no earlier kernel writes (1 = A, 2 = B, 0 = neither): under programmatic dependent launch its
    // first k-blocks are prefetched before the kernel waits for the previous one (decode: the weights).
    int independent;
    QkvEpilogue qkv;  // EPI_QKV only
    // 0 chooses; 1 one CTA per 128 x bn tile; 2 pairs of CTAs (a cluster of two SMs) sharing 256 x 256 tiles through
    // tcgen05 cta_group::2 MMAs (bn 256, one split, not EPI_PARTIAL).
    int cta_pair;
};

// nullptr when the arguments are valid, else the reason.
const char *gemm_check(const GemmArgs &a);
// Encodes the tensor maps and launches the persistent kernel on `sms` CTAs at most.
cudaError_t gemm_launch(const GemmArgs &a, int sms, cudaStream_t stream);
// Whether gemm_launch runs `a` on CTA pairs.
bool gemm_uses_pair(const GemmArgs &a);

}  // namespace lrm
