// gemm.h -- the tcgen05 GEMM's arguments (internal).
#pragma once

#include <cuda.h>
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
    // RMSNorm fused into the prefill GEMMs (CTA pairs only). A residual GEMM (EPI_RESID) with norm_u also writes the
    // next norm's inputs: u[m][n] = bf16(norm_gain[n] * out[m][n]) (row stride ldo) and, per row and 256-column
    // tile, the sum of squares of out (norm_ss[n / 256][m], row stride norm_ss_stride; the order of
    // pair_prep_kernel). A consumer (EPI_SWIGLU, EPI_QKV) with row_ss reads such u as A and multiplies each output
    // row by r[m] = 1 / sqrt(sum_g row_ss[g][m] / row_hidden + row_eps), groups in order: the norm's scale, which
    // the GEMM, linear in each row, may apply afterwards.
    const __nv_bfloat16 *norm_gain;
    __nv_bfloat16 *norm_u;
    float *norm_ss;
    size_t norm_ss_stride;
    const float *row_ss;
    int row_nss, row_hidden;
    size_t row_ss_stride;
    float row_eps;
};

// ---- decode GEMMs with their consumers fused (gemm_decode.cu) ----------------------------------------------------
//
// Y = A * B^T with A the weights [M, K] (M in 128-row tiles) and B the step's tokens [N, K] (N in 64-token tiles).
// S CTAs (one cluster) split K for one output tile; they reduce their accumulators through distributed shared memory
// in split order, and each finishes a share of the tile's tokens with the epilogue. B is a token's activation before
// its RMSNorm scale: B[t] = bf16(gain * x[t]); the scale r[t] = 1 / sqrt(sum_g ss[g][t] / hidden + eps) is applied to
// the output rows (the GEMM is linear in each token), so no kernel has to finish a whole row's norm before the GEMM.
enum DecodeEpi : int {
    DEC_QKV = 0,     // y = r * acc per head row (q heads, then k, then v): q/k get the per-head RMSNorm and RoPE; q to
                     // q_out [N][q_heads][128], k and v into the paged cache at (tok_slot[t], tok_pos[t])
    DEC_SWIGLU = 1,  // tile rows 0..63 gate j, 64..127 up j (64-row interleave): act[t][64 mt + j] = bf16(silu(r g) r u)
    DEC_RESID = 2,   // x[t][m] += acc; with gain: u[t][m] = bf16(gain[m] x[t][m]) and ss_out[m / 128][t] = the sum of
                     // x[t][m]^2 over the tile's 128 rows (decode_group_ss), the next GEMM's B and norm inputs
};

struct DecodeGemmArgs {
    int M, N, K;
    const void *A, *B;
    int epi;
    int splits, kb_per_split;  // S CTAs of a cluster split the K blocks (64 wide): kb_per_split each
    // the norm scale of B's rows (null: 1)
    const float *ss;
    int nss, hidden;
    size_t ss_stride;  // elements between groups of ss (and of ss_out)
    float eps;
    // DEC_RESID
    float *x;
    __nv_bfloat16 *u;
    const __nv_bfloat16 *gain;  // null: x only
    float *ss_out;
    // DEC_SWIGLU
    __nv_bfloat16 *act;
    int ld_act;
    // DEC_QKV (fields as QkvEpilogue)
    QkvEpilogue qkv;
    uint32_t *err;
};

const char *decode_gemm_check(const DecodeGemmArgs &a);
cudaError_t decode_gemm_launch(const DecodeGemmArgs &a, cudaStream_t stream);
// The split count for an M x K weight: clusters of at most 8 CTAs, at most one CTA an SM for one 64-token tile,
// every split at most kDecodeStages k blocks when possible (all of a CTA's weights are fetched before it waits).
int decode_gemm_splits(int M, int K, int sms);

// The decode step's norm inputs from the residual stream, as DEC_RESID writes them: u[t] = bf16(gain * x[t]) and
// ss[g][t] for 128-column groups g. With ids, x[t] = widen(embed[ids[t]]) is written first (a quiet NaN row for an id
// outside the vocabulary).
cudaError_t launch_decode_prep(const uint32_t *ids, const __nv_bfloat16 *embed, int vocab, float *x, int T,
                               int hidden, const __nv_bfloat16 *gain, __nv_bfloat16 *u, float *ss, size_t ss_stride,
                               cudaStream_t st);

// The prefill norm inputs from the residual stream in the order a residual GEMM with norm_u writes them (a pipeline
// stage that resumes a prefill): u[t] = bf16(gain * x[t]) and ss[g][t] per 256-column group g.
cudaError_t launch_pair_prep(const float *x, int T, int hidden, const __nv_bfloat16 *gain, __nv_bfloat16 *u, float *ss,
                             size_t ss_stride, cudaStream_t st);

// A tensor map over bf16 [rows, cols] (row-major, 16-byte aligned rows): boxes of 64 columns x box_rows rows with the
// 128-byte swizzle the tcgen05 operand descriptors expect.
bool gemm_tmap_2d(CUtensorMap *map, const void *ptr, uint64_t rows, uint64_t cols, uint32_t box_rows);

// nullptr when the arguments are valid, else the reason.
const char *gemm_check(const GemmArgs &a);
// Encodes the tensor maps and launches the persistent kernel on `sms` CTAs at most.
cudaError_t gemm_launch(const GemmArgs &a, int sms, cudaStream_t stream);
// Whether gemm_launch runs `a` on CTA pairs.
bool gemm_uses_pair(const GemmArgs &a);

}  // namespace lrm
