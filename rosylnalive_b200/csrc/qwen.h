// qwen.h -- the bf16 forward path's fused kernels (internal launch interface).
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace lrm {

// Paged KV cache (bf16): per layer [pages][kv_heads][2 (K, V)][kPageTokens][head_dim]; one page of one head is a
// contiguous 8 KiB block (K 4 KiB then V 4 KiB at head_dim 128), the unit the decode kernel streams.
constexpr int kPageTokens = 16;
constexpr int kHeadDim = 128;

struct KvLayout {
    __nv_bfloat16 *pool;      // this layer's pool
    const int32_t *pages;     // page table [max_seqs][max_pages_per_seq]
    int32_t max_pages_per_seq;
    int32_t kv_heads;
};

__host__ __device__ inline size_t kv_page_elems(int kv_heads) { return (size_t)kv_heads * 2 * kPageTokens * kHeadDim; }

// xn[t] = bf16(rmsnorm(x[idx[t]]) * w) for t < T (rows 0..T-1 without idx), one block a row: the final norm before
// the lm_head.
cudaError_t launch_norm_rows_block(const float *x, int T, int hidden, const __nv_bfloat16 *w, float eps,
                                   __nv_bfloat16 *xn, cudaStream_t st, const int32_t *idx = nullptr);

// Paged split-K decode attention: one query per sequence (row b, slot slots[b], seq_len[slot] keys including the new
// one), GQA group 2, pages_per_split pages per CTA; then the combine writes out bf16 [B][q_heads][128].
struct DecodeAttnArgs {
    const __nv_bfloat16 *q;  // [B][q_heads][128]
    KvLayout kv;
    const int32_t *slots;    // [B]
    const int32_t *seq_len;  // [max_seqs]
    int B, q_heads;
    int pages_per_split, max_splits;
    float scale_log2;        // head_dim^-0.5 * log2(e)
    float *part_o;           // [B][kv_heads][max_splits][2][128]
    float *part_ml;          // [B][kv_heads][max_splits][2][2]
    __nv_bfloat16 *out;      // [B][q_heads][128]
    uint32_t *err;
    // Set only when no kernel that can still be running once the previous kernel's CTAs have all started writes
    // slots, seq_len, the page table or any cached K/V other than the new token's (in each row's last page): then
    // those are read, and a split's first pages other than a row's last page are loaded, before the previous kernel
    // completes (the engine's decode step, where the previous kernel appends the new token and writes q). Otherwise
    // everything is read after it.
    bool early_pages = false;
};
// A row whose seq_len is below 1 or needs more pages than its page-table row (or than max_splits splits hold) is
// not read: the attention kernel writes kErrDecodeLen into err and the combine writes the row's output as zeros.
constexpr uint32_t kErrDecodeLen = 0x2010;
cudaError_t launch_decode_attention(const DecodeAttnArgs &a, cudaStream_t st);

// Causal prefill attention for query rows q [T][q_heads][128] of sequences packed by cu_seqlens; out bf16
// [T][q_heads][128]. K/V either contiguous (k/v [T][kv_heads][128], positions from 0 in each sequence; pool null) or
// paged (pool non-null: sequence i's rows continue past[i] cached tokens of slot seq_slot[i], and its keys
// 0 .. past[i] + rows - 1 are read from the cache, where the rows' own k/v must already be).
struct PrefillAttnArgs {
    const __nv_bfloat16 *q, *k = nullptr, *v = nullptr;
    __nv_bfloat16 *out;
    const int32_t *cu_seqlens;  // [nseq + 1]
    int nseq, max_len, q_heads, kv_heads;
    float scale_log2;
    const __nv_bfloat16 *pool = nullptr;  // this layer's pool [kv_pages][kv_heads][2][16][128]
    const int32_t *pages = nullptr, *seq_slot = nullptr, *past = nullptr;
    int pages_per_seq = 0, kv_pages = 0;
};
// A prefill sequence whose rows fall outside total_tokens, longer than max_len, or with past < 0 is not computed:
// the kernel writes kErrPrefillSeq into err and leaves its output rows unwritten.
constexpr uint32_t kErrPrefillSeq = 0x3010;
// Runs on tcgen05 tensor cores (TMA tiles, TMEM accumulators); total_tokens = rows of q/k/v.
cudaError_t launch_prefill_attention_tc(const PrefillAttnArgs &a, int total_tokens, uint32_t *err, cudaStream_t st);

// rows[r] = argmax of logits[r] ([R][V] fp32): lowest index of the maximum, 0xFFFFFFFF for a row holding a NaN.
cudaError_t launch_argmax(const float *logits, int R, int V, uint32_t *out, cudaStream_t st);

// seq_len[slots[b]] += 1 for b < B (after a decode step's append).
cudaError_t launch_advance(const int32_t *slots, int B, int32_t *seq_len, int32_t *tok_pos, cudaStream_t st);

}  // namespace lrm
