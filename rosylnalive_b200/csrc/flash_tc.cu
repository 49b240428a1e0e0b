// flash_tc.cu -- causal GQA prefill attention on the 5th-generation tensor cores (tcgen05, TMEM, TMA).
//
// One CTA owns 128 query rows of one head (rows of packed sequences, each starting at position 0) and walks the
// 128-key tiles up to the causal limit:
//   warp 0      TMA producer: Q once, then K and V tiles (3D tensor maps over [tokens][heads][128], 128-byte
//               swizzle, boxes of 64 dims x 128 rows) into a 2-stage ring;
//   warp 1      tensor-core issuer (one thread): S_j = Q K_j^T into one of two TMEM accumulators (128 x 128 fp32), and
//               O += P_j V_j into a third, with P from shared memory (K-major) and V read MN-major straight from its
//               [key][dim] tile (no transpose);
//   warps 2..5  softmax: thread = query row (its TMEM lane). Pass 1 reads the row of S for the tile maximum, pass 2
//               reads it again, writes P = exp2(S * scale * log2 e - m) as bf16 into the swizzled P tile and adds to
//               the row sum. The running maximum m only moves when a tile's maximum exceeds it by more than 8 (a
//               factor 256 in P); then O is rescaled in TMEM (tcgen05.ld / st) while the tensor core is idle on it.
//               At the end O / l is written as bf16.
// QK_{j+1} runs while the softmax of tile j runs. Every mbarrier wait is bounded and reports to the error word.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>

#include "internal.h"
#include "ptx.cuh"
#include "qwen.h"

namespace lrm {
namespace {

constexpr int TQ = 128, TK = 128, ST = 2;
constexpr int SUB = 128 * 64 * 2;  // one [128 rows][64] bf16 swizzled sub-tile
constexpr int TILE = 2 * SUB;      // [128 rows][128]
constexpr int SMEM_BYTES = TILE + ST * 2 * TILE + TILE + 1024 + 256;
constexpr int kThreads = 192;
constexpr float kRescaleThreshold = 8.0f;  // log2 units

struct FlashTcParams {
    const int32_t *cu_seqlens;
    __nv_bfloat16 *out;
    int nseq, max_len, q_heads, kv_heads;
    float scale_log2;
    uint32_t *err;
};

__device__ __forceinline__ uint32_t pack2(float a, float b) {
    __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t *>(&h);
}

__global__ void __launch_bounds__(kThreads, 1)
    flash_tc_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
                    const __grid_constant__ CUtensorMap tv, FlashTcParams p) {
    ptx::griddep_wait();
    ptx::griddep_launch();
    const int n_qt = (p.max_len + TQ - 1) / TQ;
    const int qt = n_qt - 1 - (int)blockIdx.x;  // the longest rows first
    const int h = blockIdx.y, seq = blockIdx.z;
    const int start = p.cu_seqlens[seq];
    const int len = p.cu_seqlens[seq + 1] - start;
    const int q0 = qt * TQ;
    if (q0 >= len) return;  // whole CTA, before any barrier or TMEM use
    const int kvh = h / (p.q_heads / p.kv_heads);
    const int n_kt = (min(len, q0 + TQ) - 1) / TK + 1;

    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = (uint8_t *)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    uint8_t *sQ = smem;
    uint8_t *sK = sQ + TILE;            // ST tiles
    uint8_t *sV = sK + ST * TILE;       // ST tiles
    uint8_t *sP = sV + ST * TILE;
    uint64_t *bars = (uint64_t *)(sP + TILE);
    uint64_t *q_full = bars;
    uint64_t *kv_full = bars + 1;       // ST
    uint64_t *kv_empty = kv_full + ST;  // ST
    uint64_t *s_full = kv_empty + ST;   // 2
    uint64_t *p_full = s_full + 2;
    uint64_t *o_done = p_full + 1;
    uint64_t *fin = o_done + 1;
    uint32_t *tmem_slot = (uint32_t *)(fin + 1);
    uint32_t *err = p.err;

    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    if (threadIdx.x == 0) {
        ptx::mbar_init(q_full, 1);
        for (int s = 0; s < ST; ++s) {
            ptx::mbar_init(&kv_full[s], 1);
            ptx::mbar_init(&kv_empty[s], 1);
        }
        ptx::mbar_init(&s_full[0], 1);
        ptx::mbar_init(&s_full[1], 1);
        ptx::mbar_init(p_full, 4);
        ptx::mbar_init(o_done, 1);
        ptx::mbar_init(fin, 1);
        ptx::fence_barrier_init();
        ptx::prefetch_tmap(&tq);
        ptx::prefetch_tmap(&tk);
        ptx::prefetch_tmap(&tv);
    }
    if (warp == 1) {
        ptx::tmem_alloc(tmem_slot, 512);
        ptx::tmem_relinquish();
    }
    ptx::tc_fence_before();
    __syncthreads();
    ptx::tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const uint32_t tS[2] = {tmem, tmem + 128};
    const uint32_t tO = tmem + 256;

    if (warp == 0) {
        if (ptx::elect_one()) {
            ptx::mbar_arrive_expect_tx(q_full, TILE);
            ptx::tma_load_3d(sQ, &tq, q_full, 0, h, start + q0);
            ptx::tma_load_3d(sQ + SUB, &tq, q_full, 64, h, start + q0);
            int j = 0;
            for (; j < n_kt; ++j) {
                const int s = j % ST;
                if (!ptx::mbar_wait(&kv_empty[s], ((j / ST) & 1) ^ 1, err, 0x3001)) break;
                ptx::mbar_arrive_expect_tx(&kv_full[s], 2 * TILE);
                const int rows = start + j * TK;
                ptx::tma_load_3d(sK + s * TILE, &tk, &kv_full[s], 0, kvh, rows);
                ptx::tma_load_3d(sK + s * TILE + SUB, &tk, &kv_full[s], 64, kvh, rows);
                ptx::tma_load_3d(sV + s * TILE, &tv, &kv_full[s], 0, kvh, rows);
                ptx::tma_load_3d(sV + s * TILE + SUB, &tv, &kv_full[s], 64, kvh, rows);
            }
            ptx::mbar_wait(q_full, 0, err, 0x3002);
            for (int i = j > ST ? j - ST : 0; i < j; ++i) ptx::mbar_wait(&kv_full[i % ST], (i / ST) & 1, err, 0x3002);
        }
    } else if (warp == 1) {
        if (ptx::elect_one()) {
            constexpr uint32_t idesc_qk = ptx::idesc_bf16_f32(128, 128, false);
            constexpr uint32_t idesc_pv = ptx::idesc_bf16_f32(128, 128, true);
            const uint32_t aQ = ptx::smem_u32(sQ), aP = ptx::smem_u32(sP);
            bool ok = ptx::mbar_wait(q_full, 0, err, 0x3003);
            auto issue_qk = [&](int j) -> bool {
                const int s = j % ST;
                if (!ptx::mbar_wait(&kv_full[s], (j / ST) & 1, err, 0x3004)) return false;
                ptx::tc_fence_after();
                const uint32_t aK = ptx::smem_u32(sK + s * TILE);
#pragma unroll
                for (int kk = 0; kk < 8; ++kk) {
                    const uint32_t off = (kk >> 2) * SUB + (kk & 3) * 32;
                    ptx::mma_bf16(tS[j & 1], ptx::sw128_kmajor_desc(aQ + off), ptx::sw128_kmajor_desc(aK + off),
                                  idesc_qk, kk > 0 ? 1u : 0u);
                }
                ptx::mma_commit(&s_full[j & 1]);
                return true;
            };
            if (ok) ok = issue_qk(0);
            for (int j = 0; ok && j < n_kt; ++j) {
                if (j + 1 < n_kt && !issue_qk(j + 1)) break;
                if (!ptx::mbar_wait(p_full, j & 1, err, 0x3005)) break;
                ptx::tc_fence_after();
                const uint32_t aV = ptx::smem_u32(sV + (j % ST) * TILE);
#pragma unroll
                for (int kk = 0; kk < 8; ++kk) {
                    const uint64_t da = ptx::sw128_kmajor_desc(aP + (kk >> 2) * SUB + (kk & 3) * 32);
                    const uint64_t db = ptx::sw128_mnmajor_desc(aV + kk * 2048, SUB, 1024);
                    ptx::mma_bf16(tO, da, db, idesc_pv, (j > 0 || kk > 0) ? 1u : 0u);
                }
                ptx::mma_commit(&kv_empty[j % ST]);
                ptx::mma_commit(o_done);
            }
            // No MMA may still be writing TMEM when it is freed (this matters on the error path).
            ptx::mma_commit(fin);
            ptx::mbar_wait(fin, 0, err, 0x3009);
        }
    } else {
        const int q = warp & 3;
        const int rl = q * 32 + lane;  // row within the tile
        const int row = q0 + rl;       // query position within the sequence
        const uint32_t lane_off = (uint32_t)(q * 32) << 16;
        float m_ref = -INFINITY, l = 0.f;
        bool ok = true;
        for (int j = 0; j < n_kt && ok; ++j) {
            if (!ptx::mbar_wait(&s_full[j & 1], (j >> 1) & 1, err, 0x3006)) {
                ok = false;
                break;
            }
            ptx::tc_fence_after();
            const uint32_t ts = tS[j & 1] + lane_off;
            const int key0 = j * TK;
            // pass 1: the tile maximum of this row (masked keys: beyond the row, or beyond the sequence)
            float tmax = -INFINITY;
#pragma unroll 1
            for (int c = 0; c < 8; c += 2) {
                uint32_t u0[16], u1[16];
                ptx::tmem_ld16(ts + c * 16, u0);
                ptx::tmem_ld16(ts + c * 16 + 16, u1);
                ptx::tmem_ld_wait();
#pragma unroll
                for (int e = 0; e < 16; ++e) {
                    const int k0 = key0 + c * 16 + e, k1 = k0 + 16;
                    if (k0 <= row && k0 < len) tmax = fmaxf(tmax, __uint_as_float(u0[e]) * p.scale_log2);
                    if (k1 <= row && k1 < len) tmax = fmaxf(tmax, __uint_as_float(u1[e]) * p.scale_log2);
                }
            }
            float alpha = 1.f;
            bool rescale = false;
            if (j == 0) {
                m_ref = tmax;
            } else if (tmax > m_ref + kRescaleThreshold) {
                alpha = exp2f(m_ref - tmax);
                m_ref = tmax;
                rescale = true;
            }
            // P_{j-1} V_{j-1} must be done before P is overwritten or O is rescaled.
            if (j > 0 && !ptx::mbar_wait(o_done, (j - 1) & 1, err, 0x3007)) {
                ok = false;
                break;
            }
            ptx::tc_fence_after();
            if (__any_sync(0xffffffffu, rescale)) {
                l *= alpha;
#pragma unroll 1
                for (int c = 0; c < 8; ++c) {
                    uint32_t u[16];
                    ptx::tmem_ld16(tO + lane_off + c * 16, u);
                    ptx::tmem_ld_wait();
#pragma unroll
                    for (int e = 0; e < 16; ++e) u[e] = __float_as_uint(__uint_as_float(u[e]) * alpha);
                    ptx::tmem_st16(tO + lane_off + c * 16, u);
                }
                ptx::tmem_st_wait();
            }
            // pass 2: P = exp2(s - m_ref) as bf16 into the swizzled P tile (K-major, two 64-key sub-tiles)
#pragma unroll 1
            for (int c = 0; c < 8; ++c) {
                uint32_t u[16];
                ptx::tmem_ld16(ts + c * 16, u);
                ptx::tmem_ld_wait();
                float pv[16];
#pragma unroll
                for (int e = 0; e < 16; ++e) {
                    const int key = key0 + c * 16 + e;
                    pv[e] = (key <= row && key < len) ? exp2f(__uint_as_float(u[e]) * p.scale_log2 - m_ref) : 0.f;
                    l += pv[e];
                }
                uint32_t w[8];
#pragma unroll
                for (int e = 0; e < 8; ++e) w[e] = pack2(pv[2 * e], pv[2 * e + 1]);
                const int sub = c >> 2, chunk = (c & 3) * 2;
                uint8_t *prow = sP + sub * SUB + rl * 128;
                *reinterpret_cast<uint4 *>(prow + (((chunk) ^ (rl & 7)) << 4)) = make_uint4(w[0], w[1], w[2], w[3]);
                *reinterpret_cast<uint4 *>(prow + (((chunk + 1) ^ (rl & 7)) << 4)) = make_uint4(w[4], w[5], w[6], w[7]);
            }
            ptx::fence_proxy_async();
            ptx::tc_fence_before();
            __syncwarp();
            if (lane == 0) ptx::mbar_arrive(p_full);
        }
        if (ok && ptx::mbar_wait(o_done, (n_kt - 1) & 1, err, 0x3008)) {
            ptx::tc_fence_after();
            const float inv = 1.f / l;
            __nv_bfloat16 *dst = p.out + ((size_t)(start + row) * p.q_heads + h) * kHeadDim;
#pragma unroll 1
            for (int c = 0; c < 8; ++c) {
                uint32_t u[16];
                ptx::tmem_ld16(tO + lane_off + c * 16, u);
                ptx::tmem_ld_wait();
                if (row < len) {
                    uint32_t w[8];
#pragma unroll
                    for (int e = 0; e < 8; ++e)
                        w[e] = pack2(__uint_as_float(u[2 * e]) * inv, __uint_as_float(u[2 * e + 1]) * inv);
                    uint4 *d4 = reinterpret_cast<uint4 *>(dst + c * 16);
                    d4[0] = make_uint4(w[0], w[1], w[2], w[3]);
                    d4[1] = make_uint4(w[4], w[5], w[6], w[7]);
                }
            }
        }
    }
    ptx::tc_fence_before();
    __syncthreads();
    ptx::tc_fence_after();
    if (warp == 1) ptx::tmem_dealloc(tmem, 512);
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                  const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_tiled_fn() {
    static EncodeTiledFn fn = nullptr;
    if (!fn) {
        void *ptr = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = (EncodeTiledFn)ptr;
    }
    return fn;
}

// [tokens][heads][128] bf16, boxes of 64 dims x 1 head x 128 tokens, 128-byte swizzle.
bool make_tmap_heads(CUtensorMap *map, const void *ptr, int heads, int tokens) {
    EncodeTiledFn enc = encode_tiled_fn();
    if (!enc) return false;
    cuuint64_t dims[3] = {128, (cuuint64_t)heads, (cuuint64_t)tokens};
    cuuint64_t strides[2] = {256, (cuuint64_t)heads * 256};
    cuuint32_t box[3] = {64, 1, 128};
    cuuint32_t estr[3] = {1, 1, 1};
    return enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void *>(ptr), dims, strides, box, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace

cudaError_t launch_prefill_attention_tc(const PrefillAttnArgs &a, int total_tokens, uint32_t *err, cudaStream_t st) {
    CUtensorMap tq, tk, tv;
    if (!make_tmap_heads(&tq, a.q, a.q_heads, total_tokens) || !make_tmap_heads(&tk, a.k, a.kv_heads, total_tokens) ||
        !make_tmap_heads(&tv, a.v, a.kv_heads, total_tokens))
        return cudaErrorInvalidValue;
    static bool configured[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (!configured[dev & 63]) {
        cudaError_t e = cudaFuncSetAttribute(flash_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
        if (e != cudaSuccess) return e;
        configured[dev & 63] = true;
    }
    FlashTcParams p;
    p.cu_seqlens = a.cu_seqlens;
    p.out = a.out;
    p.nseq = a.nseq;
    p.max_len = a.max_len;
    p.q_heads = a.q_heads;
    p.kv_heads = a.kv_heads;
    p.scale_log2 = a.scale_log2;
    p.err = err;
    dim3 grid((a.max_len + TQ - 1) / TQ, a.q_heads, a.nseq);
    return launch_kernel(flash_tc_kernel, grid, dim3(kThreads), SMEM_BYTES, st, tq, tk, tv, p);
}

}  // namespace lrm
