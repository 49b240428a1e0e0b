// flash_tc.cu -- causal GQA prefill attention on the 5th-generation tensor cores (tcgen05, TMEM, TMA).
//
// One CTA owns 128 query rows of up to two query heads that share a KV head (two "slots"; one when the group size
// q_heads / kv_heads is odd), so every K/V tile is loaded once for both, and walks the 128-key tiles up to the causal
// limit. K and V come either from contiguous [tokens][kv_heads][128] arrays (sequences packed, positions from 0) or
// from the paged KV cache (a 128-key tile = 8 pages of 16 tokens, one TMA box per page and half tile), in which case
// a sequence's rows are a chunk that continues `past` cached tokens: chunked prefill, and prefill onto a decoded
// sequence, attend to every cached key with the same per-row arithmetic as one whole prefill. Tensor memory (512 columns) holds per slot S (128 x 128 fp32) and O (128 x 128 fp32); P overwrites S in
// place as bf16 and the P V product reads it from tensor memory, so P never goes through shared memory.
//   warp 0      TMA producer: Q of both slots once, then K_0, V_0, K_1, V_1, ... (3D tensor maps over
//               [tokens][heads][128], 128-byte swizzle, boxes of 64 dims x 128 rows) through a ring of five 32 KiB
//               stages; K_j is released once both slots' S_j have read it, V_j after both P V_j;
//   warp 1      tensor-core issuer (one thread): S_s = Q_s K_0^T for both slots, then per key tile j and slot s
//               O_s += P_s V_j (V read MN-major straight from its [key][dim] tile) followed at once by
//               S_s = Q_s K_{j+1}^T. The tensor core executes one thread's MMAs in issue order, so S_{j+1}
//               overwrites P_s only after P_s V_j has read it;
//   warps 4..11 softmax, one warpgroup per slot, thread = query row (its TMEM lane): the row of S comes into
//               registers in one go, keys past the row or the sequence are masked (diagonal and tail tiles only),
//               P = 2^(S * scale * log2 e - m) is written back as bf16 (announced in two parts, so P V starts on
//               keys 0..95 while 96..127 are stored) and summed in fp32. The reference maximum m
//               only moves when a tile's maximum exceeds it by more than 8 (a factor 256 in P); then O is rescaled
//               in tensor memory, which is safe there because S_j completing implies P V_{j-1} has. At the end O / l
//               is written as bf16.
// While one slot's softmax runs, the tensor core works on the other slot. Every mbarrier wait is bounded and
// reports to the error word.
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

constexpr int TQ = 128, TK = 128, KV_ST = 5, SLOTS = 2;
constexpr int SUB = 128 * 64 * 2;  // one [128 rows][64] bf16 swizzled sub-tile
constexpr int TILE = 2 * SUB;      // [128 rows][128]
constexpr int SMEM_BYTES = SLOTS * TILE + KV_ST * TILE + 1024 + 256;
constexpr int P_SPLIT = 48;  // P is announced in two parts: keys 0..95 (48 packed columns), then 96..127
constexpr int kThreads = 384;      // warpgroup 0: producer, issuer (two warps idle); warpgroups 1, 2: softmax
constexpr int kRegsLaunch = 168;    // 65536 / 384, rounded down to the allocation unit of 8
constexpr int kRegsControl = 56, kRegsSoftmax = 224;
static_assert(128 * kRegsControl + 256 * kRegsSoftmax <= kThreads * kRegsLaunch, "register split exceeds the launch");
constexpr float kRescaleThreshold = 8.0f;  // log2 units
struct FlashTcParams {
    const int32_t *cu_seqlens;
    __nv_bfloat16 *out;
    int nseq, max_len, q_heads, kv_heads, heads_per_cta;
    float scale_log2;
    uint32_t *err;
    // paged K/V (paged != 0): page table [slots][pages_per_seq], each sequence's slot and cached tokens before it
    const int32_t *pages, *seq_slot, *past;
    int pages_per_seq, paged;
    int total_tokens;  // rows of q and out: every sequence must lie inside them
};

__device__ __forceinline__ uint32_t pack2(float a, float b) {
    __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t *>(&h);
}

// fp32 pairs on the packed FMA pipe (fma / add .rn.f32x2, sm_100): two results per instruction.
__device__ __forceinline__ void fma2(float &d0, float &d1, float a0, float a1, float b0, float b1, float c0,
                                     float c1) {
    asm("{\n\t.reg .b64 a, b, c, d;\n\tmov.b64 a, {%2, %3};\n\tmov.b64 b, {%4, %5};\n\tmov.b64 c, {%6, %7};\n\t"
        "fma.rn.f32x2 d, a, b, c;\n\tmov.b64 {%0, %1}, d;\n\t}"
        : "=f"(d0), "=f"(d1)
        : "f"(a0), "f"(a1), "f"(b0), "f"(b1), "f"(c0), "f"(c1));
}
__device__ __forceinline__ void add2(float &d0, float &d1, float a0, float a1, float b0, float b1) {
    asm("{\n\t.reg .b64 a, b, d;\n\tmov.b64 a, {%2, %3};\n\tmov.b64 b, {%4, %5};\n\t"
        "add.rn.f32x2 d, a, b;\n\tmov.b64 {%0, %1}, d;\n\t}"
        : "=f"(d0), "=f"(d1)
        : "f"(a0), "f"(a1), "f"(b0), "f"(b1));
}

__device__ __forceinline__ float max3(float a, float b, float c) {
    float r;
    asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
    return r;
}

__global__ void __launch_bounds__(kThreads, 1)
    flash_tc_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
                    const __grid_constant__ CUtensorMap tv, FlashTcParams p) {
    ptx::griddep_wait();
    ptx::griddep_launch();
    const int n_qt = (p.max_len + TQ - 1) / TQ;
    const int qt = n_qt - 1 - (int)blockIdx.z;  // the longest query tiles of every head and sequence first
    const int h0 = blockIdx.x * p.heads_per_cta, seq = blockIdx.y;
    const int nslots = p.heads_per_cta;
    const int start = p.cu_seqlens[seq];
    const int len = p.cu_seqlens[seq + 1] - start;
    const int q0 = qt * TQ;
    const int past = p.paged ? p.past[seq] : 0;  // row r of the chunk is position past + r
    // cu_seqlens and past live in device memory, so the host cannot check them: a sequence outside the q/out rows,
    // longer than max_len, or with negative cached tokens is not computed (its rows are left as they were) and
    // one CTA of it records the code. Whole CTA, before any barrier, TMEM use or copy.
    if (start < 0 || len < 0 || len > p.max_len || start > p.total_tokens - len || past < 0) {
        if (blockIdx.x == 0 && blockIdx.z == 0 && threadIdx.x == 0) atomicCAS(p.err, 0u, kErrPrefillSeq);
        return;
    }
    if (q0 >= len) return;  // whole CTA, before any barrier or TMEM use
    const int kvh = h0 / (p.q_heads / p.kv_heads);
    const int n_kt = (past + min(len, q0 + TQ) - 1) / TK + 1;

    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = (uint8_t *)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    uint8_t *sQ = smem;                  // SLOTS tiles
    uint8_t *sKV = sQ + SLOTS * TILE;    // KV_ST tiles: item 2j is K_j, item 2j + 1 is V_j
    uint64_t *bars = (uint64_t *)(sKV + KV_ST * TILE);
    uint64_t *q_full = bars;
    uint64_t *kv_full = q_full + 1;      // KV_ST
    uint64_t *kv_empty = kv_full + KV_ST; // KV_ST
    uint64_t *s_full = kv_empty + KV_ST; // SLOTS
    uint64_t *p_part = s_full + SLOTS;   // SLOTS: P keys 0..95 written
    uint64_t *p_full = p_part + SLOTS;   // SLOTS: all of P written
    uint64_t *o_done = p_full + SLOTS;   // SLOTS: the last P V of the slot has completed
    uint64_t *fin = o_done + SLOTS;
    uint32_t *tmem_slot = (uint32_t *)(fin + 1);
    uint32_t *err = p.err;

    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    if (threadIdx.x == 0) {
        ptx::mbar_init(q_full, 1);
        for (int s = 0; s < KV_ST; ++s) {
            ptx::mbar_init(&kv_full[s], 1);
            ptx::mbar_init(&kv_empty[s], 1);
        }
        for (int s = 0; s < SLOTS; ++s) {
            ptx::mbar_init(&s_full[s], 1);
            ptx::mbar_init(&p_part[s], 4);
            ptx::mbar_init(&p_full[s], 4);
            ptx::mbar_init(&o_done[s], 1);
        }
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
    // slot s: S at columns 256 s, O at 256 s + 128
    if (warp < 4) {
        ptx::setmaxnreg_dec<kRegsControl>();
        if (warp == 0) {
            if (ptx::elect_one()) {
                ptx::mbar_arrive_expect_tx(q_full, nslots * TILE);
                for (int s = 0; s < nslots; ++s) {
                    ptx::tma_load_3d(sQ + s * TILE, &tq, q_full, 0, h0 + s, start + q0);
                    ptx::tma_load_3d(sQ + s * TILE + SUB, &tq, q_full, 64, h0 + s, start + q0);
                }
                const int n_items = 2 * n_kt;
                int i = 0;
                for (; i < n_items; ++i) {
                    const int st = i % KV_ST;
                    if (!ptx::mbar_wait(&kv_empty[st], ((i / KV_ST) & 1) ^ 1, err, 0x3001)) break;
                    const CUtensorMap *map = (i & 1) ? &tv : &tk;
                    ptx::mbar_arrive_expect_tx(&kv_full[st], TILE);
                    if (p.paged) {
                        // 8 pages of 16 keys; a page index past the table (keys past the sequence, masked) reads
                        // page 0, whose values are finite and get weight 0
                        const int32_t *prow = p.pages + (size_t)p.seq_slot[seq] * p.pages_per_seq;
                        int pg[8];
#pragma unroll
                        for (int u = 0; u < 8; ++u) {
                            const int idx = (i >> 1) * 8 + u;
                            pg[u] = idx < p.pages_per_seq ? prow[idx] : 0;
                        }
#pragma unroll
                        for (int u = 0; u < 8; ++u) {
                            const int c2 = (pg[u] * p.kv_heads + kvh) * 2 + (i & 1);
                            ptx::tma_load_3d(sKV + st * TILE + u * 2048, map, &kv_full[st], 0, 0, c2);
                            ptx::tma_load_3d(sKV + st * TILE + SUB + u * 2048, map, &kv_full[st], 64, 0, c2);
                        }
                    } else {
                        const int rows = start + (i >> 1) * TK;
                        ptx::tma_load_3d(sKV + st * TILE, map, &kv_full[st], 0, kvh, rows);
                        ptx::tma_load_3d(sKV + st * TILE + SUB, map, &kv_full[st], 64, kvh, rows);
                    }
                }
                // Our own copies in flight must land before the CTA exits (this matters on the error path).
                ptx::mbar_wait(q_full, 0, err, 0x3002);
                for (int k = i > KV_ST ? i - KV_ST : 0; k < i; ++k)
                    ptx::mbar_wait(&kv_full[k % KV_ST], (k / KV_ST) & 1, err, 0x3002);
            }
        } else if (warp == 1) {
            if (ptx::elect_one()) {
                constexpr uint32_t idesc_qk = ptx::idesc_bf16_f32(128, 128, false);
                constexpr uint32_t idesc_pv = ptx::idesc_bf16_f32(128, 128, true);
                // Ring item i: stage i % KV_ST, phase (i / KV_ST) & 1.
                auto wait_item = [&](int i, uint32_t code) {
                    return ptx::mbar_wait(&kv_full[i % KV_ST], (i / KV_ST) & 1, err, code);
                };
                // S_s = Q_s K_j^T into slot s's S columns, announced on s_full[s]; K_j is released after the last
                // slot's product.
                auto issue_qk = [&](int s, int j) {
                    const uint32_t aQ = ptx::smem_u32(sQ + s * TILE), aK = ptx::smem_u32(sKV + ((2 * j) % KV_ST) * TILE);
#pragma unroll
                    for (int kk = 0; kk < 8; ++kk) {
                        const uint32_t off = (kk >> 2) * SUB + (kk & 3) * 32;
                        ptx::mma_bf16(tmem + 256 * s, ptx::sw128_kmajor_desc(aQ + off),
                                      ptx::sw128_kmajor_desc(aK + off), idesc_qk, kk > 0 ? 1u : 0u);
                    }
                    ptx::mma_commit(&s_full[s]);
                    if (s == nslots - 1) ptx::mma_commit(&kv_empty[(2 * j) % KV_ST]);
                };
                bool ok = ptx::mbar_wait(q_full, 0, err, 0x3003) && wait_item(0, 0x3004);
                if (ok) {
                    ptx::tc_fence_after();
                    for (int s = 0; s < nslots; ++s) issue_qk(s, 0);
                }
                // Per key tile j and slot s: O_s += P_s V_j (keys 0..95 as soon as that part of P is written), then
                // at once S_s of tile j + 1. The tensor core runs the MMAs of one thread in issue order, so S
                // overwrites P_s only after P_s V_j has read it (the softmax may rescale O_s once S_{j+1} is
                // complete for the same reason).
                for (int j = 0; ok && j < n_kt; ++j) {
                    const bool more = j + 1 < n_kt;
                    if (!wait_item(2 * j + 1, 0x3004)) break;
                    const int vst = (2 * j + 1) % KV_ST;
                    const uint32_t aV = ptx::smem_u32(sKV + vst * TILE);
                    for (int s = 0; s < nslots; ++s) {
                        const uint32_t tO = tmem + 256 * s + 128, tP = tmem + 256 * s;
                        if (!ptx::mbar_wait(&p_part[s], j & 1, err, 0x3006)) {
                            ok = false;
                            break;
                        }
                        ptx::tc_fence_after();
#pragma unroll
                        for (int kk = 0; kk < 6; ++kk)
                            ptx::mma_bf16_ts(tO, tP + kk * 8, ptx::sw128_mnmajor_desc(aV + kk * 2048, SUB, 1024),
                                             idesc_pv, (j > 0 || kk > 0) ? 1u : 0u);
                        if (!ptx::mbar_wait(&p_full[s], j & 1, err, 0x3006)) {
                            ok = false;
                            break;
                        }
                        ptx::tc_fence_after();
#pragma unroll
                        for (int kk = 6; kk < 8; ++kk)
                            ptx::mma_bf16_ts(tO, tP + kk * 8, ptx::sw128_mnmajor_desc(aV + kk * 2048, SUB, 1024),
                                             idesc_pv, 1u);
                        if (s == nslots - 1) ptx::mma_commit(&kv_empty[vst]);  // V_j is no longer read
                        if (!more) {
                            ptx::mma_commit(&o_done[s]);
                            continue;
                        }
                        if (s == 0 && !wait_item(2 * j + 2, 0x3005)) {
                            ok = false;
                            break;
                        }
                        ptx::tc_fence_after();
                        issue_qk(s, j + 1);
                    }
                }
                // No MMA may still be writing TMEM when it is freed (this matters on the error path).
                ptx::mma_commit(fin);
                ptx::mbar_wait(fin, 0, err, 0x3009);
            }
        }
    } else {
        ptx::setmaxnreg_inc<kRegsSoftmax>();
        if (warp - 4 < 4 * nslots) {
            const int s = (warp - 4) >> 2;
            const int q = warp & 3;  // TMEM lane quarter this warp may access
            const int rl = q * 32 + lane;
            const int row = q0 + rl;  // query row within the chunk; its position is past + row
            const uint32_t lane_off = (uint32_t)(q * 32) << 16;
            const uint32_t tS = tmem + 256 * s + lane_off, tO = tS + 128;
            const float sc = p.scale_log2;
            float m_ref = -INFINITY, l = 0.f;
            bool ok = true;
            for (int j = 0; j < n_kt; ++j) {
                if (!ptx::mbar_wait(&s_full[s], j & 1, err, 0x3007)) {
                    ok = false;
                    break;
                }
                ptx::tc_fence_after();
                float x[128];
                ptx::tmem_ld32(tS, reinterpret_cast<uint32_t *>(x));
                ptx::tmem_ld32(tS + 32, reinterpret_cast<uint32_t *>(x) + 32);
                ptx::tmem_ld32(tS + 64, reinterpret_cast<uint32_t *>(x) + 64);
                ptx::tmem_ld32(tS + 96, reinterpret_cast<uint32_t *>(x) + 96);
                ptx::tmem_ld_wait();
                const int key0 = j * TK;
                // Masking is needed when some key of the tile lies past the warp's first row or past the sequence.
                const bool need_mask = key0 + TK - 1 > past + q0 + q * 32 || key0 + TK > past + len;
                if (need_mask) {
                    const int lim = min(past + row - key0, past + len - 1 - key0);  // keys 0..lim are visible
#pragma unroll
                    for (int e = 0; e < 128; ++e) x[e] = e <= lim ? x[e] : -INFINITY;
                }
                float mx[8];
#pragma unroll
                for (int u = 0; u < 8; ++u) mx[u] = fmaxf(x[u], x[u + 8]);
#pragma unroll
                for (int e = 16; e < 128; e += 16) {
#pragma unroll
                    for (int u = 0; u < 8; ++u) mx[u] = max3(mx[u], x[e + u], x[e + 8 + u]);
                }
                const float tmax =
                    fmaxf(max3(mx[0], mx[1], mx[2]), max3(mx[3], mx[4], max3(mx[5], mx[6], mx[7]))) * sc;
                bool rescale = false;
                float alpha = 1.f;
                if (j == 0) {
                    m_ref = tmax;
                } else if (tmax > m_ref + kRescaleThreshold) {
                    alpha = ptx::ex2(m_ref - tmax);
                    m_ref = tmax;
                    rescale = true;
                }
                if (__any_sync(0xffffffffu, rescale)) {
                    // S_j has completed, so P V_{j-1} (issued before it) has too: O is quiescent.
                    l *= alpha;
#pragma unroll 1
                    for (int c = 0; c < 128; c += 32) {
                        uint32_t u[32];
                        ptx::tmem_ld32(tO + c, u);
                        ptx::tmem_ld_wait();
#pragma unroll
                        for (int e = 0; e < 32; ++e) u[e] = __float_as_uint(__uint_as_float(u[e]) * alpha);
                        ptx::tmem_st32(tO + c, u);
                    }
                }
                const float nm = -m_ref;
                float la = 0.f, lb = 0.f, lc = 0.f, ld = 0.f;
                uint32_t pk[64];
                if (need_mask) {
#pragma unroll
                    for (int e = 0; e < 64; ++e) {
                        float a, b;
                        fma2(a, b, x[2 * e], x[2 * e + 1], sc, sc, nm, nm);
                        a = ptx::ex2(a);
                        b = ptx::ex2(b);
                        if (e & 1)
                            add2(lc, ld, lc, ld, a, b);
                        else
                            add2(la, lb, la, lb, a, b);
                        pk[e] = pack2(a, b);
                    }
                } else {
                    // the same sums in the same order as the masked form, so a row's result does not depend on
                    // whether its warp's tile needed a mask (chunked prefill equals whole prefill bit for bit)
#pragma unroll
                    for (int e = 0; e < 64; ++e) {
                        float a, b;
                        fma2(a, b, x[2 * e], x[2 * e + 1], sc, sc, nm, nm);
                        a = ptx::ex2(a);
                        b = ptx::ex2(b);
                        if (e & 1)
                            add2(lc, ld, lc, ld, a, b);
                        else
                            add2(la, lb, la, lb, a, b);
                        pk[e] = pack2(a, b);
                    }
                }
                l += (la + lb) + (lc + ld);
                ptx::tmem_st32(tS, pk);
                ptx::tmem_st16(tS + 32, *reinterpret_cast<const uint32_t(*)[16]>(pk + 32));
                ptx::tmem_st_wait();
                ptx::tc_fence_before();
                __syncwarp();
                if (lane == 0) ptx::mbar_arrive(&p_part[s]);
                ptx::tmem_st16(tS + P_SPLIT, *reinterpret_cast<const uint32_t(*)[16]>(pk + P_SPLIT));
                ptx::tmem_st_wait();
                ptx::tc_fence_before();
                __syncwarp();
                if (lane == 0) ptx::mbar_arrive(&p_full[s]);
            }
            if (ok && ptx::mbar_wait(&o_done[s], 0, err, 0x3008)) {
                ptx::tc_fence_after();
                const float inv = 1.f / l;
                __nv_bfloat16 *dst = p.out + ((size_t)(start + row) * p.q_heads + h0 + s) * kHeadDim;
#pragma unroll 1
                for (int c = 0; c < 128; c += 32) {
                    uint32_t u[32];
                    ptx::tmem_ld32(tO + c, u);
                    ptx::tmem_ld_wait();
                    if (row < len) {
                        uint32_t w[16];
#pragma unroll
                        for (int e = 0; e < 16; ++e)
                            w[e] = pack2(__uint_as_float(u[2 * e]) * inv, __uint_as_float(u[2 * e + 1]) * inv);
                        uint4 *d4 = reinterpret_cast<uint4 *>(dst + c);
#pragma unroll
                        for (int e = 0; e < 4; ++e) d4[e] = make_uint4(w[4 * e], w[4 * e + 1], w[4 * e + 2], w[4 * e + 3]);
                    }
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
    // resolved once per process (a function-local static: thread-safe initialisation)
    static const EncodeTiledFn fn = [] {
        void *ptr = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            return (EncodeTiledFn)ptr;
        return (EncodeTiledFn) nullptr;
    }();
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

// The paged KV pool [pages][kv_heads][2][16][128] bf16 as [pages * kv_heads * 2][16 tokens][128]: boxes of 64 dims x
// 16 tokens (one page of one head, K or V), 128-byte swizzle.
bool make_tmap_pool(CUtensorMap *map, const void *pool, int kv_heads, int pages) {
    EncodeTiledFn enc = encode_tiled_fn();
    if (!enc) return false;
    cuuint64_t dims[3] = {128, 16, (cuuint64_t)pages * kv_heads * 2};
    cuuint64_t strides[2] = {256, 16 * 256};
    cuuint32_t box[3] = {64, 16, 1};
    cuuint32_t estr[3] = {1, 1, 1};
    return enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void *>(pool), dims, strides, box, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace

cudaError_t launch_prefill_attention_tc(const PrefillAttnArgs &a, int total_tokens, uint32_t *err, cudaStream_t st) {
    CUtensorMap tq, tk, tv;
    if (!make_tmap_heads(&tq, a.q, a.q_heads, total_tokens)) return cudaErrorInvalidValue;
    if (a.pool) {
        if (!a.pages || !a.seq_slot || !a.past || a.pages_per_seq < 1 || a.kv_pages < 1 ||
            !make_tmap_pool(&tk, a.pool, a.kv_heads, a.kv_pages))
            return cudaErrorInvalidValue;
        tv = tk;
    } else if (!make_tmap_heads(&tk, a.k, a.kv_heads, total_tokens) ||
               !make_tmap_heads(&tv, a.v, a.kv_heads, total_tokens)) {
        return cudaErrorInvalidValue;
    }
    static SmemOptIn opt;
    if (cudaError_t e = opt.set((const void *)flash_tc_kernel, SMEM_BYTES)) return e;
    FlashTcParams p;
    p.cu_seqlens = a.cu_seqlens;
    p.out = a.out;
    p.nseq = a.nseq;
    p.max_len = a.max_len;
    p.q_heads = a.q_heads;
    p.kv_heads = a.kv_heads;
    p.heads_per_cta = ((a.q_heads / a.kv_heads) % 2 == 0) ? 2 : 1;
    p.scale_log2 = a.scale_log2;
    p.err = err;
    p.paged = a.pool != nullptr;
    p.pages = a.pages;
    p.seq_slot = a.seq_slot;
    p.past = a.past;
    p.pages_per_seq = a.pages_per_seq;
    p.total_tokens = total_tokens;
    dim3 grid(a.q_heads / p.heads_per_cta, a.nseq, (a.max_len + TQ - 1) / TQ);
    return launch_kernel(flash_tc_kernel, grid, dim3(kThreads), SMEM_BYTES, st, tq, tk, tv, p);
}

}  // namespace lrm
