// flash_prefill.cu -- causal GQA prefill attention (bf16 in, fp32 softmax/accumulation, bf16 out).
//
// The reference's attention_gqa_causal (src/Lrm.Shaders/hlsl/kernels/attention/attention_gqa_causal.hlsl) runs one
// 64-thread group per (query row, head) with scalar fp32 math. Here one CTA of 4 warps owns 64 query rows of one
// head: Q stays in registers as mma fragments, 64-key K/V tiles are double buffered in shared memory with cp.async
// (16-byte chunks, XOR-swizzled so ldmatrix is conflict-free), S = Q K^T and O += P V run on the tensor cores
// (mma.sync m16n8k16 bf16 -> fp32), and the softmax is online in registers (log2 domain, running max per row,
// causal mask only on the diagonal tile). Sequences are packed back to back (cu_seqlens); each starts at position 0.
#include <cuda_bf16.h>
#include <math.h>
#include <stdint.h>

#include "internal.h"
#include "qwen.h"

namespace lrm {
namespace {

constexpr int BQ = 64, BKV = 64, D = kHeadDim, NWARP = 4;

__device__ __forceinline__ uint32_t smem_u32(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }

// Byte offset of 16-byte chunk c of row r in a [rows][128] bf16 tile (256-byte rows), XOR-swizzled by row.
__device__ __forceinline__ uint32_t swz(int r, int c) { return r * 256 + ((c ^ (r & 7)) << 4); }

__device__ __forceinline__ void cp_async16(uint32_t dst, const void *src, bool valid) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(valid ? 16 : 0));
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;"); }
template <int N>
__device__ __forceinline__ void cp_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N));
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t &r0, uint32_t &r1, uint32_t &r2, uint32_t &r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t &r0, uint32_t &r1, uint32_t &r2, uint32_t &r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}

__device__ __forceinline__ void mma16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%0, %1, %2, %3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t pack_bf16(float a, float b) {
    __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t *>(&h);
}

// Loads rows [row0, row0 + 64) of head `head` from a [T][heads][128] tensor into a swizzled tile (rows past `rows`
// are zero-filled).
__device__ __forceinline__ void load_tile(uint32_t tile, const __nv_bfloat16 *base, int heads, int head, int row0,
                                          int rows) {
    for (int i = threadIdx.x; i < 64 * 16; i += NWARP * 32) {
        const int r = i >> 4, c = i & 15;
        const bool ok = row0 + r < rows;
        const __nv_bfloat16 *src = base + ((size_t)(ok ? row0 + r : 0) * heads + head) * D + c * 8;
        cp_async16(tile + swz(r, c), src, ok);
    }
}

__global__ void __launch_bounds__(NWARP * 32) flash_prefill_kernel(PrefillAttnArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    const uint32_t sQ = smem_u32(smem);
    const uint32_t sK = sQ + BQ * 256;          // 2 buffers
    const uint32_t sV = sK + 2 * BKV * 256;     // 2 buffers

    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    const int seq = blockIdx.z, h = blockIdx.y;
    const int start = a.cu_seqlens[seq];
    const int len = a.cu_seqlens[seq + 1] - start;
    const int q0 = blockIdx.x * BQ;
    if (q0 >= len) return;
    const int kvh = h / (a.q_heads / a.kv_heads);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = lane >> 2, t4 = lane & 3;

    const __nv_bfloat16 *qb = a.q + (size_t)start * a.q_heads * D;
    const __nv_bfloat16 *kb = a.k + (size_t)start * a.kv_heads * D;
    const __nv_bfloat16 *vb = a.v + (size_t)start * a.kv_heads * D;

    const int last_key = min(len, q0 + BQ) - 1;
    const int n_kt = last_key / BKV + 1;

    load_tile(sQ, qb, a.q_heads, h, q0, len);
    load_tile(sK, kb, a.kv_heads, kvh, 0, len);
    load_tile(sV, vb, a.kv_heads, kvh, 0, len);
    cp_commit();

    uint32_t qf[8][4];  // A fragments of this warp's 16 rows, k steps of 16 dims
    float o[16][4];
#pragma unroll
    for (int j = 0; j < 16; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
    float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
    const int qrow0 = q0 + warp * 16 + g;  // rows qrow0 and qrow0 + 8 of the sequence

    for (int kt = 0; kt < n_kt; ++kt) {
        const int buf = kt & 1;
        if (kt + 1 < n_kt) {
            load_tile(sK + (buf ^ 1) * BKV * 256, kb, a.kv_heads, kvh, (kt + 1) * BKV, len);
            load_tile(sV + (buf ^ 1) * BKV * 256, vb, a.kv_heads, kvh, (kt + 1) * BKV, len);
        }
        cp_commit();
        cp_wait<1>();
        __syncthreads();
        if (kt == 0) {
#pragma unroll
            for (int kk = 0; kk < 8; ++kk) {
                const int r = warp * 16 + (lane & 15), c = 2 * kk + (lane >> 4);
                ldsm_x4(sQ + swz(r, c), qf[kk][0], qf[kk][1], qf[kk][2], qf[kk][3]);
            }
        }
        const uint32_t tK = sK + buf * BKV * 256, tV = sV + buf * BKV * 256;
        float s[8][4];
#pragma unroll
        for (int j = 0; j < 8; ++j) s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.f;
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
#pragma unroll
            for (int jp = 0; jp < 4; ++jp) {
                // matrices: keys 16jp..+7 dims 16kk..+7 | same keys dims +8 | keys +8 dims 16kk | keys +8 dims +8
                const int key = 16 * jp + (lane & 7) + ((lane >> 4) << 3);
                const int c = 2 * kk + ((lane >> 3) & 1);
                uint32_t b0, b1, b2, b3;
                ldsm_x4(tK + swz(key, c), b0, b1, b2, b3);
                mma16816(s[2 * jp], qf[kk], b0, b1);
                mma16816(s[2 * jp + 1], qf[kk], b2, b3);
            }
        }
        // scale, mask (diagonal tile and sequence end), online softmax
        const bool diag = (kt + 1) * BKV > q0 + warp * 16;
        float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int key = kt * BKV + 8 * j + 2 * t4 + (e & 1);
                const int qr = qrow0 + (e >> 1) * 8;
                float v = s[j][e] * a.scale_log2;
                if (diag && (key > qr || key >= len)) v = -INFINITY;
                s[j][e] = v;
            }
            mx0 = fmaxf(mx0, fmaxf(s[j][0], s[j][1]));
            mx1 = fmaxf(mx1, fmaxf(s[j][2], s[j][3]));
        }
        mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffff, mx0, 1));
        mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffff, mx0, 2));
        mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffff, mx1, 1));
        mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffff, mx1, 2));
        const float mn0 = fmaxf(m0, mx0), mn1 = fmaxf(m1, mx1);
        const float al0 = exp2f(m0 - mn0), al1 = exp2f(m1 - mn1);
        m0 = mn0;
        m1 = mn1;
        float rs0 = 0.f, rs1 = 0.f;
        uint32_t pf[8][2];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const float p0 = exp2f(s[j][0] - mn0), p1 = exp2f(s[j][1] - mn0);
            const float p2 = exp2f(s[j][2] - mn1), p3 = exp2f(s[j][3] - mn1);
            rs0 += p0 + p1;
            rs1 += p2 + p3;
            pf[j][0] = pack_bf16(p0, p1);
            pf[j][1] = pack_bf16(p2, p3);
        }
        l0 = l0 * al0 + rs0;
        l1 = l1 * al1 + rs1;
#pragma unroll
        for (int j = 0; j < 16; ++j) {
            o[j][0] *= al0;
            o[j][1] *= al0;
            o[j][2] *= al1;
            o[j][3] *= al1;
        }
        // O += P V: k steps of 16 keys; P fragments come straight from the S accumulators.
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
            const uint32_t pa[4] = {pf[2 * kk][0], pf[2 * kk][1], pf[2 * kk + 1][0], pf[2 * kk + 1][1]};
#pragma unroll
            for (int np = 0; np < 8; ++np) {
                // trans matrices: keys 16kk..+7 dims 16np..+7 | keys +8 same dims | keys 16kk dims +8 | keys +8 dims +8
                const int key = 16 * kk + (lane & 7) + (((lane >> 3) & 1) << 3);
                const int c = 2 * np + (lane >> 4);
                uint32_t b0, b1, b2, b3;
                ldsm_x4_t(tV + swz(key, c), b0, b1, b2, b3);
                mma16816(o[2 * np], pa, b0, b1);
                mma16816(o[2 * np + 1], pa, b2, b3);
            }
        }
        __syncthreads();
    }
    l0 += __shfl_xor_sync(0xffffffff, l0, 1);
    l0 += __shfl_xor_sync(0xffffffff, l0, 2);
    l1 += __shfl_xor_sync(0xffffffff, l1, 1);
    l1 += __shfl_xor_sync(0xffffffff, l1, 2);
    const float inv0 = 1.f / l0, inv1 = 1.f / l1;
#pragma unroll
    for (int j = 0; j < 16; ++j) {
        const int d = 8 * j + 2 * t4;
        if (qrow0 < len)
            *reinterpret_cast<uint32_t *>(a.out + ((size_t)(start + qrow0) * a.q_heads + h) * D + d) =
                pack_bf16(o[j][0] * inv0, o[j][1] * inv0);
        if (qrow0 + 8 < len)
            *reinterpret_cast<uint32_t *>(a.out + ((size_t)(start + qrow0 + 8) * a.q_heads + h) * D + d) =
                pack_bf16(o[j][2] * inv1, o[j][3] * inv1);
    }
}

}  // namespace

cudaError_t launch_prefill_attention(const PrefillAttnArgs &a, cudaStream_t st) {
    const int smem = (BQ + 4 * BKV) * 256;
    static bool configured[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (!configured[dev & 63]) {
        cudaError_t e = cudaFuncSetAttribute(flash_prefill_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        if (e != cudaSuccess) return e;
        configured[dev & 63] = true;
    }
    dim3 grid((a.max_len + BQ - 1) / BQ, a.q_heads, a.nseq);
    return launch_kernel(flash_prefill_kernel, grid, dim3(NWARP * 32), smem, st, a);
}

}  // namespace lrm
