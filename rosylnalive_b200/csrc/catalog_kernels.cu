// catalog_kernels.cu -- the 14 catalog kernels (docs/contracts/kernel-abi.md, "The catalog at contracts-v1") for
// sm_100a, with fp32 activations as the catalog defines them. They are the conformance surface of the CUDA device and
// the fp32 path of the forward pass; the bf16 fast path (qwen_*.cu) uses its own fused kernels.
//
// Arithmetic follows the CPU reference's definitions (src/Lrm.Tensor.CpuReference/Rows.fs): products and sums in
// element-wise formulas are rounded one by one (__fmul_rn / __fadd_rn keep nvcc from contracting them), and every
// reduction has an order that depends only on its length, never on the batch (docs/contracts/batch-invariance.md):
//   - matmul_bf16w: y[i,j] = sum over p = 0..k-1 of fmaf(x[i,p], widen(w[j,p]), .) sequentially from +0, so each
//     output is bit-identical to CpuRef F32's Rows.dotBf16 (Rows.fs:38-46), whatever m, n and the tile are;
//   - rmsnorm_rows: per-thread sequential partials over columns t, t+256, ..., then a fixed 256-way tree;
//   - attention_gqa_causal: 64-key blocks anchored at position 0 with an online softmax updated once per block.
#include <math.h>
#include <string.h>

#include "internal.h"

namespace lrm {
namespace {

__device__ __forceinline__ float widen(uint16_t b) { return __uint_as_float(((uint32_t)b) << 16); }

__device__ __forceinline__ size_t grid_stride_start() { return (size_t)blockIdx.x * blockDim.x + threadIdx.x; }
__device__ __forceinline__ size_t grid_stride() { return (size_t)gridDim.x * blockDim.x; }

float host_f32(uint32_t b) {
    float f;
    memcpy(&f, &b, 4);
    return f;
}

unsigned elementwise_blocks(size_t n) {
    size_t b = (n + 255) / 256;
    const size_t cap = 148 * 64;  // a few waves of the 148 SMs; the loops stride over the rest
    return (unsigned)(b < 1 ? 1 : (b > cap ? cap : b));
}

// 0 scale_f32: y[i] = a * x[i].
__global__ void k_scale_f32(const float *x, float *y, uint32_t n, float a) {
    for (size_t i = grid_stride_start(); i < n; i += grid_stride()) y[i] = __fmul_rn(a, x[i]);
}

// 1 table_echo: the 16 words of row `src` of the table.
__global__ void k_table_echo(const uint32_t *table, uint32_t src, uint32_t *y) {
    if (threadIdx.x < 16) y[threadIdx.x] = table[(size_t)src * 16 + threadIdx.x];
}

// 2 args_echo: all 32 words, lrm_groups_x included.
struct Words {
    uint32_t w[32];
};
__global__ void k_args_echo(Words words, uint32_t *y) {
    if (threadIdx.x < 32) y[threadIdx.x] = words.w[threadIdx.x];
}

// 3 groups_echo: logical group g writes g.
__global__ void k_groups_echo(uint32_t *y, uint32_t groups) {
    for (size_t g = grid_stride_start(); g < groups; g += grid_stride()) y[g] = (uint32_t)g;
}

// 4 bf16_unpack.
__global__ void k_bf16_unpack(const uint16_t *x, float *y, uint32_t n) {
    for (size_t i = grid_stride_start(); i < n; i += grid_stride()) y[i] = widen(x[i]);
}

// 5 embed_gather_bf16: an id at or above vocab gives the quiet-NaN row 0x7FC00000 (CpuRef.fs:74-109).
__global__ void k_embed_gather(const uint32_t *ids, const uint16_t *table, float *y, uint32_t rows, uint32_t cols,
                               uint32_t vocab) {
    size_t total = (size_t)rows * cols;
    for (size_t e = grid_stride_start(); e < total; e += grid_stride()) {
        size_t r = e / cols, c = e % cols;
        uint32_t id = ids[r];
        y[e] = id < vocab ? widen(table[(size_t)id * cols + c]) : __uint_as_float(0x7FC00000u);
    }
}

// 6 rmsnorm_rows: one 256-thread block per row (Rows.rmsNorm, Rows.fs:50-71, in a length-only order).
__global__ void __launch_bounds__(256) k_rmsnorm_rows(const float *x, const uint16_t *w, float *y, uint32_t rows,
                                                      uint32_t cols, float eps) {
    __shared__ float part[256];
    size_t row = blockIdx.x;
    if (row >= rows) return;
    const float *xr = x + row * cols;
    float *yr = y + row * cols;
    unsigned t = threadIdx.x;
    float s = 0.0f;
    for (unsigned c = t; c < cols; c += 256) s = fmaf(xr[c], xr[c], s);
    part[t] = s;
    __syncthreads();
    for (unsigned h = 128; h > 0; h >>= 1) {
        if (t < h) part[t] = __fadd_rn(part[t], part[t + h]);
        __syncthreads();
    }
    float mean = __fdiv_rn(part[0], (float)cols);
    float r = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, eps)));
    for (unsigned c = t; c < cols; c += 256) yr[c] = __fmul_rn(widen(w[c]), __fmul_rn(xr[c], r));
}

// 7 rope_apply: row r (of tokens * heads) has position pos0 + r / heads (Rows.ropeHead, Rows.fs:205-227).
__global__ void k_rope_apply(const float *x, const float *cos_t, const float *sin_t, float *y, uint32_t rows,
                             uint32_t heads, uint32_t head_dim, uint32_t pos0) {
    uint32_t half = head_dim / 2;
    size_t total = (size_t)rows * half;
    for (size_t e = grid_stride_start(); e < total; e += grid_stride()) {
        size_t r = e / half, i = e % half;
        size_t pos = pos0 + r / heads;
        float c = cos_t[pos * half + i], s = sin_t[pos * half + i];
        const float *xr = x + r * head_dim;
        float a = xr[i], b = xr[i + half];
        float ya = __fsub_rn(__fmul_rn(a, c), __fmul_rn(b, s));
        float yb = __fadd_rn(__fmul_rn(b, c), __fmul_rn(a, s));
        y[r * head_dim + i] = ya;
        y[r * head_dim + i + half] = yb;
    }
}

// 8 silu_mul: y = (g / (1 + exp(-g))) * u (Rows.siluMul, Rows.fs:185-192); expf is CUDA's accurate expf.
__global__ void k_silu_mul(const float *g, const float *u, float *y, uint32_t n) {
    for (size_t i = grid_stride_start(); i < n; i += grid_stride()) {
        float gi = g[i];
        float s = __fdiv_rn(gi, __fadd_rn(1.0f, expf(-gi)));
        y[i] = __fmul_rn(s, u[i]);
    }
}

// 9 add.
__global__ void k_add(const float *a, const float *b, float *y, uint32_t n) {
    for (size_t i = grid_stride_start(); i < n; i += grid_stride()) y[i] = __fadd_rn(a[i], b[i]);
}

// 10 copy_rows: 4-byte elements.
__global__ void k_copy_rows(const uint32_t *src, uint32_t *dst, uint32_t rows, uint32_t cols, uint32_t src_row0,
                            uint32_t dst_row0, uint32_t src_stride, uint32_t dst_stride) {
    size_t total = (size_t)rows * cols;
    for (size_t e = grid_stride_start(); e < total; e += grid_stride()) {
        size_t r = e / cols, c = e % cols;
        dst[(dst_row0 + r) * (size_t)dst_stride + c] = src[(src_row0 + r) * (size_t)src_stride + c];
    }
}

// 11 argmax_rows: lowest index of the maximum by '>' (+0 and -0 tie), 0xFFFFFFFF for a row holding a NaN
// (Rows.tryArgmax, Rows.fs:138-154). The result is order independent, so a 256-way tree is exact.
__global__ void __launch_bounds__(256) k_argmax_rows(const float *x, uint32_t *y, uint32_t rows, uint32_t cols) {
    __shared__ float bv[256];
    __shared__ int64_t bi[256];
    __shared__ int anynan;
    size_t row = blockIdx.x;
    if (row >= rows) return;
    const float *xr = x + row * cols;
    unsigned t = threadIdx.x;
    if (t == 0) anynan = 0;
    __syncthreads();
    float best = 0.0f;
    int64_t idx = -1;
    int nan = 0;
    for (unsigned c = t; c < cols; c += 256) {
        float v = xr[c];
        if (isnan(v))
            nan = 1;
        else if (idx < 0 || v > best) {
            best = v;
            idx = c;
        }
    }
    if (nan) atomicOr(&anynan, 1);
    bv[t] = best;
    bi[t] = idx;
    __syncthreads();
    for (unsigned h = 128; h > 0; h >>= 1) {
        if (t < h) {
            float v2 = bv[t + h];
            int64_t i2 = bi[t + h];
            if (i2 >= 0 && (bi[t] < 0 || v2 > bv[t] || (v2 == bv[t] && i2 < bi[t]))) {
                bv[t] = v2;
                bi[t] = i2;
            }
        }
        __syncthreads();
    }
    if (t == 0) y[row] = anynan ? 0xFFFFFFFFu : (uint32_t)bi[0];
}

// 12 matmul_bf16w: 64x64 output tile per block, 256 threads with 4x4 outputs each, k staged 32 at a time. Each output
// accumulates p = 0..k-1 in increasing order with one fmaf per step from +0 (Rows.dotBf16).
__global__ void __launch_bounds__(256) k_matmul_bf16w(const float *x, const uint16_t *w, float *y, uint32_t m,
                                                      uint32_t n, uint32_t k) {
    __shared__ float xs[64][33];
    __shared__ float ws[64][33];
    const unsigned tx = threadIdx.x % 16, ty = threadIdx.x / 16;
    const size_t row0 = (size_t)blockIdx.y * 64, col0 = (size_t)blockIdx.x * 64;
    float acc[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = 0.0f;
    for (uint32_t p0 = 0; p0 < k; p0 += 32) {
        for (unsigned e = threadIdx.x; e < 64 * 32; e += 256) {
            unsigned r = e / 32, p = e % 32;
            size_t gr = row0 + r, gp = (size_t)p0 + p;
            xs[r][p] = (gr < m && gp < k) ? x[gr * k + gp] : 0.0f;
            size_t gc = col0 + r;
            ws[r][p] = (gc < n && gp < k) ? widen(w[gc * k + gp]) : 0.0f;
        }
        __syncthreads();
        unsigned pmax = (k - p0) < 32 ? (k - p0) : 32;
        for (unsigned p = 0; p < pmax; ++p) {
            float a[4], b[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) a[i] = xs[ty + 16 * i][p];
#pragma unroll
            for (int j = 0; j < 4; ++j) b[j] = ws[tx + 16 * j][p];
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
        }
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        size_t r = row0 + ty + 16 * i;
        if (r >= m) continue;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            size_t c = col0 + tx + 16 * j;
            if (c < n) y[r * n + c] = acc[i][j];
        }
    }
}

// 13 attention_gqa_causal: one 64-thread block per (query row, q head). Keys in blocks of 64 anchored at position 0;
// thread t scores key 64b + t with a sequential fmaf dot in increasing d, times scale; the running maximum starts at
// block 0's maximum; weights e_j = exp(s_j - m'); per block, the weight sum and the weighted values are sequential in j
// from +0, and the state is updated once per block: l = fma(l, alpha, sum), o = fma(o, alpha, value); y = o / l.
// Output dimensions are handled 256 per pass (thread t owns d0 + t + 64 r), recomputing the scores per pass.
__global__ void __launch_bounds__(64) k_attention(const float *q, const float *kc, const float *vc, float *y,
                                                  uint32_t rows, uint32_t q_row0, uint32_t past, uint32_t q_heads,
                                                  uint32_t kv_heads, uint32_t head_dim, float scale) {
    extern __shared__ float smem[];
    float *qs = smem;                 // head_dim
    float *scores = smem + head_dim;  // 64
    float *weights = scores + 64;     // 64
    const uint32_t i = rows - 1 - blockIdx.x;
    const uint32_t h = blockIdx.y;
    const unsigned t = threadIdx.x;
    const uint32_t kvh = h / (q_heads / kv_heads);
    const size_t keys = (size_t)past + i + 1;
    const size_t kv_stride = (size_t)kv_heads * head_dim, kv_off = (size_t)kvh * head_dim;
    const size_t q_base = ((size_t)(q_row0 + i) * q_heads + h) * head_dim;
    for (unsigned d = t; d < head_dim; d += 64) qs[d] = q[q_base + d];
    __syncthreads();
    for (uint32_t d0 = 0; d0 < head_dim; d0 += 256) {
        float m = 0.0f, l = 0.0f, o[4] = {0.0f, 0.0f, 0.0f, 0.0f};
        for (size_t j0 = 0; j0 < keys; j0 += 64) {
            unsigned count = (keys - j0) < 64 ? (unsigned)(keys - j0) : 64u;
            float s = 0.0f;
            if (t < count) {
                const float *kr = kc + (j0 + t) * kv_stride + kv_off;
                float acc = 0.0f;
                for (uint32_t d = 0; d < head_dim; ++d) acc = fmaf(qs[d], kr[d], acc);
                s = __fmul_rn(acc, scale);
            }
            scores[t] = s;
            __syncthreads();
            float block_max = scores[0];
            for (unsigned jm = 1; jm < count; ++jm) block_max = fmaxf(block_max, scores[jm]);
            if (j0 == 0) m = block_max;
            float m_new = fmaxf(m, block_max);
            float alpha = expf(__fsub_rn(m, m_new));
            m = m_new;
            weights[t] = t < count ? expf(__fsub_rn(s, m_new)) : 0.0f;
            __syncthreads();
            float block_sum = 0.0f, acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
            for (unsigned j = 0; j < count; ++j) {
                float e = weights[j];
                block_sum = __fadd_rn(block_sum, e);
                const float *vr = vc + (j0 + j) * kv_stride + kv_off + d0;
#pragma unroll
                for (int r = 0; r < 4; ++r) {
                    uint32_t d = t + 64 * r;
                    if (d0 + d < head_dim) acc[r] = fmaf(e, vr[d], acc[r]);
                }
            }
            l = fmaf(l, alpha, block_sum);
#pragma unroll
            for (int r = 0; r < 4; ++r) o[r] = fmaf(o[r], alpha, acc[r]);
            __syncthreads();
        }
#pragma unroll
        for (int r = 0; r < 4; ++r) {
            uint32_t d = d0 + t + 64 * r;
            if (d < head_dim) y[q_base + d] = __fdiv_rn(o[r], l);
        }
    }
}

}  // namespace

bool catalog_kernel_present(uint32_t kernel) { return kernel < LRM_CATALOG_KERNELS; }

cudaError_t launch_catalog(const CatalogLaunch &L, cudaStream_t st) {
    const uint32_t *w = L.w;
    void *const *p = L.ptr;
    switch (L.kernel) {
        case 0:
            k_scale_f32<<<elementwise_blocks(w[3]), 256, 0, st>>>((const float *)p[1], (float *)p[2], w[3],
                                                                  host_f32(w[4]));
            break;
        case 1:
            k_table_echo<<<1, 32, 0, st>>>(L.table, w[1], (uint32_t *)p[2]);
            break;
        case 2: {
            Words words;
            for (int i = 0; i < 32; ++i) words.w[i] = w[i];
            k_args_echo<<<1, 32, 0, st>>>(words, (uint32_t *)p[1]);
            break;
        }
        case 3:
            k_groups_echo<<<elementwise_blocks(w[2]), 256, 0, st>>>((uint32_t *)p[1], w[2]);
            break;
        case 4:
            k_bf16_unpack<<<elementwise_blocks(w[3]), 256, 0, st>>>((const uint16_t *)p[1], (float *)p[2], w[3]);
            break;
        case 5:
            k_embed_gather<<<elementwise_blocks((size_t)w[4] * w[5]), 256, 0, st>>>(
                (const uint32_t *)p[1], (const uint16_t *)p[2], (float *)p[3], w[4], w[5], w[6]);
            break;
        case 6:
            k_rmsnorm_rows<<<w[4], 256, 0, st>>>((const float *)p[1], (const uint16_t *)p[2], (float *)p[3], w[4],
                                                 w[5], host_f32(w[6]));
            break;
        case 7:
            k_rope_apply<<<elementwise_blocks((size_t)w[5] * (w[7] / 2)), 256, 0, st>>>(
                (const float *)p[1], (const float *)p[2], (const float *)p[3], (float *)p[4], w[5], w[6], w[7], w[8]);
            break;
        case 8:
            k_silu_mul<<<elementwise_blocks(w[4]), 256, 0, st>>>((const float *)p[1], (const float *)p[2],
                                                                 (float *)p[3], w[4]);
            break;
        case 9:
            k_add<<<elementwise_blocks(w[4]), 256, 0, st>>>((const float *)p[1], (const float *)p[2], (float *)p[3],
                                                            w[4]);
            break;
        case 10:
            k_copy_rows<<<elementwise_blocks((size_t)w[3] * w[4]), 256, 0, st>>>(
                (const uint32_t *)p[1], (uint32_t *)p[2], w[3], w[4], w[5], w[6], w[7], w[8]);
            break;
        case 11:
            k_argmax_rows<<<w[3], 256, 0, st>>>((const float *)p[1], (uint32_t *)p[2], w[3], w[4]);
            break;
        case 12: {
            dim3 grid((w[5] + 63) / 64, (w[4] + 63) / 64);
            k_matmul_bf16w<<<grid, 256, 0, st>>>((const float *)p[1], (const uint16_t *)p[2], (float *)p[3], w[4],
                                                 w[5], w[6]);
            break;
        }
        case 13: {
            dim3 grid(w[5], w[8]);
            size_t smem = sizeof(float) * ((size_t)w[10] + 128);
            if (smem > 48 * 1024) {
                cudaError_t e = cudaFuncSetAttribute(k_attention, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                     (int)smem);
                if (e != cudaSuccess) return e;
            }
            k_attention<<<grid, 64, smem, st>>>((const float *)p[1], (const float *)p[2], (const float *)p[3],
                                                (float *)p[4], w[5], w[6], w[7], w[8], w[9], w[10],
                                                host_f32(w[11]));
            break;
        }
        default:
            return cudaErrorInvalidValue;
    }
    return cudaGetLastError();
}

}  // namespace lrm
