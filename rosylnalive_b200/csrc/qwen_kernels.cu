// qwen_kernels.cu -- the bf16 forward path's fused element-wise/row kernels and the paged split-K decode attention.
//
// The reference computes these as separate catalog dispatches (embed_gather_bf16, rmsnorm_rows, rope_apply,
// copy_rows, silu_mul, add, argmax_rows: src/Lrm.Shaders/hlsl/kernels/basic/*.hlsl). Here each neighbourhood is one
// kernel so an activation makes one trip through HBM:
//   norm_rows_block   RMSNorm of chosen rows before the lm_head (a block a row)
//   argmax, advance
// and decode attention streams the paged bf16 KV cache with bulk async copies (see decode_attn_kernel). The embedding
// gather, the layers' RMSNorms, residual adds, QK-norm/RoPE/KV append and SwiGLU run inside the GEMMs and their prep
// kernels (gemm_tcgen05.cu for prefill, gemm_decode.cu for decode).
#include <cuda_bf16.h>
#include <math.h>
#include <stdint.h>

#include "internal.h"
#include "ptx.cuh"
#include "qwen.h"

namespace lrm {
namespace {

constexpr unsigned FULL = 0xFFFFFFFFu;

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(FULL, v, o);
    return v;
}

// Sum over the 256 threads of a block; `red` holds 8 floats.
__device__ __forceinline__ float block_sum256(float v, float *red) {
    v = warp_sum(v);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
    __syncthreads();
    float t = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) t += red[i];
    __syncthreads();
    return t;
}

__device__ __forceinline__ float bf(const __nv_bfloat16 v) { return __bfloat162float(v); }

__device__ __forceinline__ uint2 pack4(float a, float b, float c, float d) {
    __nv_bfloat162 lo = __floats2bfloat162_rn(a, b), hi = __floats2bfloat162_rn(c, d);
    return make_uint2(*reinterpret_cast<uint32_t *>(&lo), *reinterpret_cast<uint32_t *>(&hi));
}

// ---- RMSNorm rows ----------------------------------------------------------------------------------------------

// One block per row, 4 consecutive columns per thread (hidden % 4 == 0): xn[t] = bf16(rmsnorm(x[row]) * w) with row
// idx[t] (t without idx): the final norm before the lm_head, of the decode step's rows or a prefill's last rows.
__global__ void __launch_bounds__(256) norm_rows_block_kernel(const float *x, const int32_t *idx, int hidden,
                                                              const __nv_bfloat16 *w, float eps, __nv_bfloat16 *xn) {
    ptx::griddep_wait();
    ptx::griddep_launch();
    __shared__ float red[8];
    const int t = blockIdx.x;
    const float4 *xr = reinterpret_cast<const float4 *>(x + (size_t)(idx ? idx[t] : t) * hidden);
    const int n4 = hidden / 4;
    float ss = 0.f;
    for (int c = threadIdx.x; c < n4; c += 256) {
        const float4 v = xr[c];
        ss += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
    }
    const float r = rsqrtf(block_sum256(ss, red) / hidden + eps);
    for (int c = threadIdx.x; c < n4; c += 256) {
        const float4 v = xr[c];
        const uint2 wv = *reinterpret_cast<const uint2 *>(w + 4 * c);
        *reinterpret_cast<uint2 *>(xn + (size_t)t * hidden + 4 * c) =
            pack4(v.x * r * __uint_as_float(wv.x << 16), v.y * r * __uint_as_float(wv.x & 0xFFFF0000u),
                  v.z * r * __uint_as_float(wv.y << 16), v.w * r * __uint_as_float(wv.y & 0xFFFF0000u));
    }
}

// ---- argmax -------------------------------------------------------------------------------------------------
//
// One row a cluster of kArgmaxCtas CTAs: CTA r scans the r-th contiguous part of the row (the larger value, then the
// lower index; NaN noted), and rank 0 merges the parts over distributed shared memory. The result does not depend on
// the split: the lowest index of the maximum, or 0xFFFFFFFF for a row that holds a NaN.
constexpr int kArgmaxCtas = 8;

__device__ __forceinline__ void arg_merge(float &best, int &idx, float v2, int i2) {
    if (i2 >= 0 && (idx < 0 || v2 > best || (v2 == best && i2 < idx))) {
        best = v2;
        idx = i2;
    }
}

__global__ void __launch_bounds__(256) argmax_kernel(const float *logits, int V, uint32_t *out) {
    ptx::griddep_wait();
    ptx::griddep_launch();
    __shared__ float sv[8];
    __shared__ int si[8];
    __shared__ int nan_any;
    __shared__ __align__(16) float part[4];  // this CTA's (value, index, NaN seen) for rank 0
    const int rank = blockIdx.x;             // the cluster rank: clusters of kArgmaxCtas along x
    const float *row = logits + (size_t)blockIdx.y * V;
    // A multiple of 4 columns a CTA, so that with V a multiple of 4 every row and chunk starts 16-byte aligned and the
    // scan reads float4s (each thread's elements in increasing index order, as the scalar scan).
    const int chunk = ((V + kArgmaxCtas - 1) / kArgmaxCtas + 3) & ~3;
    const int c0 = min(V, rank * chunk), c1 = min(V, c0 + chunk);
    if (threadIdx.x == 0) nan_any = 0;
    __syncthreads();
    float best = -INFINITY;
    int idx = -1;
    bool nan = false;
    auto take = [&](float v, int c) {
        if (isnan(v))
            nan = true;
        else if (idx < 0 || v > best) {
            best = v;
            idx = c;
        }
    };
    if ((V & 3) == 0) {
#pragma unroll 4
        for (int c = c0 + 4 * (int)threadIdx.x; c < c1; c += 1024) {
            const float4 v = *reinterpret_cast<const float4 *>(row + c);
            take(v.x, c);
            take(v.y, c + 1);
            take(v.z, c + 2);
            take(v.w, c + 3);
        }
    } else {
#pragma unroll 4
        for (int c = c0 + threadIdx.x; c < c1; c += 256) take(row[c], c);
    }
    if (nan) nan_any = 1;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) arg_merge(best, idx, __shfl_xor_sync(FULL, best, o), __shfl_xor_sync(FULL, idx, o));
    if ((threadIdx.x & 31) == 0) {
        sv[threadIdx.x >> 5] = best;
        si[threadIdx.x >> 5] = idx;
    }
    __syncthreads();
    if (threadIdx.x < 32) {
        best = threadIdx.x < 8 ? sv[threadIdx.x] : -INFINITY;
        idx = threadIdx.x < 8 ? si[threadIdx.x] : -1;
#pragma unroll
        for (int o = 4; o > 0; o >>= 1)
            arg_merge(best, idx, __shfl_xor_sync(FULL, best, o), __shfl_xor_sync(FULL, idx, o));
        if (threadIdx.x == 0) {
            part[0] = best;
            part[1] = __int_as_float(idx);
            part[2] = __int_as_float(nan_any);
        }
    }
    ptx::cluster_sync();  // every part is in its CTA's shared memory
    if (rank == 0 && threadIdx.x < 32) {
        float4 p = make_float4(-INFINITY, __int_as_float(-1), __int_as_float(0), 0.f);
        if (threadIdx.x < kArgmaxCtas) p = ptx::ld_cluster_f4(ptx::mapa(part, threadIdx.x));
        best = p.x;
        idx = __float_as_int(p.y);
        int any = __float_as_int(p.z);
#pragma unroll
        for (int o = 4; o > 0; o >>= 1) {
            arg_merge(best, idx, __shfl_xor_sync(FULL, best, o), __shfl_xor_sync(FULL, idx, o));
            any |= __shfl_xor_sync(FULL, any, o);
        }
        if (threadIdx.x == 0) out[blockIdx.y] = any ? 0xFFFFFFFFu : (uint32_t)idx;
    }
    ptx::cluster_sync();  // rank 0 has read every part before any CTA leaves
}

__global__ void advance_kernel(const int32_t *slots, int B, int32_t *seq_len, int32_t *tok_pos) {
    ptx::griddep_wait();
    ptx::griddep_launch();
    int b = blockIdx.x * blockDim.x + threadIdx.x;
    if (b >= B) return;
    int slot = slots[b];
    int p = seq_len[slot];
    tok_pos[b] = p;
    seq_len[slot] = p + 1;
}

// ---- paged split-K decode attention -----------------------------------------------------------------------------
//
// CTA = (split, kv head h, batch row b): the pages [split * PPS, ...) of sequence slots[b]. Warp 4 streams each page's
// K+V block of head h (8 KiB contiguous) into a ring of ST shared-memory stages with cp.async.bulk, L2 evict-first
// (every cached byte is read once a step, so the step's other data keeps its place in L2); consumer warp w
// (0..3) handles the pages w, w + 4, ... of the split with its own online softmax for the two q heads 2h, 2h + 1:
//   scores: lane (half = lane / 16, li = lane % 16) reads dims 8 li .. 8 li + 7 of keys 2i + half (16-byte smem
//           loads, conflict-free), keeps 16 partial dots (8 keys x 2 heads) and a 4-step shuffle reduce-scatter
//           over the 16 lanes leaves lane li with the full score of key 2 (li / 2) + half for head li % 2;
//   softmax: log2 domain (scale folded with log2 e), running maximum per head, lane-local sums;
//   values: lane owns dims 4 lane .. 4 lane + 3 (8-byte smem loads), weights broadcast from shared memory as
//           (p_h0, p_h0, p_h1, p_h1), so each pair of dims and head is one packed f32x2 fma.
// The four warps' states merge in shared memory (each warp's output vectors in its own stage, which no copy targets
// once the warp's pages are done) and the split's (max, sum, unnormalised output) go to part_*; the combine kernel
// merges the splits. With max_splits == 1 (a batch large enough to fill the GPU with one CTA per row and kv head)
// the CTA writes the normalised output itself and no combine runs.
// A row's key count is usable when it is at least 1 and its pages fit both the page-table row and the max_splits
// split states per (row, kv head) that the scratch holds; anything else would read another row's pages or states.
__device__ __forceinline__ bool decode_len_ok(const DecodeAttnArgs &a, int len) {
    if (len < 1) return false;
    const long long npages = ((long long)len + kPageTokens - 1) / kPageTokens;
    return npages <= a.kv.max_pages_per_seq && npages <= (long long)a.max_splits * a.pages_per_split;
}

template <int ST>
__global__ void __launch_bounds__(160, 6) decode_attn_kernel(DecodeAttnArgs a) {
    // Consumer warp w takes the pages j = w (mod 4) and page j sits in stage j % ST. With ST a multiple of 4 every
    // stage belongs to one warp, which waits on it phase after phase. Otherwise a warp running ahead could wait on a
    // phase two beyond the barrier's current one, which the parity test cannot tell from a completed phase.
    static_assert(ST % 4 == 0, "the stage count must be a multiple of the four consumer warps");
    constexpr int PAGE_BYTES = 2 * kPageTokens * kHeadDim * 2;  // K + V of one head = 8 KiB
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t *stages = smem_raw;
    float *pbuf = (float *)(stages + ST * PAGE_BYTES);  // [4 warps][16 keys][4]
    float *red_m = pbuf + 4 * 64;                       // [4][2]
    float *red_l = red_m + 8;                           // [4][2]
    uint64_t *full = (uint64_t *)(red_l + 8);
    uint64_t *empty = full + ST;

    // Dependents may launch only after this kernel's wait: the combine reads its row's inputs before its own wait.
    if (!a.early_pages) {
        ptx::griddep_wait();
        ptx::griddep_launch();
    }
    const int split = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int slot = a.slots[b];
    const int32_t *ptab = a.kv.pages + (size_t)slot * a.kv.max_pages_per_seq;
    const int p0 = split * a.pages_per_split;
    // The producer warp fetches the split's first 32 page ids (one coalesced load, issued before the row's length
    // is known; entries past the row's pages are never used), so no bulk copy waits on its own page-table load.
    int pg = 0;
    if (warp == 4 && p0 + lane < a.kv.max_pages_per_seq) pg = ptab[p0 + lane];
    const int len = a.seq_len[slot];
    if (!decode_len_ok(a, len)) {  // keys beyond the page table: nothing is read, the host sees the code
        if (split == 0 && h == 0 && threadIdx.x == 0) atomicCAS(a.err, 0u, kErrDecodeLen);
        if (a.max_splits == 1 && threadIdx.x < 128)  // no combine follows: the row's two q heads are written as zeros
            for (int hh = 0; hh < 2; ++hh)
                a.out[((size_t)b * a.q_heads + 2 * h + hh) * kHeadDim + threadIdx.x] = __float2bfloat16_rn(0.f);
        return;
    }
    const int npages = (len + kPageTokens - 1) / kPageTokens;
    if (p0 >= npages) return;  // whole CTA, before any barrier
    const int n = min(npages - p0, a.pages_per_split);
    const size_t page_elems = kv_page_elems(a.kv.kv_heads);

    if (threadIdx.x == 0) {
        for (int s = 0; s < ST; ++s) {
            ptx::mbar_init(&full[s], 1);
            ptx::mbar_init(&empty[s], 1);
        }
        ptx::fence_barrier_init();
    }
    __syncthreads();
    int pre = 0;  // pages issued before the previous kernel completed (early_pages)
    if (a.early_pages) {
        if (warp == 4) {
            pre = max(0, min(min(n, ST), npages - 1 - p0));  // never the row's last page, where the new token lands
            for (int j = 0; j < pre; ++j) {
                const int page = __shfl_sync(FULL, pg, j);
                if (lane == 0) {
                    ptx::mbar_arrive_expect_tx(&full[j], PAGE_BYTES);
                    ptx::bulk_load_hint(stages + j * PAGE_BYTES,
                                        a.kv.pool + (size_t)page * page_elems + (size_t)h * 2 * kPageTokens * kHeadDim,
                                        PAGE_BYTES, &full[j], ptx::policy_evict_first());
                }
            }
        }
        ptx::griddep_wait();
        ptx::griddep_launch();
    }

    if (warp == 4) {
        // The whole warp walks the pages (lane j % 32 holds page j's id; the next 32 ids load in one go when the
        // walk reaches them) and lane 0 issues the copies.
        int j = pre;
        for (; j < n; ++j) {
            if ((j & 31) == 0 && j > 0) pg = p0 + j + lane < a.kv.max_pages_per_seq ? ptab[p0 + j + lane] : 0;
            const int page = __shfl_sync(FULL, pg, j & 31);
            const int s = j % ST;
            int ok = 1;
            if (lane == 0) {
                ok = ptx::mbar_wait(&empty[s], ((j / ST) & 1) ^ 1, a.err, 0x2001);
                if (ok) {
                    const __nv_bfloat16 *src =
                        a.kv.pool + (size_t)page * page_elems + (size_t)h * 2 * kPageTokens * kHeadDim;
                    ptx::mbar_arrive_expect_tx(&full[s], PAGE_BYTES);
                    ptx::bulk_load_hint(stages + s * PAGE_BYTES, src, PAGE_BYTES, &full[s], ptx::policy_evict_first());
                }
            }
            if (!__shfl_sync(FULL, ok, 0)) break;
        }
        if (lane == 0)
            for (int k = j > ST ? j - ST : 0; k < j; ++k) ptx::mbar_wait(&full[k % ST], (k / ST) & 1, a.err, 0x2002);
    } else {
        const int half = lane >> 4, li = lane & 15;
        float q0[8], q1[8];
        {
            const uint4 r0 = *reinterpret_cast<const uint4 *>(a.q + ((size_t)b * a.q_heads + 2 * h) * kHeadDim + 8 * li);
            const uint4 r1 =
                *reinterpret_cast<const uint4 *>(a.q + ((size_t)b * a.q_heads + 2 * h + 1) * kHeadDim + 8 * li);
            const uint32_t w0[4] = {r0.x, r0.y, r0.z, r0.w}, w1[4] = {r1.x, r1.y, r1.z, r1.w};
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                q0[2 * i] = __uint_as_float(w0[i] << 16) * a.scale_log2;
                q0[2 * i + 1] = __uint_as_float(w0[i] & 0xFFFF0000u) * a.scale_log2;
                q1[2 * i] = __uint_as_float(w1[i] << 16) * a.scale_log2;
                q1[2 * i + 1] = __uint_as_float(w1[i] & 0xFFFF0000u) * a.scale_log2;
            }
        }
        float m_run = -INFINITY, l_lane = 0.f;
        float acc0[4] = {0, 0, 0, 0}, acc1[4] = {0, 0, 0, 0};
        float *pw = pbuf + warp * 64;
        for (int j = warp; j < n; j += 4) {
            const int s = j % ST;
            if (!ptx::mbar_wait(&full[s], (j / ST) & 1, a.err, 0x2003)) break;
            const uint8_t *kb = stages + s * PAGE_BYTES;
            const uint8_t *vb = kb + PAGE_BYTES / 2;
            const int tok0 = (p0 + j) * kPageTokens;
            const int valid = min(kPageTokens, len - tok0);
            float v[16];
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const uint4 kr = *reinterpret_cast<const uint4 *>(kb + (2 * i + half) * 256 + li * 16);
                const uint32_t w[4] = {kr.x, kr.y, kr.z, kr.w};
                // even and odd dims accumulate in the two halves of a packed pair, summed at the end
                float d0e = 0.f, d0o = 0.f, d1e = 0.f, d1o = 0.f;
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const float ka = __uint_as_float(w[e] << 16), kb2 = __uint_as_float(w[e] & 0xFFFF0000u);
                    ptx::fma_x2(d0e, d0o, q0[2 * e], q0[2 * e + 1], ka, kb2, d0e, d0o);
                    ptx::fma_x2(d1e, d1o, q1[2 * e], q1[2 * e + 1], ka, kb2, d1e, d1o);
                }
                v[2 * i] = d0e + d0o;
                v[2 * i + 1] = d1e + d1o;
            }
            // reduce-scatter over the 16 lanes of this half: lane li ends with value index li
#pragma unroll
            for (int step = 0; step < 4; ++step) {
                const int m = 8 >> step, cnt = 16 >> step;
                const bool upper = (li & m) != 0;
#pragma unroll
                for (int i = 0; i < cnt / 2; ++i) {
                    const float send = upper ? v[i] : v[i + cnt / 2];
                    const float keep = upper ? v[i + cnt / 2] : v[i];
                    v[i] = keep + __shfl_xor_sync(FULL, send, m);
                }
            }
            const int key = 2 * (li >> 1) + half;
            float sc = key < valid ? v[0] : -INFINITY;
            float pm = sc;
            pm = fmaxf(pm, __shfl_xor_sync(FULL, pm, 2));
            pm = fmaxf(pm, __shfl_xor_sync(FULL, pm, 4));
            pm = fmaxf(pm, __shfl_xor_sync(FULL, pm, 8));
            pm = fmaxf(pm, __shfl_xor_sync(FULL, pm, 16));
            const float m_new = fmaxf(m_run, pm);
            const float alpha = exp2f(m_run - m_new);
            const float p = exp2f(sc - m_new);
            m_run = m_new;
            l_lane = l_lane * alpha + p;
            *reinterpret_cast<float2 *>(pw + key * 4 + (li & 1) * 2) = make_float2(p, p);
            const float al0 = __shfl_sync(FULL, alpha, 0), al1 = __shfl_sync(FULL, alpha, 1);
            __syncwarp();
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                acc0[e] *= al0;
                acc1[e] *= al1;
            }
            for (int t = 0; t < valid; ++t) {
                const uint2 vr = *reinterpret_cast<const uint2 *>(vb + t * 256 + lane * 8);
                const float4 pp = *reinterpret_cast<const float4 *>(pw + 4 * t);
                const float va = __uint_as_float(vr.x << 16), vb2 = __uint_as_float(vr.x & 0xFFFF0000u),
                            vc = __uint_as_float(vr.y << 16), vd = __uint_as_float(vr.y & 0xFFFF0000u);
                ptx::fma_x2(acc0[0], acc0[1], pp.x, pp.y, va, vb2, acc0[0], acc0[1]);
                ptx::fma_x2(acc0[2], acc0[3], pp.x, pp.y, vc, vd, acc0[2], acc0[3]);
                ptx::fma_x2(acc1[0], acc1[1], pp.z, pp.w, va, vb2, acc1[0], acc1[1]);
                ptx::fma_x2(acc1[2], acc1[3], pp.z, pp.w, vc, vd, acc1[2], acc1[3]);
            }
            __syncwarp();
            if (lane == 0) ptx::mbar_arrive(&empty[s]);
        }
        // per-head totals of this warp
        float l = l_lane;
        l += __shfl_xor_sync(FULL, l, 2);
        l += __shfl_xor_sync(FULL, l, 4);
        l += __shfl_xor_sync(FULL, l, 8);
        l += __shfl_xor_sync(FULL, l, 16);
        if (lane < 2) {
            red_m[warp * 2 + lane] = m_run;
            red_l[warp * 2 + lane] = l;
        }
        float *racc = reinterpret_cast<float *>(stages + warp * PAGE_BYTES);  // [2][128] in the warp's own stage
        *reinterpret_cast<float4 *>(racc + 4 * lane) = make_float4(acc0[0], acc0[1], acc0[2], acc0[3]);
        *reinterpret_cast<float4 *>(racc + 128 + 4 * lane) = make_float4(acc1[0], acc1[1], acc1[2], acc1[3]);
    }
    __syncthreads();
    if (threadIdx.x < 128) {
        const int d = threadIdx.x;
        const size_t base = ((size_t)b * a.kv.kv_heads + h) * a.max_splits + split;
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
            float M = -INFINITY;
#pragma unroll
            for (int w = 0; w < 4; ++w) M = fmaxf(M, red_m[w * 2 + hh]);
            float o = 0.f, l = 0.f;
#pragma unroll
            for (int w = 0; w < 4; ++w) {
                const float f = red_m[w * 2 + hh] == -INFINITY ? 0.f : exp2f(red_m[w * 2 + hh] - M);
                o += f * reinterpret_cast<const float *>(stages + w * PAGE_BYTES)[hh * 128 + d];
                l += f * red_l[w * 2 + hh];
            }
            if (a.max_splits == 1) {
                // One split per row: this state is the result. (0 + o) / (0 + l) is what the combine computes from a
                // single split (its weight is exactly 1), so both forms give the same bits.
                a.out[((size_t)b * a.q_heads + 2 * h + hh) * kHeadDim + d] = __float2bfloat16_rn((0.f + o) / (0.f + l));
            } else {
                a.part_o[(base * 2 + hh) * 128 + d] = o;
                if (d == 0) {
                    a.part_ml[(base * 2 + hh) * 2 + 0] = M;
                    a.part_ml[(base * 2 + hh) * 2 + 1] = l;
                }
            }
        }
    }
}

__global__ void __launch_bounds__(128) decode_combine_kernel(DecodeAttnArgs a) {
    // The row's length is an input of the attention kernel, which lets this kernel launch only after its own wait,
    // so it is final here before this kernel's wait; the split states are read after it.
    const int b = blockIdx.x, qh = blockIdx.y, d = threadIdx.x;
    const int h = qh / 2, hh = qh % 2;
    const int len = a.seq_len[a.slots[b]];
    ptx::griddep_wait();
    ptx::griddep_launch();
    if (!decode_len_ok(a, len)) {  // the attention kernel recorded the error; the row is written as zeros
        a.out[((size_t)b * a.q_heads + qh) * kHeadDim + d] = __float2bfloat16_rn(0.f);
        return;
    }
    const int npages = (len + kPageTokens - 1) / kPageTokens;
    const int nsplit = (npages + a.pages_per_split - 1) / a.pages_per_split;
    const size_t base = ((size_t)b * a.kv.kv_heads + h) * a.max_splits;
    const float *ml = a.part_ml + (base * 2 + hh) * 2;    // split s: ml[4 s] = max, ml[4 s + 1] = sum
    const float *po = a.part_o + (base * 2 + hh) * 128 + d;  // split s: po[256 s]
    float M = -INFINITY, o = 0.f, l = 0.f;
    constexpr int kHeld = 16;
    if (nsplit <= kHeld) {
        // every split's state is loaded before any is used, so the loads are in flight together
        float mv[kHeld], lv[kHeld], ov[kHeld];
#pragma unroll
        for (int s = 0; s < kHeld; ++s)
            if (s < nsplit) {
                mv[s] = ml[4 * s];
                lv[s] = ml[4 * s + 1];
                ov[s] = po[256 * s];
            }
#pragma unroll
        for (int s = 0; s < kHeld; ++s)
            if (s < nsplit) M = fmaxf(M, mv[s]);
#pragma unroll
        for (int s = 0; s < kHeld; ++s)
            if (s < nsplit) {
                const float f = mv[s] == -INFINITY ? 0.f : exp2f(mv[s] - M);
                o += f * ov[s];
                l += f * lv[s];
            }
    } else {
        for (int s = 0; s < nsplit; ++s) M = fmaxf(M, ml[4 * s]);
        for (int s = 0; s < nsplit; ++s) {
            const float m = ml[4 * s];
            const float f = m == -INFINITY ? 0.f : exp2f(m - M);
            o += f * po[256 * s];
            l += f * ml[4 * s + 1];
        }
    }
    a.out[((size_t)b * a.q_heads + qh) * kHeadDim + d] = __float2bfloat16_rn(o / l);
}

}  // namespace

cudaError_t launch_norm_rows_block(const float *x, int T, int hidden, const __nv_bfloat16 *w, float eps,
                                   __nv_bfloat16 *xn, cudaStream_t st, const int32_t *idx) {
    return launch_kernel(norm_rows_block_kernel, dim3(T), dim3(256), 0, st, x, idx, hidden, w, eps, xn);
}

cudaError_t launch_argmax(const float *logits, int R, int V, uint32_t *out, cudaStream_t st) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(kArgmaxCtas, R);
    cfg.blockDim = dim3(256);
    cfg.stream = st;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = kArgmaxCtas;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl_enabled() ? 2 : 1;
    return cudaLaunchKernelEx(&cfg, argmax_kernel, logits, V, out);
}

cudaError_t launch_advance(const int32_t *slots, int B, int32_t *seq_len, int32_t *tok_pos, cudaStream_t st) {
    return launch_kernel(advance_kernel, dim3((B + 127) / 128), dim3(128), 0, st, slots, B, seq_len, tok_pos);
}

cudaError_t launch_decode_attention(const DecodeAttnArgs &a, cudaStream_t st) {
    constexpr int ST = 4;  // 34 KiB of shared memory a CTA, six CTAs an SM (measured faster than 8 / 12 / 16)
    const size_t smem = ST * 8192 + (4 * 64 + 16) * sizeof(float) + 2 * ST * sizeof(uint64_t);
    static SmemOptIn opt;
    cudaError_t e = opt.set((const void *)decode_attn_kernel<ST>, (int)smem);
    if (e != cudaSuccess) return e;
    e = launch_kernel(decode_attn_kernel<ST>, dim3(a.max_splits, a.kv.kv_heads, a.B), dim3(160), smem, st, a);
    if (e != cudaSuccess || a.max_splits == 1) return e;  // a single split writes the output itself
    return launch_kernel(decode_combine_kernel, dim3(a.B, a.q_heads), dim3(128), 0, st, a);
}

}  // namespace lrm
