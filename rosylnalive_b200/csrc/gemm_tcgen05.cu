// gemm_tcgen05.cu -- D = A * B^T on the 5th-generation tensor cores (tcgen05) for sm_100a.
//
// A [M, K] and B [N, K] are bf16, K-major (the PyTorch Linear layout for weights; activations row-major); the
// accumulation is fp32 in tensor memory (TMEM). One persistent CTA per SM walks the output tiles (128 x BN) and, with
// split-K, the K ranges:
//   warp 0      TMA producer: one elected thread loads A and B k-blocks (64 wide, 128-byte swizzle) into a ring of
//               STAGES shared-memory stages, each completing a `full` mbarrier;
//   warp 1      allocates TMEM (2 x BN columns: two accumulators, so the epilogue of tile i overlaps the MMAs of tile
//               i + 1) and one elected thread issues tcgen05.mma (M=128, N=BN, K=16) per 16-wide k step, releasing a
//               stage with tcgen05.commit on its `empty` mbarrier and a finished accumulator on `acc_full`;
//   warps 2..5  epilogue: each thread owns one accumulator row (TMEM lane), reads it 16 columns at a time with
//               tcgen05.ld and applies the epilogue, then frees the accumulator on `acc_empty`.
// No TMA multicast is used. Every mbarrier wait is bounded (ptx::mbar_wait) and reports a code in the error word.
//
// Epilogues:
//   EPI_F32      out_f32[m, n] = acc
//   EPI_RESID    out_f32[m, n] = resid[m, n] + acc      (resid may be out: the residual stream updated in place)
//   EPI_SWIGLU   B rows are gate/up interleaved in blocks of 64 (gate 64, up 64, ...); out_bf16[m, n/2 + j] =
//                bf16(silu(gate_j) * up_j) for the 64-blocks of each 128 columns
//   EPI_PARTIAL  swap-AB split-K partials, transposed: partial[split][n][m] = acc (M indexes weight rows and N
//                tokens, so this writes Y[token][feature] partial sums for a consumer to reduce in a fixed order)
//   EPI_BF16     out_bf16[m, n] = bf16(acc)
//   EPI_QKV      prefill q/k/v: per 128-column head, QK-RMSNorm and RoPE for q and k, then bf16 q/k/v written to their
//                contiguous buffers and k/v appended to the paged KV cache (QkvEpilogue)
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include <string.h>

#include "gemm.h"
#include "internal.h"
#include "ptx.cuh"

namespace lrm {

namespace {

constexpr int BM = 128;
constexpr int BK = 64;
constexpr int UMMA_K = 16;
constexpr int kThreads = 192;

template <int BN>
struct Cfg {
    static constexpr int A_BYTES = BM * BK * 2;
    static constexpr int B_BYTES = BN * BK * 2;
    static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
    static constexpr int STAGES = (BN == 256) ? 4 : (BN == 128 ? 6 : 8);
    static constexpr int TMEM_COLS = 2 * BN;
    static constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024 /*align*/ + 256 /*barriers*/;
};

__device__ __forceinline__ float bf16lo(uint32_t u) { return __uint_as_float(u << 16); }

__device__ __forceinline__ uint32_t pack_bf16(float a, float b) {
    __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t *>(&h);
}

// The per-head RMSNorm and NeoX rotation of one dim pair (i, i + 64) of q or k, as the same operations in the same
// order on every path (the one-CTA and CTA-pair epilogues must agree bit for bit): x = (v * r) * w, then
// lo' = fma(x_lo, c, -(x_hi * s)) and hi' = fma(x_hi, c, x_lo * s), both lanes at once on the packed f32x2 pipe.
__device__ __forceinline__ void norm_rope_pair(float &lo, float &hi, float r, float wl, float wh, float c, float s) {
    asm("{\n\t.reg .b64 v, rr, w, x, xs, ns, cc, u, d;\n\t"
        "mov.b64 v, {%0, %1};\n\tmov.b64 rr, {%2, %2};\n\tmov.b64 w, {%3, %4};\n\t"
        "mul.rn.f32x2 x, v, rr;\n\tmul.rn.f32x2 x, x, w;\n\t"  // (x_lo, x_hi)
        "{\n\t.reg .f32 xl, xh, nsv;\n\tmov.b64 {xl, xh}, x;\n\tmov.b64 xs, {xh, xl};\n\t"
        "neg.f32 nsv, %6;\n\tmov.b64 ns, {nsv, %6};\n\t}\n\t"
        "mul.rn.f32x2 u, xs, ns;\n\t"                              // (-(x_hi s), x_lo s)
        "mov.b64 cc, {%5, %5};\n\tfma.rn.f32x2 d, x, cc, u;\n\t"
        "mov.b64 {%0, %1}, d;\n\t}"
        : "+f"(lo), "+f"(hi)
        : "f"(r), "f"(wl), "f"(wh), "f"(c), "f"(s));
}

// silu(g) = g / (1 + e^-g) with the approximate division (rcp.approx, about 2 ulp in fp32; the result is rounded to
// bf16 next), the form the decode GEMMs' SwiGLU epilogue (gemm_decode.cu) uses too.
__device__ __forceinline__ float silu_f(float g) { return __fdividef(g, 1.0f + __expf(-g)); }

// The epilogue of one accumulator row (thread = TMEM lane): row `row` of the output, columns n0..n0+BN-1, read
// from tensor memory at t_row (the row's lane, the accumulator's first column). has_k is false for an empty k
// range (the accumulator is then treated as zero).
template <int BN, int EPI>
__device__ __forceinline__ void epilogue_tile(const GemmArgs &args, uint32_t t_row, int row, int n0, bool has_k,
                                              int split) {
    if (EPI == EPI_QKV) {
        // Two light passes over TMEM per 128-column head: the sum of squares, then the RoPE pairs (i, i + 64)
        // sixteen at a time, normalised, rotated, rounded to bf16 and stored; few registers, vector loads.
        const QkvEpilogue &E = args.qkv;
        const bool row_ok = row < args.M;
        const int pos = row_ok ? E.tok_pos[row] : 0;
        const int slot = row_ok ? E.tok_slot[row] : 0;
#pragma unroll 1
        for (int hh = 0; hh < BN / 128; ++hh) {
            const uint32_t t_head = t_row + hh * 128;
            const int head_row = (n0 + hh * 128) / 128;
            const bool is_q = head_row < E.q_heads, is_k = !is_q && head_row < E.q_heads + E.kv_heads;
            const bool rotate = is_q || is_k;
            float r = 1.f;
            if (rotate) {
                float ss = 0.f;
#pragma unroll 1
                for (int c = 0; c < 8; c += 2) {
                    uint32_t u0[16], u1[16];
                    ptx::tmem_ld16(t_head + c * 16, u0);
                    ptx::tmem_ld16(t_head + c * 16 + 16, u1);
                    ptx::tmem_ld_wait();
                    // columns in order, as the staged (CTA-pair) epilogue sums them
#pragma unroll
                    for (int j = 0; j < 16; ++j) ss = fmaf(__uint_as_float(u0[j]), __uint_as_float(u0[j]), ss);
#pragma unroll
                    for (int j = 0; j < 16; ++j) ss = fmaf(__uint_as_float(u1[j]), __uint_as_float(u1[j]), ss);
                }
                r = rsqrtf(ss / 128.0f + E.eps);
            }
            __nv_bfloat16 *dst0 = nullptr, *dst1 = nullptr;
            if (row_ok && n0 + hh * 128 < args.N) {
                if (is_q) {
                    dst0 = E.q_out + ((size_t)row * E.q_heads + head_row) * 128;
                } else {
                    const int kvh = is_k ? head_row - E.q_heads : head_row - E.q_heads - E.kv_heads;
                    __nv_bfloat16 *flat = is_k ? E.k_out : E.v_out;  // optional contiguous copy
                    dst0 = flat ? flat + ((size_t)row * E.kv_heads + kvh) * 128 : nullptr;
                    const int page = E.pages[(size_t)slot * E.pages_per_seq + pos / 16];
                    dst1 = E.pool + (size_t)page * E.kv_heads * 2 * 16 * 128 +
                           ((size_t)(kvh * 2 + (is_k ? 0 : 1)) * 16 + pos % 16) * 128;
                }
            }
            const __nv_bfloat16 *nw = is_q ? E.q_norm : E.k_norm;
#pragma unroll 1
            for (int c = 0; c < 4; ++c) {  // dims 16c..16c+15 pair with 64+16c..64+16c+15
                uint32_t lo[16], hi[16];
                ptx::tmem_ld16(t_head + c * 16, lo);
                ptx::tmem_ld16(t_head + 64 + c * 16, hi);
                ptx::tmem_ld_wait();
                float a[16], b[16];
#pragma unroll
                for (int j = 0; j < 16; ++j) {
                    a[j] = has_k ? __uint_as_float(lo[j]) : 0.f;
                    b[j] = has_k ? __uint_as_float(hi[j]) : 0.f;
                }
                if (rotate && (dst0 || dst1)) {
                    const float4 *cs4 = reinterpret_cast<const float4 *>(E.cos_t + (size_t)pos * 64 + 16 * c);
                    const float4 *sn4 = reinterpret_cast<const float4 *>(E.sin_t + (size_t)pos * 64 + 16 * c);
                    const uint4 *wl4 = reinterpret_cast<const uint4 *>(nw + 16 * c);
                    const uint4 *wh4 = reinterpret_cast<const uint4 *>(nw + 64 + 16 * c);
                    float cf[16], sf[16], wl[16], wh[16];
#pragma unroll
                    for (int q = 0; q < 4; ++q) {
                        const float4 cv = cs4[q], sv = sn4[q];
                        cf[4 * q] = cv.x; cf[4 * q + 1] = cv.y; cf[4 * q + 2] = cv.z; cf[4 * q + 3] = cv.w;
                        sf[4 * q] = sv.x; sf[4 * q + 1] = sv.y; sf[4 * q + 2] = sv.z; sf[4 * q + 3] = sv.w;
                    }
#pragma unroll
                    for (int q = 0; q < 2; ++q) {
                        const uint4 l = wl4[q], h = wh4[q];
                        const uint32_t lw[4] = {l.x, l.y, l.z, l.w}, hw[4] = {h.x, h.y, h.z, h.w};
#pragma unroll
                        for (int e = 0; e < 4; ++e) {
                            wl[8 * q + 2 * e] = __uint_as_float(lw[e] << 16);
                            wl[8 * q + 2 * e + 1] = __uint_as_float(lw[e] & 0xFFFF0000u);
                            wh[8 * q + 2 * e] = __uint_as_float(hw[e] << 16);
                            wh[8 * q + 2 * e + 1] = __uint_as_float(hw[e] & 0xFFFF0000u);
                        }
                    }
#pragma unroll
                    for (int j = 0; j < 16; ++j) norm_rope_pair(a[j], b[j], r, wl[j], wh[j], cf[j], sf[j]);
                }
                if (dst0 || dst1) {
                    uint32_t pl[8], ph[8];
#pragma unroll
                    for (int e = 0; e < 8; ++e) {
                        pl[e] = pack_bf16(a[2 * e], a[2 * e + 1]);
                        ph[e] = pack_bf16(b[2 * e], b[2 * e + 1]);
                    }
                    const uint4 l0 = make_uint4(pl[0], pl[1], pl[2], pl[3]), l1 = make_uint4(pl[4], pl[5], pl[6], pl[7]);
                    const uint4 h0 = make_uint4(ph[0], ph[1], ph[2], ph[3]), h1 = make_uint4(ph[4], ph[5], ph[6], ph[7]);
                    if (dst0) {
                        uint4 *d0 = reinterpret_cast<uint4 *>(dst0 + 16 * c);
                        uint4 *e0 = reinterpret_cast<uint4 *>(dst0 + 64 + 16 * c);
                        d0[0] = l0; d0[1] = l1; e0[0] = h0; e0[1] = h1;
                    }
                    if (dst1) {
                        uint4 *d1 = reinterpret_cast<uint4 *>(dst1 + 16 * c);
                        uint4 *e1 = reinterpret_cast<uint4 *>(dst1 + 64 + 16 * c);
                        d1[0] = l0; d1[1] = l1; e1[0] = h0; e1[1] = h1;
                    }
                }
            }
        }
    } else if (EPI == EPI_SWIGLU) {
        for (int b = 0; b < BN / 128; ++b) {
#pragma unroll 1
            for (int j = 0; j < 4; ++j) {
                uint32_t g[16], u[16];
                ptx::tmem_ld16(t_row + b * 128 + j * 16, g);
                ptx::tmem_ld16(t_row + b * 128 + 64 + j * 16, u);
                ptx::tmem_ld_wait();
                if (row < args.M && n0 + b * 128 < args.N) {
                    uint32_t packed[8];
#pragma unroll
                    for (int e = 0; e < 8; ++e) {
                        float g0 = has_k ? __uint_as_float(g[2 * e]) : 0.f;
                        float g1 = has_k ? __uint_as_float(g[2 * e + 1]) : 0.f;
                        float u0 = has_k ? __uint_as_float(u[2 * e]) : 0.f;
                        float u1 = has_k ? __uint_as_float(u[2 * e + 1]) : 0.f;
                        packed[e] = pack_bf16(silu_f(g0) * u0, silu_f(g1) * u1);
                    }
                    __nv_bfloat16 *dst = args.out_bf16 + (size_t)row * args.ldo + (n0 + b * 128) / 2 + j * 16;
                    uint4 *d4 = reinterpret_cast<uint4 *>(dst);
                    d4[0] = make_uint4(packed[0], packed[1], packed[2], packed[3]);
                    d4[1] = make_uint4(packed[4], packed[5], packed[6], packed[7]);
                }
            }
        }
    } else {
#pragma unroll 1
        for (int c = 0; c < BN / 16; ++c) {
            uint32_t v[16];
            ptx::tmem_ld16(t_row + c * 16, v);
            ptx::tmem_ld_wait();
            if (!has_k)
#pragma unroll
                for (int e = 0; e < 16; ++e) v[e] = 0;
            const int col = n0 + c * 16;
            if (col >= args.N) continue;
            const int ncols = min(16, args.N - col);
            if (EPI == EPI_PARTIAL) {
                if (row < args.M) {
                    float *p = args.partial + (size_t)split * args.split_stride + (size_t)col * args.ldo + row;
#pragma unroll
                    for (int e = 0; e < 16; ++e)
                        if (e < ncols) p[(size_t)e * args.ldo] = __uint_as_float(v[e]);
                }
            } else if (row < args.M) {
                if (EPI == EPI_BF16) {
                    __nv_bfloat16 *dst = args.out_bf16 + (size_t)row * args.ldo + col;
                    if (ncols == 16) {
                        uint4 *d4 = reinterpret_cast<uint4 *>(dst);
                        d4[0] = make_uint4(pack_bf16(__uint_as_float(v[0]), __uint_as_float(v[1])),
                                           pack_bf16(__uint_as_float(v[2]), __uint_as_float(v[3])),
                                           pack_bf16(__uint_as_float(v[4]), __uint_as_float(v[5])),
                                           pack_bf16(__uint_as_float(v[6]), __uint_as_float(v[7])));
                        d4[1] = make_uint4(pack_bf16(__uint_as_float(v[8]), __uint_as_float(v[9])),
                                           pack_bf16(__uint_as_float(v[10]), __uint_as_float(v[11])),
                                           pack_bf16(__uint_as_float(v[12]), __uint_as_float(v[13])),
                                           pack_bf16(__uint_as_float(v[14]), __uint_as_float(v[15])));
                    } else {
                        for (int e = 0; e < ncols; ++e) dst[e] = __float2bfloat16_rn(__uint_as_float(v[e]));
                    }
                } else {
                    float *dst = args.out_f32 + (size_t)row * args.ldo + col;
                    float f[16];
#pragma unroll
                    for (int e = 0; e < 16; ++e) f[e] = __uint_as_float(v[e]);
                    if (EPI == EPI_RESID) {
                        const float *r = args.resid + (size_t)row * args.ldr + col;
                        if (ncols == 16) {
#pragma unroll
                            for (int e4 = 0; e4 < 4; ++e4) {
                                float4 rv = reinterpret_cast<const float4 *>(r)[e4];
                                f[4 * e4 + 0] += rv.x;
                                f[4 * e4 + 1] += rv.y;
                                f[4 * e4 + 2] += rv.z;
                                f[4 * e4 + 3] += rv.w;
                            }
                        } else {
                            for (int e = 0; e < ncols; ++e) f[e] += r[e];
                        }
                    }
                    if (ncols == 16) {
                        float4 *d4 = reinterpret_cast<float4 *>(dst);
#pragma unroll
                        for (int e4 = 0; e4 < 4; ++e4)
                            d4[e4] = make_float4(f[4 * e4], f[4 * e4 + 1], f[4 * e4 + 2], f[4 * e4 + 3]);
                    } else {
                        for (int e = 0; e < ncols; ++e) dst[e] = f[e];
                    }
                }
            }
        }
    }
}

template <int BN, int EPI>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
                GemmArgs args) {
    using C = Cfg<BN>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = (uint8_t *)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    uint64_t *full = (uint64_t *)(smem + C::STAGES * C::STAGE_BYTES);
    uint64_t *empty = full + C::STAGES;
    uint64_t *acc_full = empty + C::STAGES;
    uint64_t *acc_empty = acc_full + 2;
    uint64_t *mma_done = acc_empty + 2;
    uint32_t *tmem_slot = (uint32_t *)(mma_done + 1);

    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    const int m_tiles = (args.M + BM - 1) / BM, n_tiles = (args.N + BN - 1) / BN;
    const int nkb = (args.K + BK - 1) / BK;
    const int kbps = args.kb_per_split;
    const int total = m_tiles * n_tiles * args.splits;
    uint32_t *err = args.err;

    if (threadIdx.x == 0) {
        for (int s = 0; s < C::STAGES; ++s) {
            ptx::mbar_init(&full[s], 1);
            ptx::mbar_init(&empty[s], 1);
        }
        for (int a = 0; a < 2; ++a) {
            ptx::mbar_init(&acc_full[a], 1);
            ptx::mbar_init(&acc_empty[a], 4);
        }
        ptx::mbar_init(mma_done, 1);
        ptx::fence_barrier_init();
        ptx::prefetch_tmap(&tmap_a);
        ptx::prefetch_tmap(&tmap_b);
    }
    if (warp == 1) {
        ptx::tmem_alloc(tmem_slot, C::TMEM_COLS);
        ptx::tmem_relinquish();
    }
    ptx::tc_fence_before();
    __syncthreads();
    ptx::tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    ptx::griddep_launch();

    // Tile t -> (split, m block, n block); n is fastest so consecutive CTAs share the A rows.
    auto decode_tile = [&](int t, int &split, int &mb, int &nb) {
        split = t / (m_tiles * n_tiles);
        int r = t % (m_tiles * n_tiles);
        mb = r / n_tiles;
        nb = r % n_tiles;
    };
    auto kb_range = [&](int split, int &k0, int &k1) {
        k0 = split * kbps;
        k1 = min(nkb, k0 + kbps);
    };

    if (warp == 0) {
        if (ptx::elect_one()) {
            uint32_t it = 0;
            bool ok = true;
            // Under programmatic dependent launch, the operand no earlier kernel writes (the weights) is fetched for
            // the first stages of the first tile before waiting for the previous kernel; the other operand after.
            int pre = 0;
            if (args.independent && (int)blockIdx.x < total) {
                int split, mb, nb, k0, k1;
                decode_tile(blockIdx.x, split, mb, nb);
                kb_range(split, k0, k1);
                pre = min(C::STAGES, max(0, k1 - k0));
                for (int j = 0; j < pre; ++j) {
                    uint8_t *sa = smem + j * C::STAGE_BYTES;
                    ptx::mbar_arrive_expect_tx(&full[j], C::STAGE_BYTES);
                    if (args.independent == 1)
                        ptx::tma_load_2d(sa, &tmap_a, &full[j], (k0 + j) * BK, mb * BM);
                    else
                        ptx::tma_load_2d(sa + C::A_BYTES, &tmap_b, &full[j], (k0 + j) * BK, nb * BN);
                }
            }
            ptx::griddep_wait();
            for (int t = blockIdx.x; t < total && ok; t += gridDim.x) {
                int split, mb, nb, k0, k1;
                decode_tile(t, split, mb, nb);
                kb_range(split, k0, k1);
                for (int kb = k0; kb < k1; ++kb, ++it) {
                    int s = it % C::STAGES;
                    uint32_t ph = (it / C::STAGES) & 1;
                    uint8_t *sa = smem + s * C::STAGE_BYTES;
                    uint8_t *sb = sa + C::A_BYTES;
                    if ((int)it < pre) {  // armed above; only the dependent operand is left
                        if (args.independent == 1)
                            ptx::tma_load_2d(sb, &tmap_b, &full[s], kb * BK, nb * BN);
                        else
                            ptx::tma_load_2d(sa, &tmap_a, &full[s], kb * BK, mb * BM);
                        continue;
                    }
                    if (!ptx::mbar_wait(&empty[s], ph ^ 1, err, 0x1001)) {
                        ok = false;
                        break;
                    }
                    ptx::mbar_arrive_expect_tx(&full[s], C::STAGE_BYTES);
                    ptx::tma_load_2d(sa, &tmap_a, &full[s], kb * BK, mb * BM);
                    ptx::tma_load_2d(sb, &tmap_b, &full[s], kb * BK, nb * BN);
                }
            }
            // Let every load this thread issued land before the CTA can exit (normally they all have).
            uint32_t first = it > (uint32_t)C::STAGES ? it - C::STAGES : 0;
            for (uint32_t j = first; j < it; ++j)
                ptx::mbar_wait(&full[j % C::STAGES], (j / C::STAGES) & 1, err, 0x1002);
        }
    } else if (warp == 1) {
        ptx::griddep_wait();
        if (ptx::elect_one()) {
            constexpr uint32_t idesc = ptx::idesc_bf16_f32(BM, BN);
            uint32_t it = 0, local = 0;
            bool ok = true;
            for (int t = blockIdx.x; t < total && ok; t += gridDim.x, ++local) {
                int split, mb, nb, k0, k1;
                decode_tile(t, split, mb, nb);
                kb_range(split, k0, k1);
                const int a = local & 1;
                if (!ptx::mbar_wait(&acc_empty[a], ((local >> 1) & 1) ^ 1, err, 0x1003)) break;
                ptx::tc_fence_after();
                const uint32_t d_tmem = tmem_base + a * BN;
                for (int kb = k0; kb < k1; ++kb, ++it) {
                    int s = it % C::STAGES;
                    if (!ptx::mbar_wait(&full[s], (it / C::STAGES) & 1, err, 0x1004)) {
                        ok = false;
                        break;
                    }
                    ptx::tc_fence_after();
                    uint32_t sa = ptx::smem_u32(smem + s * C::STAGE_BYTES);
                    uint32_t sb = sa + C::A_BYTES;
#pragma unroll
                    for (int k = 0; k < BK / UMMA_K; ++k) {
                        uint64_t da = ptx::sw128_kmajor_desc(sa + k * UMMA_K * 2);
                        uint64_t db = ptx::sw128_kmajor_desc(sb + k * UMMA_K * 2);
                        ptx::mma_bf16(d_tmem, da, db, idesc, (kb > k0 || k > 0) ? 1u : 0u);
                    }
                    ptx::mma_commit(&empty[s]);
                }
                ptx::mma_commit(&acc_full[a]);
            }
            ptx::mma_commit(mma_done);
            ptx::mbar_wait(mma_done, 0, err, 0x1005);
        }
    } else {
        // Epilogue warps 2..5: TMEM lane quarter q = warp % 4 holds rows 32q..32q+31 of the tile. They read the
        // residual and write outputs that the previous kernel may still use, so they wait for it first.
        ptx::griddep_wait();
        const int q = warp & 3;
        uint32_t local = 0;
        for (int t = blockIdx.x; t < total; t += gridDim.x, ++local) {
            int split, mb, nb, k0, k1;
            decode_tile(t, split, mb, nb);
            kb_range(split, k0, k1);
            const int a = local & 1;
            if (!ptx::mbar_wait(&acc_full[a], (local >> 1) & 1, err, 0x1006)) break;
            ptx::tc_fence_after();
            const int row = mb * BM + q * 32 + lane;  // M index
            const uint32_t t_row = tmem_base + a * BN + ((uint32_t)(q * 32) << 16);
            const int n0 = nb * BN;
            const bool has_k = k1 > k0;
            epilogue_tile<BN, EPI>(args, t_row, row, n0, has_k, split);
            ptx::tc_fence_before();
            __syncwarp();
            if (lane == 0) ptx::mbar_arrive(&acc_empty[a]);
        }
    }
    ptx::tc_fence_before();
    __syncthreads();
    ptx::tc_fence_after();
    if (warp == 1) ptx::tmem_dealloc(tmem_base, C::TMEM_COLS);
}

// ---- CTA-pair variant (tcgen05 cta_group::2) ----------------------------------------------------------------------
//
// A cluster of two CTAs on neighbouring SMs shares a 256 x 256 output tile: CTA r loads A rows 128 r..128 r + 127
// and B rows 128 r..128 r + 127 of the tile (32 KiB a stage, so 7 stages fit), and one thread of the even CTA issues
// M = 256, N = 256 MMAs that read both CTAs' shared memory and write rows 0..127 of the accumulator into the even CTA's
// TMEM and rows 128..255 into the odd CTA's. Each CTA thus streams half the B traffic of a 128 x 256 tile for the
// same MMA work. Both CTAs' loads complete on the even CTA's `full` barrier (armed there for both); the MMA commits
// arrive on `empty` / `acc_full` in both CTAs; both CTAs' epilogue warps release an accumulator on the even CTA's
// `acc_empty`. Split-K and the transposed partial epilogue are not offered here.
//
// The epilogue is staged through shared memory: each thread moves its accumulator row from TMEM into a per-warp
// buffer of 32 rows x 128 bytes (16-byte chunks XOR-swizzled by row, so the warp's row-wise writes and its
// line-wise reads are free of bank conflicts), then the warp reads the buffer back eight lanes to a 128-byte row
// segment, so every global load and store covers whole 128-byte lines. A residual is prefetched into L2 for the
// whole tile before its accumulator is ready.
constexpr int kPairStages = 6;
constexpr int kPairStageBytes = 2 * 128 * BK * 2;  // A half + B half
constexpr int kStageBuf = 32 * 128;                 // one warp's 32 rows x 128 bytes
constexpr int kEpiBytes = 4 * 2 * kStageBuf;        // four epilogue warps, two buffers each
constexpr int kNormBytes = 2 * 128 * 2;           // q_norm and k_norm gains (EPI_QKV), staged once per CTA
constexpr int kPairSmem = kPairStages * kPairStageBytes + kEpiBytes + 1024 + 256 + kNormBytes;
// The i-th tile of a pair (tiles n fastest within a 256-row block): runs of RUN consecutive tiles, run p, p + npairs,
// ... for pair p. The q/k/v epilogue takes 4-tile runs: a run's tiles share their rows, so the rows' RoPE table
// entries, loaded for its first tile, serve the rest (4-tile runs keep the pairs' loads within one tile of even at
// the prefill sizes). The other epilogues take single tiles, which keep fewer row blocks (A panels) in L2 at once.
template <int RUN>
__device__ __forceinline__ int pair_tile(int pair, int npairs, int i) {
    return ((i / RUN) * npairs + pair) * RUN + i % RUN;
}

__device__ __forceinline__ uint32_t swz(uint32_t buf, int r, int chunk) {
    return buf + r * 128 + ((chunk ^ (r & 7)) << 4);
}

// Writes the 8 bf16 of `v` to dst[0..n) (n < 8: the ragged right edge).
__device__ __forceinline__ void store_bf16_tail(__nv_bfloat16 *dst, uint4 v, int n) {
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
    for (int e = 0; e < n; ++e) {
        const uint16_t h = (uint16_t)(w[e >> 1] >> ((e & 1) * 16));
        dst[e] = *reinterpret_cast<const __nv_bfloat16 *>(&h);
    }
}

// A row's sum of squares over a 256-column tile in the staged epilogue, in two steps. Each lane adds the squares of
// its four columns of every pass to its own partial (fused multiply-adds in pass, then column order: lane_ss), and
// after the eight passes a butterfly over the eight lanes that hold the row (lanes 8 rq .. 8 rq + 7: row_ss) leaves
// the total, the same bits in all eight. pair_prep_kernel computes the same sums from the residual stream in the
// same order.
__device__ __forceinline__ float lane_ss(float4 f, float acc) {
    acc = fmaf(f.x, f.x, acc);
    acc = fmaf(f.y, f.y, acc);
    acc = fmaf(f.z, f.z, acc);
    return fmaf(f.w, f.w, acc);
}
__device__ __forceinline__ float row_ss(float lane_partial) {
    lane_partial += __shfl_xor_sync(0xffffffffu, lane_partial, 1);
    lane_partial += __shfl_xor_sync(0xffffffffu, lane_partial, 2);
    return lane_partial + __shfl_xor_sync(0xffffffffu, lane_partial, 4);
}

// The RMSNorm scale of output row m for a consumer GEMM whose A rows are bf16(gain * x): the row's group sums added
// in group order (1 for a row past M, or without row_ss).
__device__ __forceinline__ float row_norm_scale(const GemmArgs &args, int m) {
    if (!args.row_ss || m >= args.M) return 1.f;
    float s = 0.f;
    for (int g = 0; g < args.row_nss; ++g) s += args.row_ss[(size_t)g * args.row_ss_stride + m];
    return rsqrtf(s / args.row_hidden + args.row_eps);
}

// One warp's share of a 256 x 256 pair tile: output rows row0..row0+31 (TMEM lanes of t_warp), columns n0..n0+255.
// buf: the warp's two staging buffers (shared::cta addresses).
template <int EPI>
__device__ __forceinline__ void epilogue_staged(const GemmArgs &args, uint32_t t_warp, int row0, int n0,
                                                uint32_t buf, int lane) {
    const int sub = lane & 7, rq = lane >> 3;  // read-back: 16-byte chunk, row within each group of four
    if (EPI == EPI_F32 || EPI == EPI_RESID) {
        // With the fused norm (EPI_RESID and norm_u): the lane's partial sums of squares of the rows it writes (rows
        // 4 it + rq) over this 256-column tile; see lane_ss / row_ss.
        const bool fused_norm = EPI == EPI_RESID && args.norm_u != nullptr;
        float ssacc[8];
#pragma unroll
        for (int it = 0; it < 8; ++it) ssacc[it] = 0.f;
#pragma unroll 1
        for (int c = 0; c < 8; ++c) {  // 32 fp32 columns a pass
            const uint32_t b = buf + (c & 1) * kStageBuf;
            uint32_t v[32];
            ptx::tmem_ld32(t_warp + c * 32, v);
            ptx::tmem_ld_wait();
#pragma unroll
            for (int j = 0; j < 8; ++j) ptx::st_shared_v4(swz(b, lane, j), v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
            __syncwarp();
            const int col = n0 + c * 32 + sub * 4;
            const int ncols = min(4, args.N - col);
            float4 res[8];
            if (EPI == EPI_RESID) {
#pragma unroll
                for (int it = 0; it < 8; ++it) {
                    const int grow = row0 + 4 * it + rq;
                    res[it] = make_float4(0.f, 0.f, 0.f, 0.f);
                    if (grow < args.M && ncols == 4)
                        res[it] = *reinterpret_cast<const float4 *>(args.resid + (size_t)grow * args.ldr + col);
                }
            }
            uint2 gw = make_uint2(0, 0);
            if (fused_norm && ncols == 4) gw = *reinterpret_cast<const uint2 *>(args.norm_gain + col);
#pragma unroll
            for (int it = 0; it < 8; ++it) {
                const int r = 4 * it + rq, grow = row0 + r;
                const uint4 u = ptx::ld_shared_v4(swz(b, r, sub));
                float4 f = make_float4(__uint_as_float(u.x), __uint_as_float(u.y), __uint_as_float(u.z),
                                       __uint_as_float(u.w));
                const bool live = grow < args.M && ncols > 0;
                if (live) {
                    float *dst = args.out_f32 + (size_t)grow * args.ldo + col;
                    if (ncols == 4) {
                        if (EPI == EPI_RESID) {
                            f.x += res[it].x;
                            f.y += res[it].y;
                            f.z += res[it].z;
                            f.w += res[it].w;
                        }
                        *reinterpret_cast<float4 *>(dst) = f;
                    } else {
                        float fe[4] = {f.x, f.y, f.z, f.w};
                        const float *rr = args.resid + (size_t)grow * args.ldr + col;
                        for (int e = 0; e < ncols; ++e) {
                            fe[e] = EPI == EPI_RESID ? fe[e] + rr[e] : fe[e];
                            dst[e] = fe[e];
                        }
                        f = make_float4(fe[0], ncols > 1 ? fe[1] : 0.f, ncols > 2 ? fe[2] : 0.f, 0.f);
                    }
                }
                if (fused_norm) {
                    if (!live) f = make_float4(0.f, 0.f, 0.f, 0.f);
                    if (live && ncols == 4)
                        *reinterpret_cast<uint2 *>(args.norm_u + (size_t)grow * args.ldo + col) =
                            make_uint2(pack_bf16(f.x * bf16lo(gw.x), f.y * __uint_as_float(gw.x & 0xFFFF0000u)),
                                       pack_bf16(f.z * bf16lo(gw.y), f.w * __uint_as_float(gw.y & 0xFFFF0000u)));
                    else if (live)
                        for (int e = 0; e < ncols; ++e)
                            args.norm_u[(size_t)grow * args.ldo + col + e] =
                                __float2bfloat16_rn((&f.x)[e] * __bfloat162float(args.norm_gain[col + e]));
                    ssacc[it] = lane_ss(f, ssacc[it]);
                }
            }
        }
        if (fused_norm) {
#pragma unroll
            for (int it = 0; it < 8; ++it) {
                const float total = row_ss(ssacc[it]);
                const int grow = row0 + 4 * it + rq;
                if (sub == 0 && grow < args.M) args.norm_ss[(size_t)(n0 / 256) * args.norm_ss_stride + grow] = total;
            }
        }
    } else if (EPI == EPI_BF16) {
#pragma unroll 1
        for (int c = 0; c < 4; ++c) {  // 64 columns a pass
            const uint32_t b = buf + (c & 1) * kStageBuf;
            uint32_t v[32], w[32];
            ptx::tmem_ld32(t_warp + c * 64, v);
            ptx::tmem_ld32(t_warp + c * 64 + 32, w);
            ptx::tmem_ld_wait();
#pragma unroll
            for (int j = 0; j < 4; ++j)
                ptx::st_shared_v4(swz(b, lane, j), pack_bf16(__uint_as_float(v[8 * j]), __uint_as_float(v[8 * j + 1])),
                                  pack_bf16(__uint_as_float(v[8 * j + 2]), __uint_as_float(v[8 * j + 3])),
                                  pack_bf16(__uint_as_float(v[8 * j + 4]), __uint_as_float(v[8 * j + 5])),
                                  pack_bf16(__uint_as_float(v[8 * j + 6]), __uint_as_float(v[8 * j + 7])));
#pragma unroll
            for (int j = 0; j < 4; ++j)
                ptx::st_shared_v4(swz(b, lane, 4 + j),
                                  pack_bf16(__uint_as_float(w[8 * j]), __uint_as_float(w[8 * j + 1])),
                                  pack_bf16(__uint_as_float(w[8 * j + 2]), __uint_as_float(w[8 * j + 3])),
                                  pack_bf16(__uint_as_float(w[8 * j + 4]), __uint_as_float(w[8 * j + 5])),
                                  pack_bf16(__uint_as_float(w[8 * j + 6]), __uint_as_float(w[8 * j + 7])));
            __syncwarp();
            const int col = n0 + c * 64 + sub * 8;
            const int ncols = min(8, args.N - col);
#pragma unroll
            for (int it = 0; it < 8; ++it) {
                const int r = 4 * it + rq, grow = row0 + r;
                const uint4 u = ptx::ld_shared_v4(swz(b, r, sub));
                if (grow >= args.M || ncols <= 0) continue;
                __nv_bfloat16 *dst = args.out_bf16 + (size_t)grow * args.ldo + col;
                if (ncols == 8)
                    *reinterpret_cast<uint4 *>(dst) = u;
                else
                    store_bf16_tail(dst, u, ncols);
            }
        }
    } else if (EPI == EPI_SWIGLU) {
        const float rs = row_norm_scale(args, row0 + lane);  // this thread's row (its TMEM lane)
#pragma unroll 1
        for (int c = 0; c < 2; ++c) {  // 128 accumulator columns (64 gate, 64 up) -> 64 outputs a pass
            const uint32_t b = buf + (c & 1) * kStageBuf;
#pragma unroll 1
            for (int h = 0; h < 2; ++h) {
                uint32_t g[32], u[32];
                ptx::tmem_ld32(t_warp + c * 128 + h * 32, g);
                ptx::tmem_ld32(t_warp + c * 128 + 64 + h * 32, u);
                ptx::tmem_ld_wait();
                uint32_t p[16];
#pragma unroll
                for (int e = 0; e < 16; ++e) {
                    const float g0 = __uint_as_float(g[2 * e]) * rs, g1 = __uint_as_float(g[2 * e + 1]) * rs;
                    p[e] = pack_bf16(silu_f(g0) * (__uint_as_float(u[2 * e]) * rs),
                                     silu_f(g1) * (__uint_as_float(u[2 * e + 1]) * rs));
                }
#pragma unroll
                for (int j = 0; j < 4; ++j) ptx::st_shared_v4(swz(b, lane, 4 * h + j), p[4 * j], p[4 * j + 1], p[4 * j + 2], p[4 * j + 3]);
            }
            __syncwarp();
            const bool live = n0 + c * 128 < args.N;
            const int col = (n0 + c * 128) / 2 + sub * 8;
#pragma unroll
            for (int it = 0; it < 8; ++it) {
                const int r = 4 * it + rq, grow = row0 + r;
                const uint4 v = ptx::ld_shared_v4(swz(b, r, sub));
                if (live && grow < args.M)
                    *reinterpret_cast<uint4 *>(args.out_bf16 + (size_t)grow * args.ldo + col) = v;
            }
        }
    }
}

// The row's RoPE table entries (cos and sin of its position), loaded before the accumulator is ready: they depend
// only on the token, so their latency hides behind the main loop and both heads of the tile use them.
struct QkvRow {
    float cs[64], sn[64];
    int pos, slot;
    float r;  // the row's RMSNorm scale (1 without the fused norm)
    bool ok;
};

__device__ __forceinline__ void qkv_preload(const GemmArgs &args, int row, bool rotates, QkvRow &R) {
    const QkvEpilogue &E = args.qkv;
    R.ok = row < args.M;
    R.r = row_norm_scale(args, row);
    R.pos = R.ok ? E.tok_pos[row] : 0;
    R.slot = R.ok ? E.tok_slot[row] : 0;
    if (rotates && R.ok) {
        const float4 *c4 = reinterpret_cast<const float4 *>(E.cos_t + (size_t)R.pos * 64);
        const float4 *s4 = reinterpret_cast<const float4 *>(E.sin_t + (size_t)R.pos * 64);
#pragma unroll
        for (int i = 0; i < 16; ++i) {
            const float4 c = c4[i], sv = s4[i];
            R.cs[4 * i] = c.x; R.cs[4 * i + 1] = c.y; R.cs[4 * i + 2] = c.z; R.cs[4 * i + 3] = c.w;
            R.sn[4 * i] = sv.x; R.sn[4 * i + 1] = sv.y; R.sn[4 * i + 2] = sv.z; R.sn[4 * i + 3] = sv.w;
        }
    }
}

// EPI_QKV for one warp's 32 rows of a pair tile (two 128-column heads): per head the sum of squares, then the RoPE
// pairs (i, i + 64) sixteen at a time, normalised, rotated and rounded to bf16 into the two staging buffers (dims
// 0..63, 64..127); the warp then writes each row's 256 bytes to its contiguous buffer and, for k and v, to the row's
// page of the KV cache.
__device__ __forceinline__ void epilogue_qkv_staged(const GemmArgs &args, uint32_t t_warp, int n0, uint32_t buf,
                                                    uint32_t norm_smem, int lane, int row, const QkvRow &R) {
    const QkvEpilogue &E = args.qkv;
#pragma unroll 1
    for (int hh = 0; hh < 2; ++hh) {
        if (n0 + hh * 128 >= args.N) break;  // warp-uniform
        const uint32_t t_head = t_warp + hh * 128;
        const int head_row = (n0 + hh * 128) / 128;
        const bool is_q = head_row < E.q_heads, is_k = !is_q && head_row < E.q_heads + E.kv_heads;
        const bool rotate = is_q || is_k;
        float r = 1.f;
        if (rotate) {
            float ss = 0.f;
#pragma unroll 1
            for (int c = 0; c < 4; ++c) {
                uint32_t u[32];
                ptx::tmem_ld32(t_head + c * 32, u);
                ptx::tmem_ld_wait();
#pragma unroll
                for (int j = 0; j < 32; ++j) {
                    const float v = __uint_as_float(u[j]) * R.r;
                    ss = fmaf(v, v, ss);
                }
            }
            r = rsqrtf(ss / 128.0f + E.eps);
        }
        __nv_bfloat16 *dst0 = nullptr, *dst1 = nullptr;
        if (R.ok) {
            if (is_q) {
                dst0 = E.q_out + ((size_t)row * E.q_heads + head_row) * 128;
            } else {
                const int kvh = is_k ? head_row - E.q_heads : head_row - E.q_heads - E.kv_heads;
                __nv_bfloat16 *flat = is_k ? E.k_out : E.v_out;  // optional contiguous copy
                dst0 = flat ? flat + ((size_t)row * E.kv_heads + kvh) * 128 : nullptr;
                const int page = E.pages[(size_t)R.slot * E.pages_per_seq + R.pos / 16];
                dst1 = E.pool + (size_t)page * E.kv_heads * 2 * 16 * 128 +
                       ((size_t)(kvh * 2 + (is_k ? 0 : 1)) * 16 + R.pos % 16) * 128;
            }
        }
        const uint32_t nwb = norm_smem + (is_q ? 0 : 256);  // the head's gains (q_norm or k_norm) in shared memory
#pragma unroll
        for (int c = 0; c < 4; ++c) {  // dims 16c..16c+15 pair with 64+16c..64+16c+15
            uint32_t lo[16], hi[16];
            ptx::tmem_ld16(t_head + c * 16, lo);
            ptx::tmem_ld16(t_head + 64 + c * 16, hi);
            ptx::tmem_ld_wait();
            float a[16], bb[16];
#pragma unroll
            for (int j = 0; j < 16; ++j) {
                a[j] = __uint_as_float(lo[j]) * R.r;
                bb[j] = __uint_as_float(hi[j]) * R.r;
            }
            if (rotate && R.ok) {
#pragma unroll
                for (int q = 0; q < 2; ++q) {
                    const uint4 l = ptx::ld_shared_v4(nwb + 32 * c + 16 * q), h = ptx::ld_shared_v4(nwb + 128 + 32 * c + 16 * q);
                    const uint32_t lw[4] = {l.x, l.y, l.z, l.w}, hw[4] = {h.x, h.y, h.z, h.w};
#pragma unroll
                    for (int e = 0; e < 8; ++e) {
                        const int j = 8 * q + e;
                        const float wl = __uint_as_float((e & 1) ? (lw[e >> 1] & 0xFFFF0000u) : (lw[e >> 1] << 16));
                        const float wh = __uint_as_float((e & 1) ? (hw[e >> 1] & 0xFFFF0000u) : (hw[e >> 1] << 16));
                        norm_rope_pair(a[j], bb[j], r, wl, wh, R.cs[16 * c + j], R.sn[16 * c + j]);
                    }
                }
            }
            uint32_t pl[8], ph[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) {
                pl[e] = pack_bf16(a[2 * e], a[2 * e + 1]);
                ph[e] = pack_bf16(bb[2 * e], bb[2 * e + 1]);
            }
            ptx::st_shared_v4(swz(buf, lane, 2 * c), pl[0], pl[1], pl[2], pl[3]);
            ptx::st_shared_v4(swz(buf, lane, 2 * c + 1), pl[4], pl[5], pl[6], pl[7]);
            ptx::st_shared_v4(swz(buf + kStageBuf, lane, 2 * c), ph[0], ph[1], ph[2], ph[3]);
            ptx::st_shared_v4(swz(buf + kStageBuf, lane, 2 * c + 1), ph[4], ph[5], ph[6], ph[7]);
        }
        __syncwarp();
        // Two rows of 256 bytes per pass: lanes 0..15 row 2 it, lanes 16..31 row 2 it + 1.
        const int ch = lane & 15, seg = ch >> 3;
#pragma unroll 4
        for (int it = 0; it < 16; ++it) {
            const int rr = 2 * it + (lane >> 4);
            const uint4 v = ptx::ld_shared_v4(swz(buf + seg * kStageBuf, rr, ch & 7));
            __nv_bfloat16 *d0 = (__nv_bfloat16 *)__shfl_sync(0xffffffffu, (unsigned long long)dst0, rr);
            __nv_bfloat16 *d1 = (__nv_bfloat16 *)__shfl_sync(0xffffffffu, (unsigned long long)dst1, rr);
            if (d0) *reinterpret_cast<uint4 *>(d0 + ch * 8) = v;
            if (d1) *reinterpret_cast<uint4 *>(d1 + ch * 8) = v;
        }
        __syncwarp();
    }
}

template <int EPI>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
    gemm_pair_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
                     GemmArgs args) {
    constexpr int S = kPairStages, HALF = 128 * BK * 2;
    constexpr int RUN = EPI == EPI_QKV ? 4 : 1;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = (uint8_t *)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    uint8_t *epi_bufs = smem + S * kPairStageBytes;
    uint64_t *full = (uint64_t *)(epi_bufs + kEpiBytes);
    uint64_t *empty = full + S;
    uint64_t *acc_full = empty + S;
    uint64_t *acc_empty = acc_full + 2;
    uint64_t *mma_done = acc_empty + 2;
    uint32_t *tmem_slot = (uint32_t *)(mma_done + 1);
    uint8_t *norm_gains = epi_bufs + kEpiBytes + 256;  // EPI_QKV: q_norm then k_norm, bf16

    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    const uint32_t rank = ptx::cluster_ctarank();
    const bool leader = rank == 0;
    const int pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;
    const int m_tiles = (args.M + 255) / 256, n_tiles = (args.N + 255) / 256;
    const int nkb = (args.K + BK - 1) / BK;
    const int total = m_tiles * n_tiles;
    uint32_t *err = args.err;

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; ++s) {
            ptx::mbar_init(&full[s], 1);
            ptx::mbar_init(&empty[s], 1);
        }
        for (int a = 0; a < 2; ++a) {
            ptx::mbar_init(&acc_full[a], 1);
            ptx::mbar_init(&acc_empty[a], 8);  // four epilogue warps in each CTA
        }
        ptx::mbar_init(mma_done, 1);
        ptx::fence_barrier_init();
        ptx::prefetch_tmap(&tmap_a);
        ptx::prefetch_tmap(&tmap_b);
    }
    if (warp == 1) {
        ptx::tmem_alloc_pair(tmem_slot, 512);
        ptx::tmem_relinquish_pair();
    }
    ptx::tc_fence_before();
    ptx::cluster_sync();  // barriers of both CTAs initialised before any remote arrive or load completes on them
    ptx::tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    ptx::griddep_launch();

    // Tile t -> (m block, n block) of 256 x 256; n fastest.
    if (warp == 0) {
        if (ptx::elect_one()) {
            uint32_t it = 0;
            bool ok = true;
            int pre = 0;
            const int row_a = (int)rank * 128, row_b = (int)rank * 128;
            const int t0 = pair_tile<RUN>(pair, npairs, 0);
            if (args.independent && t0 < total) {
                const int mb = t0 / n_tiles, nb = t0 % n_tiles;
                pre = min(S, nkb);
                for (int j = 0; j < pre; ++j) {
                    uint8_t *sa = smem + j * kPairStageBytes;
                    if (leader) ptx::mbar_arrive_expect_tx(&full[j], 2 * kPairStageBytes);
                    const uint32_t bar = ptx::mapa(&full[j], 0);
                    if (args.independent == 1)
                        ptx::tma_load_2d_pair(sa, &tmap_a, bar, j * BK, mb * 256 + row_a);
                    else
                        ptx::tma_load_2d_pair(sa + HALF, &tmap_b, bar, j * BK, nb * 256 + row_b);
                }
            }
            ptx::griddep_wait();
            for (int i = 0; ok; ++i) {
                const int t = pair_tile<RUN>(pair, npairs, i);
                if (t >= total) break;
                const int mb = t / n_tiles, nb = t % n_tiles;
                for (int kb = 0; kb < nkb; ++kb, ++it) {
                    const int s = it % S;
                    const uint32_t ph = (it / S) & 1;
                    uint8_t *sa = smem + s * kPairStageBytes;
                    uint8_t *sb = sa + HALF;
                    const uint32_t bar = ptx::mapa(&full[s], 0);
                    if ((int)it < pre) {
                        if (args.independent == 1)
                            ptx::tma_load_2d_pair(sb, &tmap_b, bar, kb * BK, nb * 256 + row_b);
                        else
                            ptx::tma_load_2d_pair(sa, &tmap_a, bar, kb * BK, mb * 256 + row_a);
                        continue;
                    }
                    if (!ptx::mbar_wait(&empty[s], ph ^ 1, err, 0x1011)) {
                        ok = false;
                        break;
                    }
                    if (leader) ptx::mbar_arrive_expect_tx(&full[s], 2 * kPairStageBytes);
                    ptx::tma_load_2d_pair(sa, &tmap_a, bar, kb * BK, mb * 256 + row_a);
                    ptx::tma_load_2d_pair(sb, &tmap_b, bar, kb * BK, nb * 256 + row_b);
                }
            }
            // Both CTAs' loads complete on the even CTA's barriers: it waits for the last stages to land before the
            // closing cluster barrier, which keeps either CTA from exiting with a copy in flight.
            if (leader) {
                uint32_t first = it > (uint32_t)S ? it - S : 0;
                for (uint32_t j = first; j < it; ++j) ptx::mbar_wait(&full[j % S], (j / S) & 1, err, 0x1012);
            }
        }
    } else if (warp == 1) {
        if (leader && ptx::elect_one()) {
            constexpr uint32_t idesc = ptx::idesc_bf16_f32(256, 256);
            uint32_t it = 0, local = 0;
            bool ok = true;
            for (int i = 0; ok; ++i, ++local) {
                if (pair_tile<RUN>(pair, npairs, i) >= total) break;
                const int a = local & 1;
                if (!ptx::mbar_wait(&acc_empty[a], ((local >> 1) & 1) ^ 1, err, 0x1013)) break;
                ptx::tc_fence_after();
                const uint32_t d_tmem = tmem_base + a * 256;
                for (int kb = 0; kb < nkb; ++kb, ++it) {
                    const int s = it % S;
                    if (!ptx::mbar_wait(&full[s], (it / S) & 1, err, 0x1014)) {
                        ok = false;
                        break;
                    }
                    ptx::tc_fence_after();
                    const uint32_t sa = ptx::smem_u32(smem + s * kPairStageBytes), sb = sa + HALF;
#pragma unroll
                    for (int k = 0; k < BK / UMMA_K; ++k)
                        ptx::mma_bf16_pair(d_tmem, ptx::sw128_kmajor_desc(sa + k * UMMA_K * 2),
                                           ptx::sw128_kmajor_desc(sb + k * UMMA_K * 2), idesc,
                                           (kb > 0 || k > 0) ? 1u : 0u);
                    ptx::mma_commit_pair(&empty[s], 0x3);
                }
                ptx::mma_commit_pair(&acc_full[a], 0x3);
            }
            ptx::mma_commit_pair(mma_done, 0x1);
            ptx::mbar_wait(mma_done, 0, err, 0x1015);
        }
    } else {
        ptx::griddep_wait();
        const int q = warp & 3;
        uint32_t local = 0;
        const uint32_t rel0 = ptx::mapa(&acc_empty[0], 0), rel1 = ptx::mapa(&acc_empty[1], 0);
        const uint32_t buf = ptx::smem_u32(epi_bufs + (warp - 2) * 2 * kStageBuf);
        if constexpr (EPI == EPI_QKV) {
            if (warp == 2) {  // stage the gains once; the four epilogue warps meet on named barrier 1
                const uint4 *src = reinterpret_cast<const uint4 *>(lane < 16 ? args.qkv.q_norm : args.qkv.k_norm);
                reinterpret_cast<uint4 *>(norm_gains)[lane] = src[lane & 15];
            }
            asm volatile("bar.sync 1, 128;" ::: "memory");
        }
        QkvRow R;
        int r_mb = -1;
        bool r_table = false;
        for (int i = 0;; ++i, ++local) {
            const int t = pair_tile<RUN>(pair, npairs, i);
            if (t >= total) break;
            const int mb = t / n_tiles, nb = t % n_tiles;
            const int a = local & 1;
            const int row0 = mb * 256 + (int)rank * 128 + q * 32;
            if (EPI == EPI_RESID && row0 + lane < args.M) {
                const uint32_t bytes = (uint32_t)(min(256, args.N - nb * 256) * 4) & ~15u;
                if (bytes) ptx::prefetch_l2_bulk(args.resid + (size_t)(row0 + lane) * args.ldr + nb * 256, bytes);
            }
            if constexpr (EPI == EPI_QKV) {
                // a row's position, slot and RoPE entries carry over while the run stays on the same rows
                const bool rotates = nb * 256 < (args.qkv.q_heads + args.qkv.kv_heads) * 128;
                if (mb != r_mb || (rotates && !r_table)) {
                    qkv_preload(args, row0 + lane, rotates, R);
                    r_mb = mb;
                    r_table = rotates;
                }
                if (!ptx::mbar_wait(&acc_full[a], (local >> 1) & 1, err, 0x1016)) break;
                ptx::tc_fence_after();
                const uint32_t t_warp = tmem_base + a * 256 + ((uint32_t)(q * 32) << 16);
                epilogue_qkv_staged(args, t_warp, nb * 256, buf, ptx::smem_u32(norm_gains), lane, row0 + lane, R);
            } else {
                if (!ptx::mbar_wait(&acc_full[a], (local >> 1) & 1, err, 0x1016)) break;
                ptx::tc_fence_after();
                const uint32_t t_warp = tmem_base + a * 256 + ((uint32_t)(q * 32) << 16);
                epilogue_staged<EPI>(args, t_warp, row0, nb * 256, buf, lane);
            }
            ptx::tc_fence_before();
            __syncwarp();
            if (lane == 0) ptx::mbar_arrive_cluster(a ? rel1 : rel0);
        }
    }
    ptx::tc_fence_before();
    ptx::cluster_sync();  // no CTA frees TMEM or exits while its partner's MMAs or arrivals may still reach it
    ptx::tc_fence_after();
    if (warp == 1) ptx::tmem_dealloc_pair(tmem_base, 512);
}

// ---- host side --------------------------------------------------------------------------------------------------

// The driver's tensor-map encoder, resolved at run time through the runtime (so the library has no link-time
// dependency on libcuda and still loads on a machine without a GPU driver).
typedef CUresult (*EncodeTiledFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                  const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_tiled() {
    // resolved once per process (a function-local static: thread-safe initialisation)
    static const EncodeTiledFn fn = [] {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            return (EncodeTiledFn)p;
        return (EncodeTiledFn) nullptr;
    }();
    return fn;
}

bool make_tmap_2d(CUtensorMap *map, const void *ptr, uint64_t rows, uint64_t cols, uint32_t box_rows) {
    // bf16 [rows, cols] row-major: dim 0 = cols (inner), dim 1 = rows. Box {64, box_rows}, 128-byte swizzle.
    EncodeTiledFn enc = encode_tiled();
    if (!enc) return false;
    cuuint64_t dims[2] = {cols, rows};
    cuuint64_t strides[1] = {cols * 2};
    cuuint32_t box[2] = {64, box_rows};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void *>(ptr), dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

template <int BN, int EPI>
cudaError_t launch_bn(const CUtensorMap &ta, const CUtensorMap &tb, const GemmArgs &args, int sms,
                      cudaStream_t stream) {
    using C = Cfg<BN>;
    static SmemOptIn opt;
    if (cudaError_t e = opt.set((const void *)gemm_kernel<BN, EPI>, C::SMEM_BYTES)) return e;
    int m_tiles = (args.M + BM - 1) / BM, n_tiles = (args.N + BN - 1) / BN;
    int total = m_tiles * n_tiles * args.splits;
    int grid = total < sms ? total : sms;
    return launch_kernel(gemm_kernel<BN, EPI>, dim3(grid), dim3(kThreads), C::SMEM_BYTES, stream, ta, tb, args);
}

// One cluster of two CTAs per pair of SMs, persistent over the 256 x 256 tiles.
template <int EPI>
cudaError_t launch_pair(const CUtensorMap &ta, const CUtensorMap &tb, const GemmArgs &args, int sms,
                        cudaStream_t stream) {
    static SmemOptIn opt;
    if (cudaError_t e = opt.set((const void *)gemm_pair_kernel<EPI>, kPairSmem)) return e;
    const int total = ((args.M + 255) / 256) * ((args.N + 255) / 256);
    const int pairs = total < sms / 2 ? total : sms / 2;
    return launch_kernel(gemm_pair_kernel<EPI>, dim3(2 * pairs), dim3(kThreads), kPairSmem, stream, ta, tb, args);
}

template <int BN>
cudaError_t launch_epi(const CUtensorMap &ta, const CUtensorMap &tb, const GemmArgs &args, int sms,
                       cudaStream_t stream) {
    switch (args.epi) {
        case EPI_F32: return launch_bn<BN, EPI_F32>(ta, tb, args, sms, stream);
        case EPI_RESID: return launch_bn<BN, EPI_RESID>(ta, tb, args, sms, stream);
        case EPI_SWIGLU: return launch_bn<BN, EPI_SWIGLU>(ta, tb, args, sms, stream);
        case EPI_PARTIAL: return launch_bn<BN, EPI_PARTIAL>(ta, tb, args, sms, stream);
        case EPI_BF16: return launch_bn<BN, EPI_BF16>(ta, tb, args, sms, stream);
        case EPI_QKV:
            if (BN >= 128) return launch_bn<BN, EPI_QKV>(ta, tb, args, sms, stream);
            return cudaErrorInvalidValue;
    }
    return cudaErrorInvalidValue;
}

}  // namespace

namespace {

// One warp per 32 rows and 256-column group: the rows' u = bf16(gain * x) and their group sums of squares, with the
// lanes laid over the columns as the staged residual epilogue lays them (lane = 8 rq + sub: rows 4 it + rq, columns
// 32 c + 4 sub of pass c), so the sums come out in the same order and bits.
__global__ void __launch_bounds__(256) pair_prep_kernel(const float *x, int T, int hidden, const __nv_bfloat16 *gain,
                                                        __nv_bfloat16 *u, float *ss, size_t ss_stride) {
    ptx::griddep_wait();
    ptx::griddep_launch();
    const int lane = threadIdx.x & 31, sub = lane & 7, rq = lane >> 3;
    const int groups = (hidden + 255) / 256;
    const int wg = blockIdx.x * 8 + (threadIdx.x >> 5);
    const int row0 = (wg / groups) * 32, g = wg % groups;
    if (row0 >= T) return;  // whole warp
    float ssacc[8];
#pragma unroll
    for (int it = 0; it < 8; ++it) ssacc[it] = 0.f;
#pragma unroll 1
    for (int c = 0; c < 8; ++c) {
        const int col = g * 256 + c * 32 + sub * 4;
        const int ncols = min(4, hidden - col);
#pragma unroll
        for (int it = 0; it < 8; ++it) {
            const int row = row0 + 4 * it + rq;
            float4 f = make_float4(0.f, 0.f, 0.f, 0.f);
            if (row < T && ncols > 0) {
                const float *xr = x + (size_t)row * hidden + col;
                if (ncols == 4) {
                    f = *reinterpret_cast<const float4 *>(xr);
                    const uint2 gw = *reinterpret_cast<const uint2 *>(gain + col);
                    *reinterpret_cast<uint2 *>(u + (size_t)row * hidden + col) =
                        make_uint2(pack_bf16(f.x * bf16lo(gw.x), f.y * __uint_as_float(gw.x & 0xFFFF0000u)),
                                   pack_bf16(f.z * bf16lo(gw.y), f.w * __uint_as_float(gw.y & 0xFFFF0000u)));
                } else {
                    float fe[4] = {0.f, 0.f, 0.f, 0.f};
                    for (int e = 0; e < ncols; ++e) {
                        fe[e] = xr[e];
                        u[(size_t)row * hidden + col + e] = __float2bfloat16_rn(fe[e] * __bfloat162float(gain[col + e]));
                    }
                    f = make_float4(fe[0], fe[1], fe[2], 0.f);
                }
            }
            ssacc[it] = lane_ss(f, ssacc[it]);
        }
    }
#pragma unroll
    for (int it = 0; it < 8; ++it) {
        const float total = row_ss(ssacc[it]);
        const int row = row0 + 4 * it + rq;
        if (sub == 0 && row < T) ss[(size_t)g * ss_stride + row] = total;
    }
}

}  // namespace

cudaError_t launch_pair_prep(const float *x, int T, int hidden, const __nv_bfloat16 *gain, __nv_bfloat16 *u, float *ss,
                             size_t ss_stride, cudaStream_t st) {
    if (T < 1 || hidden < 4 || hidden % 4 || !x || !gain || !u || !ss) return cudaErrorInvalidValue;
    const int warps = (T + 31) / 32 * ((hidden + 255) / 256);
    return launch_kernel(pair_prep_kernel, dim3((warps + 7) / 8), dim3(256), 0, st, x, T, hidden, gain, u, ss,
                         ss_stride);
}

bool gemm_tmap_2d(CUtensorMap *map, const void *ptr, uint64_t rows, uint64_t cols, uint32_t box_rows) {
    return make_tmap_2d(map, ptr, rows, cols, box_rows);
}

const char *gemm_check(const GemmArgs &a) {
    // tile and k-block counts are int32 ((K + 63) / 64 and the like): a bound well below INT_MAX
    if (a.M < 1 || a.N < 1 || a.K < 1 || a.M > (1 << 30) || a.N > (1 << 30) || a.K > (1 << 30))
        return "M, N and K must be 1 .. 2^30";
    if (a.K % 8) return "K must be a multiple of 8 (16-byte rows for TMA)";
    if (((uintptr_t)a.A & 15) || ((uintptr_t)a.B & 15)) return "A and B must be 16-byte aligned";
    if (a.bn != 64 && a.bn != 128 && a.bn != 256) return "bn must be 64, 128 or 256";
    if (a.splits < 1 || a.kb_per_split < 1) return "splits and kb_per_split must be positive";
    int nkb = (a.K + BK - 1) / BK;
    if ((long)a.splits * a.kb_per_split < nkb) return "splits * kb_per_split must cover K";
    if (a.epi == EPI_SWIGLU && (a.N % 128 || a.bn < 128)) return "SwiGLU needs N % 128 == 0 and bn >= 128";
    if (a.epi == EPI_SWIGLU && (a.ldo % 8 || ((uintptr_t)a.out_bf16 & 15))) return "SwiGLU output needs 16-byte rows";
    if (a.epi != EPI_PARTIAL && a.splits != 1) return "split-K writes partials only (EPI_PARTIAL)";
    if ((a.epi == EPI_F32 || a.epi == EPI_RESID) && (a.ldo % 4 || ((uintptr_t)a.out_f32 & 15)))
        return "fp32 output needs 16-byte aligned rows";
    if (a.epi == EPI_RESID && (a.ldr % 4 || ((uintptr_t)a.resid & 15))) return "resid needs 16-byte aligned rows";
    if (a.epi == EPI_BF16 && (a.ldo % 8 || ((uintptr_t)a.out_bf16 & 15))) return "bf16 output needs 16-byte rows";
    if (a.epi == EPI_PARTIAL && !a.partial) return "partial output missing";
    if (a.epi == EPI_QKV) {
        const QkvEpilogue &q = a.qkv;
        if (a.bn < 128 || a.N % 128 || a.N != (q.q_heads + 2 * q.kv_heads) * 128)
            return "the q/k/v epilogue needs bn >= 128 and N = (q_heads + 2 kv_heads) * 128";
        if (!q.q_out || !q.pool || !q.pages || !q.q_norm || !q.k_norm || !q.cos_t || !q.sin_t || !q.tok_slot ||
            !q.tok_pos)
            return "the q/k/v epilogue is missing a pointer";
        if (((uintptr_t)q.q_out | (uintptr_t)q.k_out | (uintptr_t)q.v_out | (uintptr_t)q.pool) & 15)
            return "the q/k/v epilogue outputs must be 16-byte aligned";
    }
    if (a.norm_u && (a.epi != EPI_RESID || a.cta_pair != 2 || !a.norm_gain || !a.norm_ss ||
                     a.norm_ss_stride < (size_t)a.M || ((uintptr_t)a.norm_u & 7) || ((uintptr_t)a.norm_gain & 7)))
        return "the fused norm's outputs need EPI_RESID on CTA pairs, a gain, sums and 8-byte aligned u";
    if (a.row_ss && ((a.epi != EPI_SWIGLU && a.epi != EPI_QKV) || a.cta_pair != 2 || a.row_nss < 1 ||
                     a.row_hidden < 1 || a.row_ss_stride < (size_t)a.M))
        return "a row norm scale needs EPI_SWIGLU or EPI_QKV on CTA pairs and valid sums";
    if (a.cta_pair < 0 || a.cta_pair > 2) return "cta_pair must be 0, 1 or 2";
    if (a.cta_pair == 2 && (a.bn != 256 || a.splits != 1 || a.epi == EPI_PARTIAL))
        return "CTA pairs need bn 256, one split and a non-partial epilogue";
    if (!a.err) return "error word missing";
    return nullptr;
}

bool gemm_uses_pair(const GemmArgs &a) {
    if (a.cta_pair == 1) return false;
    if (a.cta_pair == 2) return true;
    return a.bn == 256 && a.splits == 1 && a.epi != EPI_PARTIAL && a.M >= 1024;
}

cudaError_t gemm_launch(const GemmArgs &args, int sms, cudaStream_t stream) {
    CUtensorMap ta, tb;
    const bool pair = gemm_uses_pair(args);
    if (!make_tmap_2d(&ta, args.A, args.M, args.K, BM)) return cudaErrorInvalidValue;
    if (!make_tmap_2d(&tb, args.B, args.N, args.K, pair ? 128 : args.bn)) return cudaErrorInvalidValue;
    if (pair) {
        switch (args.epi) {
            case EPI_F32: return launch_pair<EPI_F32>(ta, tb, args, sms, stream);
            case EPI_RESID: return launch_pair<EPI_RESID>(ta, tb, args, sms, stream);
            case EPI_SWIGLU: return launch_pair<EPI_SWIGLU>(ta, tb, args, sms, stream);
            case EPI_BF16: return launch_pair<EPI_BF16>(ta, tb, args, sms, stream);
            case EPI_QKV: return launch_pair<EPI_QKV>(ta, tb, args, sms, stream);
        }
        return cudaErrorInvalidValue;
    }
    switch (args.bn) {
        case 64: return launch_epi<64>(ta, tb, args, sms, stream);
        case 128: return launch_epi<128>(ta, tb, args, sms, stream);
        case 256: return launch_epi<256>(ta, tb, args, sms, stream);
    }
    return cudaErrorInvalidValue;
}

}  // namespace lrm
