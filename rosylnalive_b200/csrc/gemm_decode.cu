// gemm_decode.cu -- the decode step's weight GEMMs with their consumers fused, on the tcgen05 tensor cores (sm_100a).
//
// A decode step multiplies each weight matrix by the step's few tokens: Y[m][t] = sum_k W[m][k] B[t][k], W the
// weights [M, K] (bf16, the 128-row tensor-core tile) and B the tokens' activations [N, K] (N = 64 a tile: the MMA's
// N). The work is far too small to fill 148 SMs with whole tiles, so S CTAs split K for each output tile; they form
// one thread-block cluster, and instead of writing fp32 partials for another kernel to add up, they reduce through
// distributed shared memory:
//   warp 0      TMA producer: the CTA's weight k-blocks are requested before the kernel waits for the previous one
//               (programmatic dependent launch; the weights are written by no kernel), L2 evict-first (each weight
//               byte is read once a step), then the token k-blocks;
//   warp 1      TMEM allocation (64 columns) and one thread issuing tcgen05.mma M=128, N=64, K=16;
//   warps 2..5  the epilogue: each thread moves its accumulator row (TMEM lane) into the CTA's shared memory as
//               [token][row], the cluster synchronises, and every CTA then sums one share of the tile's tokens over
//               the S CTAs' shared memory (ld.shared::cluster, in split order, so the result does not depend on
//               timing) and finishes those tokens:
//     DEC_QKV     per head row: the RMSNorm scale of the tokens' input, then QK-RMSNorm and RoPE for q and k; q to
//                 its buffer, k and v into the paged KV cache;
//     DEC_SWIGLU  the norm scale, then silu(gate) * up of the tile's 64 gate/up row pairs;
//     DEC_RESID   the residual add x += y, then the next norm's inputs: u = bf16(gain * x) for the next GEMM and the
//                 per-128-column sums of squares of x (the norm's scale is applied by the consumer, which is linear
//                 in each token).
// No TMA multicast is used; the cluster exchanges data only through shared::cluster loads. Every mbarrier wait is
// bounded (ptx::mbar_wait) and every thread reaches both cluster barriers on every path, so a wait that gives up
// reports a code in the error word and the kernel still returns.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include <string.h>

#include <string>

#include "../../include/lrm_cuda.h"
#include "gemm.h"
#include "internal.h"
#include "ptx.cuh"
#include "qwen.h"

namespace lrm {
namespace {

constexpr int kBM = 128, kBN = 64, kBK = 64, kUK = 16;
constexpr int kStages = 4;  // 98 KiB of shared memory: two CTAs an SM, so the next GEMM's CTAs are resident early
constexpr int kABytes = kBM * kBK * 2;  // 16 KiB of weights a stage
constexpr int kBBytes = kBN * kBK * 2;  // 8 KiB of tokens
constexpr int kStageBytes = kABytes + kBBytes;
constexpr int kSmem = kStages * kStageBytes + 1024 /*align*/ + 256 /*barriers*/;
constexpr int kThreads = 192;
constexpr int kCtasPerSm = 2;
constexpr int kMaxSplits = 16;  // clusters above 8 CTAs are a non-portable size, opted into per kernel
static_assert(kBN * kBM * 4 <= kStages * kStageBytes, "the staged accumulator reuses the stage ring");
constexpr unsigned FULL = 0xFFFFFFFFu;

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(FULL, v, o);
    return v;
}

__device__ __forceinline__ uint2 pack4(float a, float b, float c, float d) {
    __nv_bfloat162 lo = __floats2bfloat162_rn(a, b), hi = __floats2bfloat162_rn(c, d);
    return make_uint2(*reinterpret_cast<uint32_t *>(&lo), *reinterpret_cast<uint32_t *>(&hi));
}

__device__ __forceinline__ float bflo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bfhi(uint32_t w) { return __uint_as_float(w & 0xFFFF0000u); }

// The sum of squares of a 128-column group held as one float4 a lane (lane l: columns 4l..4l+3): each lane's four in
// order, then a butterfly over the warp, which leaves the same bits in every lane. DEC_RESID and the prep kernel both
// use it, so a pipeline stage that resumes from the residual computes the same norm inputs as the unsplit engine.
__device__ __forceinline__ float group_ss(float4 v) {
    float s = v.x * v.x;
    s = fmaf(v.y, v.y, s);
    s = fmaf(v.z, v.z, s);
    s = fmaf(v.w, v.w, s);
    return warp_sum(s);
}

// u = bf16(gain * x) for four consecutive columns starting at gain[m] (8-byte aligned).
__device__ __forceinline__ uint2 gained(float4 x, const __nv_bfloat16 *gain) {
    const uint2 g = *reinterpret_cast<const uint2 *>(gain);
    return pack4(x.x * bflo(g.x), x.y * bfhi(g.x), x.z * bflo(g.y), x.w * bfhi(g.y));
}

__device__ __forceinline__ float4 scale4(float4 v, float r) { return make_float4(v.x * r, v.y * r, v.z * r, v.w * r); }

// Tokens one epilogue warp finishes: the CTA's share of a 64-token tile (64 / S, rounded up) over four warps.
template <int S>
constexpr int tokens_per_warp() {
    return ((kBN + S - 1) / S + 3) / 4;
}

// What an epilogue warp needs for NT of its tokens besides the GEMM's result. None of it depends on the result, so
// it is loaded while the tensor cores work, and only the cluster reduction is left once the accumulators are ready.
template <int NT>
struct TokenInputs {
    int tok[NT];       // the token's index in the step, -1 when the warp has no such token
    int tl[NT];        // its index in the tile
    float4 xv[NT];     // DEC_RESID: the residual x[t] at the lane's four rows
    float r[NT];       // DEC_SWIGLU, DEC_QKV: the token's RMSNorm scale
    int pos[NT];       // DEC_QKV: the token's position
    int page[NT];      // DEC_QKV (k, v): the cache page the position lies in
    float4 cs[NT], sn[NT];  // DEC_QKV (q, k): the RoPE row at the position, the lane's four pairs
    uint2 g;           // DEC_RESID: the next norm's gains at the lane's rows; DEC_QKV: the q/k norm's
};

// Warp w takes tokens t0 + w, t0 + w + 4, ... of this CTA's share [t0, t1) of tile (mt, nt); this loads the NT of
// them from the warp's i0-th on. Every load is issued for all NT tokens before any result is used.
// PART 1 is what no kernel of a decode step after its first writes (the q/k/v tokens' positions, pages, RoPE rows
// and norm gains), which may load before the kernel waits on the previous one; PART 2 is the rest, loaded after the
// wait (and after PART 1); PART 3 both.
template <int EPI, int S, int NT, int PART = 3>
__device__ __forceinline__ void load_inputs(const DecodeGemmArgs &a, TokenInputs<NT> &in, int split, int mt, int nt,
                                            int w, int lane, int i0) {
    const int t0 = split * kBN / S, t1 = (split + 1) * kBN / S;
    if (PART & 1) {
#pragma unroll
        for (int i = 0; i < NT; ++i) {
            in.tl[i] = t0 + w + 4 * (i0 + i);
            in.tok[i] = (in.tl[i] < t1 && nt * kBN + in.tl[i] < a.N) ? nt * kBN + in.tl[i] : -1;
        }
    }
    const int m = mt * kBM + 4 * lane;
    if (EPI == DEC_RESID) {
        if (!(PART & 2)) return;
#pragma unroll
        for (int i = 0; i < NT; ++i)
            if (in.tok[i] >= 0) in.xv[i] = *reinterpret_cast<const float4 *>(a.x + (size_t)in.tok[i] * a.M + m);
        in.g = a.gain ? __ldg(reinterpret_cast<const uint2 *>(a.gain + m)) : make_uint2(0, 0);
        return;
    }
    if (EPI == DEC_QKV && (PART & 1)) {
        const QkvEpilogue &E = a.qkv;
#pragma unroll
        for (int i = 0; i < NT; ++i) in.pos[i] = in.tok[i] >= 0 ? __ldg(E.tok_pos + in.tok[i]) : 0;
        const int hr = mt;
        const bool is_q = hr < E.q_heads, is_k = !is_q && hr < E.q_heads + E.kv_heads;
        if (!is_q) {
#pragma unroll
            for (int i = 0; i < NT; ++i) in.page[i] = in.tok[i] >= 0 ? __ldg(E.tok_slot + in.tok[i]) : 0;
#pragma unroll
            for (int i = 0; i < NT; ++i)
                in.page[i] =
                    in.tok[i] >= 0 ? __ldg(E.pages + (size_t)in.page[i] * E.pages_per_seq + in.pos[i] / kPageTokens) : 0;
        }
        if (is_q || is_k) {
            in.g = __ldg(reinterpret_cast<const uint2 *>((is_q ? E.q_norm : E.k_norm) + 4 * lane));
            const int ci = 4 * (lane & 15);
#pragma unroll
            for (int i = 0; i < NT; ++i) {
                if (in.tok[i] < 0) continue;
                in.cs[i] = __ldg(reinterpret_cast<const float4 *>(E.cos_t + (size_t)in.pos[i] * 64 + ci));
                in.sn[i] = __ldg(reinterpret_cast<const float4 *>(E.sin_t + (size_t)in.pos[i] * 64 + ci));
            }
        }
    }
    // The RMSNorm scale of each token's input: lane g holds the sums of squares of column groups g, g + 32, ...
    // (added in that order), then a butterfly over the warp, which leaves the same bits in every lane.
    if (PART & 2) {
        float part[NT];
#pragma unroll
        for (int i = 0; i < NT; ++i) {
            part[i] = 0.f;
            if (in.tok[i] >= 0 && a.ss)
                for (int gi = lane; gi < a.nss; gi += 32) part[i] += __ldg(a.ss + (size_t)gi * a.ss_stride + in.tok[i]);
        }
#pragma unroll
        for (int i = 0; i < NT; ++i) in.r[i] = a.ss ? rsqrtf(warp_sum(part[i]) / a.hidden + a.eps) : 1.f;
    }
}

// The cluster reduction of the same NT tokens (the S CTAs' staged accumulators, remote loads all in flight at
// once, summed in split order) and the epilogue, lane l holding rows 4l..4l+3 of each token.
template <int S, int NT>
__device__ __forceinline__ void reduce_tokens(const TokenInputs<NT> &in, const float *stg, int lane, float4 (&y)[NT]) {
    {
        float4 z[NT][S];
#pragma unroll
        for (int i = 0; i < NT; ++i) {
            if (in.tok[i] < 0) continue;
            const float *src = stg + in.tl[i] * kBM + 4 * lane;
#pragma unroll
            for (int s = 0; s < S; ++s) z[i][s] = ptx::ld_cluster_f4(ptx::mapa(src, s));
        }
#pragma unroll
        for (int i = 0; i < NT; ++i) {
            y[i] = z[i][0];
#pragma unroll
            for (int s = 1; s < S; ++s) {  // split order
                y[i].x += z[i][s].x;
                y[i].y += z[i][s].y;
                y[i].z += z[i][s].z;
                y[i].w += z[i][s].w;
            }
        }
    }
}

template <int EPI, int NT>
__device__ __forceinline__ void finish_tokens(const DecodeGemmArgs &a, const TokenInputs<NT> &in,
                                              const float4 (&y)[NT], int mt, int lane) {
    const int m = mt * kBM + 4 * lane;
    if (EPI == DEC_RESID) {
#pragma unroll
        for (int i = 0; i < NT; ++i) {
            if (in.tok[i] < 0) continue;
            float4 x = in.xv[i];
            x.x += y[i].x;
            x.y += y[i].y;
            x.z += y[i].z;
            x.w += y[i].w;
            *reinterpret_cast<float4 *>(a.x + (size_t)in.tok[i] * a.M + m) = x;
            if (a.gain) {
                *reinterpret_cast<uint2 *>(a.u + (size_t)in.tok[i] * a.M + m) =
                    pack4(x.x * bflo(in.g.x), x.y * bfhi(in.g.x), x.z * bflo(in.g.y), x.w * bfhi(in.g.y));
                const float ss = group_ss(x);
                if (lane == 0) a.ss_out[(size_t)mt * a.ss_stride + in.tok[i]] = ss;
            }
        }
    } else if (EPI == DEC_SWIGLU) {
#pragma unroll
        for (int i = 0; i < NT; ++i) {
            if (in.tok[i] < 0) continue;
            const float4 v = scale4(y[i], in.r[i]);
            const float u0 = __shfl_xor_sync(FULL, v.x, 16), u1 = __shfl_xor_sync(FULL, v.y, 16),
                        u2 = __shfl_xor_sync(FULL, v.z, 16), u3 = __shfl_xor_sync(FULL, v.w, 16);
            if (lane < 16) {  // gate rows 4l..4l+3 here, their up rows 64 + 4l.. in lane l + 16
                const float s0 = __fdividef(v.x, 1.0f + __expf(-v.x)), s1 = __fdividef(v.y, 1.0f + __expf(-v.y)),
                            s2 = __fdividef(v.z, 1.0f + __expf(-v.z)), s3 = __fdividef(v.w, 1.0f + __expf(-v.w));
                *reinterpret_cast<uint2 *>(a.act + (size_t)in.tok[i] * a.ld_act + mt * 64 + 4 * lane) =
                    pack4(s0 * u0, s1 * u1, s2 * u2, s3 * u3);
            }
        }
    } else {  // DEC_QKV: the tile is head row mt (q heads, then k heads, then v heads)
        const QkvEpilogue &E = a.qkv;
        const int hr = mt;
        const bool is_q = hr < E.q_heads, is_k = !is_q && hr < E.q_heads + E.kv_heads;
        const int kvh = is_k ? hr - E.q_heads : hr - E.q_heads - E.kv_heads;
        const float w0 = bflo(in.g.x), w1 = bfhi(in.g.x), w2 = bflo(in.g.y), w3 = bfhi(in.g.y);
#pragma unroll
        for (int i = 0; i < NT; ++i) {
            if (in.tok[i] < 0) continue;
            float4 v = scale4(y[i], in.r[i]);
            if (is_q || is_k) {
                const float ss = warp_sum(v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w);
                const float rr = rsqrtf(ss / kHeadDim + E.eps);
                const float y0 = v.x * rr * w0, y1 = v.y * rr * w1, y2 = v.z * rr * w2, y3 = v.w * rr * w3;
                // NeoX rotate-half: dim i pairs with i + 64, held by lane l ^ 16
                const float o0 = __shfl_xor_sync(FULL, y0, 16), o1 = __shfl_xor_sync(FULL, y1, 16),
                            o2 = __shfl_xor_sync(FULL, y2, 16), o3 = __shfl_xor_sync(FULL, y3, 16);
                const float4 c = in.cs[i], s = in.sn[i];
                if (lane < 16)  // y[i] = x[i] c - x[i+64] s
                    v = make_float4(y0 * c.x - o0 * s.x, y1 * c.y - o1 * s.y, y2 * c.z - o2 * s.z,
                                    y3 * c.w - o3 * s.w);
                else  // y[i+64] = x[i+64] c + x[i] s
                    v = make_float4(y0 * c.x + o0 * s.x, y1 * c.y + o1 * s.y, y2 * c.z + o2 * s.z,
                                    y3 * c.w + o3 * s.w);
            }
            const uint2 packed = pack4(v.x, v.y, v.z, v.w);
            if (is_q) {
                *reinterpret_cast<uint2 *>(E.q_out + ((size_t)in.tok[i] * E.q_heads + hr) * kHeadDim + 4 * lane) =
                    packed;
            } else {
                __nv_bfloat16 *dst = E.pool + (size_t)in.page[i] * kv_page_elems(E.kv_heads) +
                                     ((size_t)(kvh * 2 + (is_k ? 0 : 1)) * kPageTokens + in.pos[i] % kPageTokens) *
                                         kHeadDim +
                                     4 * lane;
                *reinterpret_cast<uint2 *>(dst) = packed;
            }
        }
    }
}

// grid (S x m tiles, n tiles), clusters of S CTAs along x: CTA (split, mt, nt) = blockIdx (mt S + split, nt), its
// cluster rank = split.
template <int EPI, int S>
__global__ void __launch_bounds__(kThreads, kCtasPerSm)
    gemm_dec_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
                    const DecodeGemmArgs args) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = (uint8_t *)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    uint64_t *full = (uint64_t *)(smem + kStages * kStageBytes);
    uint64_t *empty = full + kStages;
    uint64_t *acc_full = empty + kStages;
    uint32_t *tmem_slot = (uint32_t *)(acc_full + 1);
    float *stg = reinterpret_cast<float *>(smem);  // [64 tokens][128 rows] once the MMAs are done

    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    const int split = (int)blockIdx.x % S, mt = (int)blockIdx.x / S, nt = (int)blockIdx.y;
    const int nkb = (args.K + kBK - 1) / kBK;
    const int k0 = split * args.kb_per_split, k1 = min(nkb, k0 + args.kb_per_split);
    const int nk = max(0, k1 - k0);
    uint32_t *err = args.err;
    constexpr int NT = tokens_per_warp<S>();
    constexpr int CH = NT < 4 ? NT : 4;
    TokenInputs<CH> in;  // the epilogue warps' per-token inputs

    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; ++s) {
            ptx::mbar_init(&full[s], 1);
            ptx::mbar_init(&empty[s], 1);
        }
        ptx::mbar_init(acc_full, 1);
        ptx::fence_barrier_init();
        ptx::prefetch_tmap(&tmap_a);
        ptx::prefetch_tmap(&tmap_b);
    }
    if (warp == 1) {
        ptx::tmem_alloc(tmem_slot, kBN);
        ptx::tmem_relinquish();
    }
    ptx::tc_fence_before();
    __syncthreads();
    ptx::tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    ptx::griddep_launch();

    if (warp == 0) {
        if (ptx::elect_one()) {
            const uint64_t wpol = ptx::policy_evict_first();  // each weight byte is read once a step
            const int pre = min(kStages, nk);
            for (int j = 0; j < pre; ++j) {  // the weights: no earlier kernel writes them
                ptx::mbar_arrive_expect_tx(&full[j], kStageBytes);
                ptx::tma_load_2d_hint(smem + j * kStageBytes, &tmap_a, &full[j], (k0 + j) * kBK, mt * kBM, wpol);
            }
            ptx::griddep_wait();  // the tokens' activations come from the previous kernel
            int j = 0;
            for (; j < nk; ++j) {
                const int s = j % kStages;
                uint8_t *sa = smem + s * kStageBytes;
                if (j >= pre) {
                    if (!ptx::mbar_wait(&empty[s], ((j / kStages) & 1) ^ 1, err, 0x4001)) break;
                    ptx::mbar_arrive_expect_tx(&full[s], kStageBytes);
                    ptx::tma_load_2d_hint(sa, &tmap_a, &full[s], (k0 + j) * kBK, mt * kBM, wpol);
                }
                ptx::tma_load_2d(sa + kABytes, &tmap_b, &full[s], (k0 + j) * kBK, nt * kBN);
            }
            // every load this thread issued lands before the CTA can exit
            for (int i = j > kStages ? j - kStages : 0; i < j; ++i)
                ptx::mbar_wait(&full[i % kStages], (i / kStages) & 1, err, 0x4002);
        }
        __syncwarp();
    } else if (warp == 1) {
        if (ptx::elect_one()) {
            constexpr uint32_t idesc = ptx::idesc_bf16_f32(kBM, kBN);
            for (int j = 0; j < nk; ++j) {
                const int s = j % kStages;
                if (!ptx::mbar_wait(&full[s], (j / kStages) & 1, err, 0x4003)) break;
                ptx::tc_fence_after();
                const uint32_t sa = ptx::smem_u32(smem + s * kStageBytes), sb = sa + kABytes;
#pragma unroll
                for (int k = 0; k < kBK / kUK; ++k)
                    ptx::mma_bf16(tmem, ptx::sw128_kmajor_desc(sa + k * kUK * 2),
                                  ptx::sw128_kmajor_desc(sb + k * kUK * 2), idesc, (j > 0 || k > 0) ? 1u : 0u);
                ptx::mma_commit(&empty[s]);
            }
            ptx::mma_commit(acc_full);  // also with no k range, or after a wait gave up: the epilogue never hangs
        }
        __syncwarp();
    } else {
        // Epilogue warps. What no kernel of the decode step after its first writes (load_inputs PART 1) loads before
        // the wait; the outputs and the norm inputs belong to the previous kernel until it completes, so the rest of
        // this warp's first tokens' inputs loads after it, while the tensor cores work.
        load_inputs<EPI, S, CH, 1>(args, in, split, mt, nt, warp - 2, lane, 0);
        ptx::griddep_wait();
        load_inputs<EPI, S, CH, 2>(args, in, split, mt, nt, warp - 2, lane, 0);
        // TMEM lane quarter q = warp % 4 holds tile rows 32q..32q+31, one row a thread, 64 token columns.
        const int q = warp & 3;
        const bool ok = ptx::mbar_wait(acc_full, 0, err, 0x4004);
        ptx::tc_fence_after();
        uint32_t v[64];
        const uint32_t taddr = tmem + ((uint32_t)(q * 32) << 16);
        ptx::tmem_ld32(taddr, v);
        ptx::tmem_ld32(taddr + 32, v + 32);
        ptx::tmem_ld_wait();
        const int row = q * 32 + lane;
        const bool zero = !ok || nk == 0;
#pragma unroll
        for (int t = 0; t < kBN; ++t) stg[t * kBM + row] = zero ? 0.f : __uint_as_float(v[t]);
    }
    ptx::tc_fence_before();
    ptx::cluster_sync();  // every CTA's accumulator is in its shared memory

    // A thread arrives at the second cluster barrier once it has read all it needs of the other CTAs' shared memory,
    // and waits on it just before exiting: no CTA exits while another may still read its shared memory, and the
    // barrier's latency overlaps the epilogue's stores.
    if (warp >= 2) {
        if (NT <= CH) {
            float4 y[CH];
            reduce_tokens<S, CH>(in, stg, lane, y);
            __syncwarp();
            ptx::cluster_arrive();
            finish_tokens<EPI, CH>(args, in, y, mt, lane);
        } else {  // tokens beyond the first CH of the warp (S below 4)
            for (int i0 = 0; i0 < NT; i0 += CH) {
                if (i0 > 0) load_inputs<EPI, S, CH>(args, in, split, mt, nt, warp - 2, lane, i0);
                float4 y[CH];
                reduce_tokens<S, CH>(in, stg, lane, y);
                finish_tokens<EPI, CH>(args, in, y, mt, lane);
            }
            __syncwarp();
            ptx::cluster_arrive();
        }
    } else {
        __syncwarp();
        ptx::cluster_arrive();
    }
    __syncwarp();
    ptx::cluster_wait();
    ptx::tc_fence_after();
    if (warp == 1) ptx::tmem_dealloc(tmem, kBN);
}

// Norm inputs from the residual stream (and, with ids, the embedding first): one block of 8 warps a token, warp w
// taking the 128-column groups w, w + 8, ...
__global__ void __launch_bounds__(256) decode_prep_kernel(const uint32_t *ids, const __nv_bfloat16 *embed, int vocab,
                                                          float *x, int hidden, const __nv_bfloat16 *gain,
                                                          __nv_bfloat16 *u, float *ss, size_t ss_stride) {
    ptx::griddep_wait();
    ptx::griddep_launch();
    const int t = blockIdx.x, w = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int g = w; g < hidden / 128; g += 8) {
        const int m = g * 128 + 4 * lane;
        float4 *xp = reinterpret_cast<float4 *>(x + (size_t)t * hidden + m);
        float4 xv;
        if (ids) {
            const uint32_t id = ids[t];
            if (id < (uint32_t)vocab) {
                const uint2 e = *reinterpret_cast<const uint2 *>(embed + (size_t)id * hidden + m);
                xv = make_float4(bflo(e.x), bfhi(e.x), bflo(e.y), bfhi(e.y));
            } else {
                const float nan = __uint_as_float(0x7FC00000u);
                xv = make_float4(nan, nan, nan, nan);
            }
            *xp = xv;
        } else {
            xv = *xp;
        }
        *reinterpret_cast<uint2 *>(u + (size_t)t * hidden + m) = gained(xv, gain + m);
        const float s = group_ss(xv);
        if (lane == 0) ss[(size_t)g * ss_stride + t] = s;
    }
}

template <int EPI, int S>
cudaError_t launch_dec(const CUtensorMap &ta, const CUtensorMap &tb, const DecodeGemmArgs &a, cudaStream_t st) {
    static SmemOptIn opt;
    if (cudaError_t e = opt.set((const void *)gemm_dec_kernel<EPI, S>, kSmem, S > 8)) return e;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(S * (a.M / kBM), (a.N + kBN - 1) / kBN);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = kSmem;
    cfg.stream = st;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = S;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl_enabled() ? 2 : 1;
    return cudaLaunchKernelEx(&cfg, gemm_dec_kernel<EPI, S>, ta, tb, a);
}

template <int EPI>
cudaError_t launch_dec_s(const CUtensorMap &ta, const CUtensorMap &tb, const DecodeGemmArgs &a, cudaStream_t st) {
    switch (a.splits) {
        case 1: return launch_dec<EPI, 1>(ta, tb, a, st);
        case 2: return launch_dec<EPI, 2>(ta, tb, a, st);
        case 3: return launch_dec<EPI, 3>(ta, tb, a, st);
        case 4: return launch_dec<EPI, 4>(ta, tb, a, st);
        case 8: return launch_dec<EPI, 8>(ta, tb, a, st);
        case 16: return launch_dec<EPI, 16>(ta, tb, a, st);
    }
    return cudaErrorInvalidValue;
}

}  // namespace

int decode_gemm_splits(int M, int K, int sms) {
    const int m_tiles = (M + kBM - 1) / kBM, nkb = (K + kBK - 1) / kBK;
    static const int kSizes[] = {1, 2, 3, 4, 8, 16};  // the compiled cluster sizes
    // The fewest splits that leave every CTA at most kStages k blocks (all its weights fetched before it waits for
    // the previous kernel), as long as one wave holds the grid; else the most splits one wave holds.
    int s = kMaxSplits;
    for (int c : kSizes)
        if ((nkb + c - 1) / c <= kStages) {
            s = c;
            break;
        }
    auto smaller = [](int c) { return c == 16 ? 8 : (c == 8 ? 4 : c - 1); };
    while (s > 1 && (long)m_tiles * s > (long)kCtasPerSm * sms) s = smaller(s);
    while (s > 1 && (s > nkb || (s - 1) * ((nkb + s - 1) / s) >= nkb)) s = smaller(s);  // no empty split
    return s;
}

const char *decode_gemm_check(const DecodeGemmArgs &a) {
    if (a.M < kBM || a.M % kBM || a.N < 1 || a.K < 1) return "M must be a positive multiple of 128, N and K positive";
    if (a.K % 8) return "K must be a multiple of 8 (16-byte rows for TMA)";
    if (((uintptr_t)a.A & 15) || ((uintptr_t)a.B & 15)) return "A and B must be 16-byte aligned";
    const int nkb = (a.K + kBK - 1) / kBK;
    if (a.splits < 1 || a.splits > kMaxSplits || (a.splits > 4 && a.splits != 8 && a.splits != 16) ||
        a.kb_per_split < 1)
        return "splits must be 1, 2, 3, 4, 8 or 16 and kb_per_split positive";
    if ((long)a.splits * a.kb_per_split < nkb || (long)(a.splits - 1) * a.kb_per_split >= nkb)
        return "the splits must cover K with no empty split";
    if (a.ss && (a.nss < 1 || a.hidden < 1 || a.ss_stride < (size_t)a.N)) return "bad norm-scale inputs";
    if (!a.err) return "error word missing";
    switch (a.epi) {
        case DEC_RESID:
            if (!a.x || ((uintptr_t)a.x & 15)) return "the residual stream must be 16-byte aligned";
            if (a.gain && (!a.u || !a.ss_out || ((uintptr_t)a.u & 7) || ((uintptr_t)a.gain & 7) ||
                           a.ss_stride < (size_t)a.N))
                return "the next norm's inputs need u, ss_out (8-byte aligned) and a stride of at least N";
            if (a.ss) return "the residual GEMM takes finished activations (no norm scale)";
            return nullptr;
        case DEC_SWIGLU:
            if (!a.act || ((uintptr_t)a.act & 7) || a.ld_act % 4 || a.ld_act < a.M / 2) return "bad SwiGLU output";
            return nullptr;
        case DEC_QKV: {
            const QkvEpilogue &q = a.qkv;
            if (a.M != (q.q_heads + 2 * q.kv_heads) * kHeadDim) return "M must be (q_heads + 2 kv_heads) * 128";
            if (!q.q_out || !q.pool || !q.pages || !q.q_norm || !q.k_norm || !q.cos_t || !q.sin_t || !q.tok_slot ||
                !q.tok_pos)
                return "the q/k/v epilogue is missing a pointer";
            if (((uintptr_t)q.q_out | (uintptr_t)q.pool) & 7) return "q and the KV pool must be 8-byte aligned";
            return nullptr;
        }
    }
    return "unknown decode epilogue";
}

cudaError_t decode_gemm_launch(const DecodeGemmArgs &a, cudaStream_t st) {
    CUtensorMap ta, tb;
    if (!gemm_tmap_2d(&ta, a.A, a.M, a.K, kBM) || !gemm_tmap_2d(&tb, a.B, a.N, a.K, kBN))
        return cudaErrorInvalidValue;
    switch (a.epi) {
        case DEC_QKV: return launch_dec_s<DEC_QKV>(ta, tb, a, st);
        case DEC_SWIGLU: return launch_dec_s<DEC_SWIGLU>(ta, tb, a, st);
        case DEC_RESID: return launch_dec_s<DEC_RESID>(ta, tb, a, st);
    }
    return cudaErrorInvalidValue;
}

cudaError_t launch_decode_prep(const uint32_t *ids, const __nv_bfloat16 *embed, int vocab, float *x, int T,
                               int hidden, const __nv_bfloat16 *gain, __nv_bfloat16 *u, float *ss, size_t ss_stride,
                               cudaStream_t st) {
    if (T < 1 || hidden % 128 || !x || !gain || !u || !ss || (ids && !embed)) return cudaErrorInvalidValue;
    return launch_kernel(decode_prep_kernel, dim3(T), dim3(256), 0, st, ids, embed, vocab, x, hidden, gain, u, ss,
                         ss_stride);
}

}  // namespace lrm

namespace lrm {
uint32_t *device_error_word();
int device_sms();
lrm_status op_fail(lrm_status s, const std::string &m);
lrm_status op_cuda(cudaError_t e, const char *what);
}  // namespace lrm

extern "C" lrm_status lrm_op_decode_gemm(void *stream, const lrm_decode_gemm_desc *d) {
    using namespace lrm;
    if (!d) return op_fail(LRM_ERR_ARGUMENT, "decode gemm: descriptor is null");
    if (d->epilogue != LRM_DEC_RESID && d->epilogue != LRM_DEC_SWIGLU)
        return op_fail(LRM_ERR_ARGUMENT, "decode gemm: the epilogue must be LRM_DEC_RESID or LRM_DEC_SWIGLU");
    // the tile and k-block counts are int32 ((k + 63) / 64 and the like): a bound well below INT_MAX
    if (d->m < 1 || d->n < 1 || d->k < 1 || d->m > (1 << 30) || d->n > (1 << 30) || d->k > (1 << 30))
        return op_fail(LRM_ERR_ARGUMENT, "decode gemm: sizes must be 1 .. 2^30");
    DecodeGemmArgs a;
    memset(&a, 0, sizeof a);
    a.M = d->m;
    a.N = d->n;
    a.K = d->k;
    a.A = (const void *)d->w;
    a.B = (const void *)d->b;
    a.epi = d->epilogue == LRM_DEC_RESID ? DEC_RESID : DEC_SWIGLU;
    a.splits = d->splits ? d->splits : decode_gemm_splits(d->m, d->k, device_sms());
    const int nkb = (d->k + kBK - 1) / kBK;
    a.kb_per_split = a.splits > 0 ? (nkb + a.splits - 1) / a.splits : 0;
    a.ss_stride = (size_t)d->ss_stride;
    if (a.epi == DEC_SWIGLU) {
        a.ss = (const float *)d->ss;
        a.nss = d->nss;
        a.hidden = d->hidden;
        a.eps = d->eps;
        a.act = (__nv_bfloat16 *)d->act;
        a.ld_act = d->ld_act;
    } else {
        a.x = (float *)d->x;
        a.gain = (const __nv_bfloat16 *)d->gain;
        a.u = (__nv_bfloat16 *)d->u;
        a.ss_out = (float *)d->ss_out;
    }
    a.err = device_error_word();
    if (!a.err) return LRM_ERR_CUDA;
    if (const char *why = decode_gemm_check(a)) return op_fail(LRM_ERR_ARGUMENT, std::string("decode gemm: ") + why);
    return op_cuda(decode_gemm_launch(a, (cudaStream_t)stream), "decode gemm");
}

