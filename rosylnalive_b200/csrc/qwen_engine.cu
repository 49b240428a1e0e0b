// qwen_engine.cu -- the Qwen3 decoder forward on one B200 (bf16 fast path), exported as lrm_qwen_* in lrm_cuda.h.
//
// It composes the forward of tests/Lrm.Tensor.Tests/TinyModel.fs:144-204 (embed; per layer input norm, q/k/v,
// QK-norm, RoPE, KV append, causal GQA attention, o_proj + residual, post norm, gate/up, SwiGLU, down + residual;
// final norm; tied lm_head; argmax) from the fused kernels:
//
//   prefill (T tokens of packed sequences)            decode step (B rows, one token each)
//   decode_prep (embed; layer 0's norm inputs)        advance (positions, lengths) ; decode_prep (embed; norm inputs)
//   per layer:                                        per layer:
//     GEMM u.Wqkv^T + norm scale; q/k/v epilogue:       GEMM Wqkv.u^T + norm scale, QK-norm, RoPE, KV append
//       QK-norm, RoPE, q; k, v into the paged cache     paged split-K decode attention + combine
//     flash prefill attention over the cache -> attn    GEMM Wo.attn^T + x += . ; next norm's inputs
//     GEMM attn.Wo^T: x += . ; next norm's inputs       GEMM Wgu.u^T + norm scale, SwiGLU
//     GEMM u.Wgu^T + norm scale, SwiGLU -> act          GEMM Wdown.act^T + x += . ; next norm's inputs
//     GEMM act.Wdown^T: x += . ; next norm's inputs
//   final norm of the last rows ; lm_head ; argmax    final norm ; lm_head GEMM ; argmax
//
// RMSNorm runs inside the GEMMs on both paths: the GEMM that updates the residual stream x also writes the next
// norm's inputs, u = bf16(gain * x) and per-column-group sums of squares of x, and the GEMM that consumes u multiplies
// its output rows by the norm's scale 1 / sqrt(mean(x^2) + eps) (it is linear in each row), so no kernel boundary
// waits for a whole row's norm. Prefill GEMMs run on CTA pairs (gemm_tcgen05.cu).
//
// Decode GEMMs swap A and B (weights fill the 128-row tensor-core tile, the B <= 64 tokens are N) and split K over a
// cluster of CTAs that reduces through distributed shared memory and runs the consumer itself (gemm_decode.cu). A
// token's RMSNorm is applied as a scale of the next GEMM's output rows: the GEMM reads u = bf16(gain * x) and the
// per-128-column sums of squares of x, which the producing GEMM writes, so no kernel boundary waits for a whole
// row's norm. The decode step is a fixed sequence of launches over device-resident inputs, so it is captured once as
// a CUDA graph and replayed.
//
// A pipeline stage (lrm_qwen_create_stage) holds layers [first, end) of the model and their KV cache: the first
// stage embeds ids, the last applies the final norm and the tied head; between stages the fp32 residual x crosses
// (lrm_qwen_residual). A stage resumes with the norm form the unsplit forward uses at that point (warp rows in
// prefill, block rows in decode) and ends with the residual sum alone, so a split forward is bit-identical to the
// unsplit one.
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdio.h>
#include <string.h>

#include <algorithm>
#include <memory>
#include <string>
#include <vector>

#include "../../include/lrm_cuda.h"
#include "gemm.h"
#include "internal.h"
#include "qwen.h"

namespace lrm {
uint32_t *device_error_word();
int device_sms();
}  // namespace lrm

using namespace lrm;

namespace {

struct Layer {
    __nv_bfloat16 *w_qkv, *w_o, *w_gu, *w_down;
    __nv_bfloat16 *in_norm, *post_norm, *q_norm, *k_norm;
};

template <class T>
T *carve(uint8_t *&p, size_t n) {
    T *r = (T *)p;
    p += (n * sizeof(T) + 255) & ~(size_t)255;
    return r;
}

}  // namespace

struct lrm_qwen_s {
    lrm_qwen_config c;
    int first = 0, nl = 0;               // this stage's layers: [first, first + nl) of c.layers
    bool is_first = true, is_last = true;  // embeds ids / applies the final norm and the head
    int device = 0;
    cudaStream_t stream = nullptr;
    int sms = 148;
    uint32_t *err = nullptr;
    std::string error;
    // weights
    uint8_t *wmem = nullptr;
    size_t wbytes = 0;
    __nv_bfloat16 *embed = nullptr, *final_norm = nullptr;
    std::vector<Layer> layers;
    float *cos_t = nullptr, *sin_t = nullptr;
    bool rope_set = false;
    // KV
    __nv_bfloat16 *pool = nullptr;
    size_t layer_pool_elems = 0;
    int32_t *d_pages = nullptr, *d_seq_len = nullptr;
    std::vector<int32_t> h_pages, h_seq_len;
    std::vector<std::vector<int32_t>> slot_pages;
    std::vector<int32_t> free_pages;
    int maxp = 0;
    // activations
    uint8_t *amem = nullptr;
    uint32_t *ids = nullptr, *next = nullptr;
    int32_t *tok_slot = nullptr, *tok_pos = nullptr, *cu = nullptr, *last_idx = nullptr, *d_slots = nullptr;
    int32_t *pf_slot = nullptr, *pf_past = nullptr;  // per prefill sequence: its slot and cached tokens before it
    float *x = nullptr, *qkv = nullptr, *partial = nullptr, *part_o = nullptr, *part_ml = nullptr;
    float *ss = nullptr;  // decode: per-128-column sums of squares of x [hidden / 128][ss_stride], the norm inputs
    size_t ss_stride = 0;
    __nv_bfloat16 *xn = nullptr, *q = nullptr, *attn = nullptr, *act = nullptr, *xl = nullptr;
    size_t partial_elems = 0;
    int max_splits_attn = 0;
    int pps = 32;
    // decode graphs: the most recent capture (replay, last ids, timers) and every kept capture by slot set
    struct KeptGraph {
        std::vector<int32_t> slots;
        cudaGraphExec_t exec;
    };
    static constexpr size_t kKeptGraphs = 8;
    std::vector<KeptGraph> kept;
    cudaGraphExec_t graph = nullptr;
    int graph_batch = 0;
    int graph_kernels = 0;
    bool graph_timed = false;
    std::vector<cudaEvent_t> attn_ev;  // 2 per layer, recorded inside a timed graph
    std::vector<int32_t> graph_slots;
    std::vector<int32_t> dev_slots;  // what d_slots holds (set_slots is its only writer): an unchanged list is not copied
    // the slot list whose last step's next ids the id buffer holds (the input a replay of their graph reads); empty
    // after a prefill, which fills the buffer with prompt ids
    std::vector<int32_t> ids_slots;
    // staging
    uint32_t *h_pinned = nullptr;
    uint32_t *h_err = nullptr;  // the error word read back on the stream, so one synchronise covers it
    int qkv_rows = 0;
};

static lrm_status qfail(lrm_qwen q, lrm_status s, const std::string &m) {
    if (q) q->error = m;
    set_thread_error(m);
    return s;
}
static lrm_status qcuda(lrm_qwen q, cudaError_t e, const char *what) {
    if (e == cudaSuccess) return LRM_OK;
    return qfail(q, LRM_ERR_CUDA, std::string(what) + ": " + cudaGetErrorName(e) + " (" + cudaGetErrorString(e) + ")");
}
#define QTRY(q, call, what)                              \
    do {                                                 \
        cudaError_t e_ = (call);                         \
        if (e_ != cudaSuccess) return qcuda(q, e_, what); \
    } while (0)

// `fused` (prefill) carries the CTA-pair choice and the fused norm's fields (norm_* outputs, row_* scale inputs).
static lrm_status gemm(lrm_qwen Q, const void *A, const void *B, int M, int N, int K, int epi, int bn, int splits,
                       void *out, int ldo, const float *resid, int ldr, size_t split_stride,
                       const QkvEpilogue *qkv = nullptr, const GemmArgs *fused = nullptr) {
    GemmArgs a;
    memset(&a, 0, sizeof a);
    if (fused) a = *fused;
    if (qkv) a.qkv = *qkv;
    a.M = M;
    a.N = N;
    a.K = K;
    a.A = A;
    a.B = B;
    a.epi = epi;
    a.bn = bn;
    a.splits = splits;
    int nkb = (K + 63) / 64;
    a.kb_per_split = (nkb + splits - 1) / splits;
    if (epi == EPI_SWIGLU || epi == EPI_BF16)
        a.out_bf16 = (__nv_bfloat16 *)out;
    else if (epi == EPI_PARTIAL)
        a.partial = (float *)out;
    else
        a.out_f32 = (float *)out;
    a.ldo = ldo;
    a.resid = resid;
    a.ldr = ldr;
    a.split_stride = split_stride;
    a.err = Q->err;
    // The weight operand is written by no kernel, so under programmatic dependent launch it is prefetched early.
    auto is_weight = [&](const void *p) {
        return (const uint8_t *)p >= Q->wmem && (const uint8_t *)p < Q->wmem + Q->wbytes;
    };
    a.independent = is_weight(A) ? 1 : (is_weight(B) ? 2 : 0);
    if (const char *why = gemm_check(a)) return qfail(Q, LRM_ERR_ARGUMENT, std::string("gemm: ") + why);
    if (epi == EPI_PARTIAL && out == Q->partial && (size_t)splits * split_stride > Q->partial_elems)
        return qfail(Q, LRM_ERR_STATE, "gemm: the split-K partials do not fit the partial buffer");
    return qcuda(Q, gemm_launch(a, Q->sms, Q->stream), "gemm");
}

// A decode-step GEMM with its consumer fused (gemm_decode.cu): W [M, K] times the step's B tokens [B, K].
static lrm_status dgemm(lrm_qwen Q, DecodeGemmArgs &a, int epi, const void *W, const void *Bop, int M, int K, int B) {
    a.M = M;
    a.N = B;
    a.K = K;
    a.A = W;
    a.B = Bop;
    a.epi = epi;
    a.splits = decode_gemm_splits(M, K, Q->sms);
    const int nkb = (K + 63) / 64;
    a.kb_per_split = (nkb + a.splits - 1) / a.splits;
    a.err = Q->err;
    if (const char *why = decode_gemm_check(a)) return qfail(Q, LRM_ERR_ARGUMENT, std::string("decode gemm: ") + why);
    return qcuda(Q, decode_gemm_launch(a, Q->stream), "decode gemm");
}

#define LTRY(expr)                      \
    do {                                \
        lrm_status s_ = (expr);         \
        if (s_ != LRM_OK) return s_;    \
    } while (0)
#define KTRY(Q, call, what) QTRY(Q, call, what)

// One decode step over device-resident ids/slots (Q->ids[0..B), Q->d_slots) -> Q->next; logits in Q->partial.
// Turns programmatic dependent launch on for the kernels an engine sequence launches on this thread.
struct PdlScope {
    PdlScope() { set_pdl(true); }
    ~PdlScope() { set_pdl(false); }
};

// The gain of the norm after local layer l: the next layer's input norm, the final norm after the model's last
// layer, or null after the last layer of an earlier stage.
static const __nv_bfloat16 *next_norm_of(lrm_qwen Q, int l) {
    if (l + 1 < Q->nl) return Q->layers[l + 1].in_norm;
    return Q->is_last ? Q->final_norm : nullptr;
}

static lrm_status decode_step(lrm_qwen Q, int B, bool timed = false) {
    PdlScope pdl;
    const lrm_qwen_config &c = Q->c;
    cudaStream_t st = Q->stream;
    const int H = c.hidden, qh = c.q_heads, kvh = c.kv_heads, I = c.intermediate;
    const int nqkv = Q->qkv_rows;
    KTRY(Q, launch_advance(Q->d_slots, B, Q->d_seq_len, Q->tok_pos, st), "advance");
    // The first layer's norm inputs: u = bf16(in_norm * x) (in xn) and the per-128-column sums of squares of x.
    // x[0, B) is the embedding of the ids on the first stage, the previous stage's residual on the others.
    KTRY(Q, launch_decode_prep(Q->is_first ? Q->ids : nullptr, Q->embed, c.vocab, Q->x, B, H, Q->layers[0].in_norm,
                               Q->xn, Q->ss, Q->ss_stride, st),
         "decode prep");
    DecodeGemmArgs base;
    memset(&base, 0, sizeof base);
    for (int l = 0; l < Q->nl; ++l) {
        const Layer &L = Q->layers[l];
        // q/k/v with the input norm's scale, QK-norm, RoPE and the paged KV append
        DecodeGemmArgs qa = base;
        qa.ss = Q->ss;
        qa.nss = H / 128;
        qa.hidden = H;
        qa.ss_stride = Q->ss_stride;
        qa.eps = c.eps;
        QkvEpilogue &qe = qa.qkv;
        qe.q_out = Q->q;
        qe.pool = Q->pool + (size_t)l * Q->layer_pool_elems;
        qe.pages = Q->d_pages;
        qe.pages_per_seq = Q->maxp;
        qe.q_heads = qh;
        qe.kv_heads = kvh;
        qe.q_norm = L.q_norm;
        qe.k_norm = L.k_norm;
        qe.eps = c.eps;
        qe.cos_t = Q->cos_t;
        qe.sin_t = Q->sin_t;
        qe.tok_slot = Q->d_slots;
        qe.tok_pos = Q->tok_pos;
        LTRY(dgemm(Q, qa, DEC_QKV, L.w_qkv, Q->xn, nqkv, H, B));
        DecodeAttnArgs da;
        da.q = Q->q;
        da.kv = KvLayout{qe.pool, Q->d_pages, Q->maxp, kvh};
        da.slots = Q->d_slots;
        da.seq_len = Q->d_seq_len;
        da.B = B;
        da.q_heads = qh;
        da.pages_per_split = Q->pps;
        da.max_splits = Q->max_splits_attn;
        da.scale_log2 = 1.4426950408889634f / sqrtf((float)kHeadDim);
        da.part_o = Q->part_o;
        da.part_ml = Q->part_ml;
        da.out = Q->attn;
        da.err = Q->err;
        da.early_pages = true;  // the q/k/v GEMM before it writes only q and the new token's K/V
        if (timed) KTRY(Q, cudaEventRecordWithFlags(Q->attn_ev[2 * l], st, cudaEventRecordExternal), "event");
        KTRY(Q, launch_decode_attention(da, st), "decode_attention");
        if (timed) KTRY(Q, cudaEventRecordWithFlags(Q->attn_ev[2 * l + 1], st, cudaEventRecordExternal), "event");
        // o_proj: x += attn Wo^T, then the post-attention norm's inputs
        DecodeGemmArgs oa = base;
        oa.x = Q->x;
        oa.gain = L.post_norm;
        oa.u = Q->xn;
        oa.ss_out = Q->ss;
        oa.ss_stride = Q->ss_stride;
        LTRY(dgemm(Q, oa, DEC_RESID, L.w_o, Q->attn, H, qh * kHeadDim, B));
        // gate/up with the post norm's scale and SwiGLU
        DecodeGemmArgs ga = base;
        ga.ss = Q->ss;
        ga.nss = H / 128;
        ga.hidden = H;
        ga.ss_stride = Q->ss_stride;
        ga.eps = c.eps;
        ga.act = Q->act;
        ga.ld_act = I;
        LTRY(dgemm(Q, ga, DEC_SWIGLU, L.w_gu, Q->xn, 2 * I, H, B));
        // down: x += act Wdown^T, then the next layer's norm inputs (none after a stage's or the model's last layer)
        DecodeGemmArgs dn = base;
        dn.x = Q->x;
        dn.gain = l + 1 < Q->nl ? Q->layers[l + 1].in_norm : nullptr;
        dn.u = Q->xn;
        dn.ss_out = Q->ss;
        dn.ss_stride = Q->ss_stride;
        LTRY(dgemm(Q, dn, DEC_RESID, L.w_down, Q->act, H, I, B));
    }
    if (!Q->is_last) return LRM_OK;
    KTRY(Q, launch_norm_rows_block(Q->x, B, H, Q->final_norm, c.eps, Q->xn, st), "final norm");
    LTRY(gemm(Q, Q->embed, Q->xn, c.vocab, B, H, EPI_PARTIAL, 64, 1, Q->partial, c.vocab, nullptr, 0,
              (size_t)B * c.vocab));
    KTRY(Q, launch_argmax(Q->partial, B, c.vocab, Q->next, st), "argmax");
    return LRM_OK;
}

static lrm_status check_ready(lrm_qwen Q) {
    if (!Q) return qfail(nullptr, LRM_ERR_ARGUMENT, "engine is null");
    if (!Q->rope_set) return qfail(Q, LRM_ERR_STATE, "set the RoPE table first");
    cudaSetDevice(Q->device);
    return LRM_OK;
}

static lrm_status sync_check(lrm_qwen Q) {
    // the kernels write the error word on this stream: read it back behind them, then wait once
    QTRY(Q, cudaMemcpyAsync(Q->h_err, Q->err, 4, cudaMemcpyDeviceToHost, Q->stream), "error word");
    QTRY(Q, cudaStreamSynchronize(Q->stream), "stream");
    const uint32_t code = *Q->h_err;
    if (code) {
        cudaMemset(Q->err, 0, 4);
        char buf[96];
        if (code == kErrDecodeLen) {
            snprintf(buf, sizeof buf, "decode attention: a row's key count exceeds its page table (code 0x%x)", code);
            return qfail(Q, LRM_ERR_STATE, buf);
        }
        if (code == kErrPrefillSeq) {
            snprintf(buf, sizeof buf, "prefill attention: a sequence lies outside its rows (code 0x%x)", code);
            return qfail(Q, LRM_ERR_STATE, buf);
        }
        snprintf(buf, sizeof buf, "a kernel's bounded wait gave up (code 0x%x)", code);
        return qfail(Q, LRM_ERR_TIMEOUT, buf);
    }
    return LRM_OK;
}

static lrm_status upload_page_row(lrm_qwen Q, int slot) {
    int32_t *row = &Q->h_pages[(size_t)slot * Q->maxp];
    QTRY(Q, cudaMemcpyAsync(Q->d_pages + (size_t)slot * Q->maxp, row, sizeof(int32_t) * Q->maxp,
                            cudaMemcpyHostToDevice, Q->stream),
         "page table");
    return sync_check(Q);
}

extern "C" {

lrm_status lrm_qwen_create(int32_t device, const lrm_qwen_config *cfg, lrm_qwen *out) {
    if (!cfg) return qfail(nullptr, LRM_ERR_ARGUMENT, "null argument");
    return lrm_qwen_create_stage(device, cfg, 0, cfg->layers, out);
}

lrm_status lrm_qwen_create_stage(int32_t device, const lrm_qwen_config *cfg, int32_t first_layer, int32_t end_layer,
                                 lrm_qwen *out) {
    if (!cfg || !out) return qfail(nullptr, LRM_ERR_ARGUMENT, "null argument");
    *out = nullptr;
    const lrm_qwen_config c = *cfg;
    if (c.head_dim != kHeadDim) return qfail(nullptr, LRM_ERR_ARGUMENT, "the bf16 engine needs head_dim 128");
    if (c.kv_heads < 1 || c.q_heads != 2 * c.kv_heads)
        return qfail(nullptr, LRM_ERR_ARGUMENT, "the bf16 engine needs q_heads = 2 * kv_heads");
    if (c.hidden % 128 || c.intermediate % 128 || c.hidden < 128)
        return qfail(nullptr, LRM_ERR_ARGUMENT, "hidden and intermediate must be multiples of 128");
    if (c.layers < 1 || c.vocab < 1 || c.max_pos < 1 || c.max_seqs < 1 || c.kv_pages < 1 || c.max_tokens < 1 ||
        c.max_batch < 1 || c.max_batch > 65535)
        return qfail(nullptr, LRM_ERR_ARGUMENT, "sizes must be positive");
    if (first_layer < 0 || end_layer <= first_layer || end_layer > c.layers)
        return qfail(nullptr, LRM_ERR_ARGUMENT, "a stage holds layers [first, end) with 0 <= first < end <= layers");
    cudaError_t e = cudaSetDevice(device);
    if (e != cudaSuccess) return qcuda(nullptr, e, "cudaSetDevice");
    std::unique_ptr<lrm_qwen_s> Q(new lrm_qwen_s());
    Q->c = c;
    Q->first = first_layer;
    Q->nl = end_layer - first_layer;
    Q->is_first = first_layer == 0;
    Q->is_last = end_layer == c.layers;
    Q->device = device;
    Q->err = device_error_word();
    Q->sms = device_sms();
    if (!Q->err) return LRM_ERR_CUDA;
    QTRY(Q.get(), cudaStreamCreateWithFlags(&Q->stream, cudaStreamNonBlocking), "stream");
    const int H = c.hidden, qh = c.q_heads, kvh = c.kv_heads, I = c.intermediate, V = c.vocab;
    Q->qkv_rows = (qh + 2 * kvh) * kHeadDim;
    // weights
    size_t per_layer = (size_t)Q->qkv_rows * H + (size_t)H * qh * kHeadDim + (size_t)2 * I * H + (size_t)H * I +
                       2 * H + 2 * kHeadDim;
    const bool has_embed = Q->is_first || Q->is_last;  // the gather table, and the tied head
    size_t wbytes = ((has_embed ? (size_t)V * H : 0) + H) * 2 + (size_t)Q->nl * (per_layer * 2 + 8 * 256) + 4096;
    QTRY(Q.get(), cudaMalloc(&Q->wmem, wbytes), "weights");
    Q->wbytes = wbytes;
    QTRY(Q.get(), cudaMemset(Q->wmem, 0, wbytes), "weights");
    uint8_t *p = Q->wmem;
    Q->embed = has_embed ? carve<__nv_bfloat16>(p, (size_t)V * H) : nullptr;
    Q->final_norm = Q->is_last ? carve<__nv_bfloat16>(p, H) : nullptr;
    Q->layers.resize(Q->nl);
    for (auto &L : Q->layers) {
        L.w_qkv = carve<__nv_bfloat16>(p, (size_t)Q->qkv_rows * H);
        L.w_o = carve<__nv_bfloat16>(p, (size_t)H * qh * kHeadDim);
        L.w_gu = carve<__nv_bfloat16>(p, (size_t)2 * I * H);
        L.w_down = carve<__nv_bfloat16>(p, (size_t)H * I);
        L.in_norm = carve<__nv_bfloat16>(p, H);
        L.post_norm = carve<__nv_bfloat16>(p, H);
        L.q_norm = carve<__nv_bfloat16>(p, kHeadDim);
        L.k_norm = carve<__nv_bfloat16>(p, kHeadDim);
    }
    QTRY(Q.get(), cudaMalloc(&Q->cos_t, sizeof(float) * (size_t)c.max_pos * 64), "rope");
    QTRY(Q.get(), cudaMalloc(&Q->sin_t, sizeof(float) * (size_t)c.max_pos * 64), "rope");
    // KV pool and page tables
    Q->maxp = (c.max_pos + kPageTokens - 1) / kPageTokens;
    Q->layer_pool_elems = (size_t)c.kv_pages * kv_page_elems(kvh);
    e = cudaMalloc(&Q->pool, Q->layer_pool_elems * Q->nl * sizeof(__nv_bfloat16));
    if (e != cudaSuccess) return qfail(Q.get(), LRM_ERR_OUT_OF_MEMORY, "KV pool allocation failed");
    QTRY(Q.get(), cudaMemset(Q->pool, 0, Q->layer_pool_elems * Q->nl * sizeof(__nv_bfloat16)), "KV pool");
    QTRY(Q.get(), cudaMalloc(&Q->d_pages, sizeof(int32_t) * (size_t)c.max_seqs * Q->maxp), "pages");
    QTRY(Q.get(), cudaMemset(Q->d_pages, 0, sizeof(int32_t) * (size_t)c.max_seqs * Q->maxp), "pages");
    QTRY(Q.get(), cudaMalloc(&Q->d_seq_len, sizeof(int32_t) * c.max_seqs), "seq_len");
    QTRY(Q.get(), cudaMemset(Q->d_seq_len, 0, sizeof(int32_t) * c.max_seqs), "seq_len");
    Q->h_pages.assign((size_t)c.max_seqs * Q->maxp, 0);
    Q->h_seq_len.assign(c.max_seqs, 0);
    Q->slot_pages.resize(c.max_seqs);
    for (int i = c.kv_pages - 1; i >= 0; --i) Q->free_pages.push_back(i);
    // activations
    const int T = c.max_tokens > c.max_batch ? c.max_tokens : c.max_batch;
    const int R = c.max_batch > c.max_seqs ? c.max_batch : c.max_seqs;
    Q->max_splits_attn = (Q->maxp + Q->pps - 1) / Q->pps;
    size_t part = (size_t)R * V;
    size_t dec = (size_t)16 * c.max_batch * (Q->qkv_rows > 2 * I ? Q->qkv_rows : 2 * I) * 2;
    if (dec > part) part = dec;
    Q->partial_elems = part;
    size_t abytes = 0;
    abytes += (size_t)T * 4 * 3 + (size_t)R * 4 * 3 + (size_t)(c.max_seqs + 1) * 4 * 4;
    abytes += (size_t)T * H * 4 + (size_t)T * Q->qkv_rows * 4 + part * 4;
    abytes += (size_t)c.max_batch * kvh * Q->max_splits_attn * 2 * (128 + 2) * 4;
    abytes += (size_t)T * (H + qh * kHeadDim * 2 + I) * 2 + (size_t)R * H * 2;
    abytes += (size_t)(H / 128) * (T > R ? T : R) * 4;
    abytes += 64 * 256;
    QTRY(Q.get(), cudaMalloc(&Q->amem, abytes), "activations");
    p = Q->amem;
    Q->ids = carve<uint32_t>(p, T);
    Q->tok_slot = carve<int32_t>(p, T);
    Q->tok_pos = carve<int32_t>(p, T);
    Q->next = carve<uint32_t>(p, R);
    Q->last_idx = carve<int32_t>(p, R);
    Q->d_slots = carve<int32_t>(p, R);
    Q->cu = carve<int32_t>(p, c.max_seqs + 1);
    Q->pf_slot = carve<int32_t>(p, c.max_seqs);
    Q->pf_past = carve<int32_t>(p, c.max_seqs);
    Q->x = carve<float>(p, (size_t)T * H);
    Q->qkv = carve<float>(p, (size_t)T * Q->qkv_rows);
    Q->partial = carve<float>(p, part);
    Q->part_o = carve<float>(p, (size_t)c.max_batch * kvh * Q->max_splits_attn * 2 * 128);
    Q->part_ml = carve<float>(p, (size_t)c.max_batch * kvh * Q->max_splits_attn * 2 * 2);
    Q->xn = carve<__nv_bfloat16>(p, (size_t)T * H);
    Q->q = carve<__nv_bfloat16>(p, (size_t)T * qh * kHeadDim);
    Q->attn = carve<__nv_bfloat16>(p, (size_t)T * qh * kHeadDim);
    Q->act = carve<__nv_bfloat16>(p, (size_t)T * I);
    Q->xl = carve<__nv_bfloat16>(p, (size_t)R * H);
    Q->ss_stride = (size_t)(T > R ? T : R);
    Q->ss = carve<float>(p, (size_t)(H / 128) * Q->ss_stride);
    if ((size_t)(p - Q->amem) > abytes) return qfail(Q.get(), LRM_ERR_STATE, "activation plan overflow");
    QTRY(Q.get(), cudaMallocHost(&Q->h_pinned, sizeof(uint32_t) * (size_t)T * 4), "pinned staging");
    QTRY(Q.get(), cudaMallocHost(&Q->h_err, sizeof(uint32_t)), "pinned error word");
    *out = Q.release();
    return LRM_OK;
}

lrm_status lrm_qwen_destroy(lrm_qwen Q) {
    if (!Q) return LRM_ERR_ARGUMENT;
    cudaSetDevice(Q->device);
    cudaStreamSynchronize(Q->stream);
    for (auto &k : Q->kept) cudaGraphExecDestroy(k.exec);
    for (auto e : Q->attn_ev) cudaEventDestroy(e);
    cudaFree(Q->wmem);
    cudaFree(Q->cos_t);
    cudaFree(Q->sin_t);
    cudaFree(Q->pool);
    cudaFree(Q->d_pages);
    cudaFree(Q->d_seq_len);
    cudaFree(Q->amem);
    cudaFreeHost(Q->h_pinned);
    cudaFreeHost(Q->h_err);
    cudaStreamDestroy(Q->stream);
    delete Q;
    return LRM_OK;
}

// Where an HF-named weight lives on the device: `count` bf16 elements at `dst`, or for gate/up (interleave 0 / 64)
// rows j at row (j / 64) * 128 + interleave + j % 64 of w_gu (64-row blocks, so a 128-column GEMM tile holds matching
// gate and up columns).
struct WeightDst {
    __nv_bfloat16 *dst = nullptr;  // null for a weight this stage does not hold
    uint64_t count = 0;
    int interleave = -1;
};

static lrm_status resolve_weight(lrm_qwen Q, const std::string &n, WeightDst &w) {
    const lrm_qwen_config &c = Q->c;
    const int H = c.hidden, qh = c.q_heads, kvh = c.kv_heads, I = c.intermediate;
    auto set = [&](__nv_bfloat16 *d, uint64_t cnt, int il = -1) {
        w.dst = d;
        w.count = cnt;
        w.interleave = il;
        return LRM_OK;
    };
    if (n == "model.embed_tokens.weight") return set(Q->embed, (uint64_t)c.vocab * H);
    if (n == "model.norm.weight") return set(Q->final_norm, H);
    int layer = -1, consumed = 0;
    if (sscanf(n.c_str(), "model.layers.%d.%n", &layer, &consumed) != 1 || consumed == 0 || layer < 0 ||
        layer >= c.layers)
        return qfail(Q, LRM_ERR_ARGUMENT, n + ": not a Qwen3 weight name of this model");
    const bool held = layer >= Q->first && layer < Q->first + Q->nl;
    static const Layer none{};
    const Layer &L = held ? Q->layers[layer - Q->first] : none;
    auto at = [&](__nv_bfloat16 *base, size_t off) { return base ? base + off : nullptr; };
    const std::string rest = n.substr(consumed);
    if (rest == "input_layernorm.weight") return set(L.in_norm, H);
    if (rest == "post_attention_layernorm.weight") return set(L.post_norm, H);
    if (rest == "self_attn.q_norm.weight") return set(L.q_norm, kHeadDim);
    if (rest == "self_attn.k_norm.weight") return set(L.k_norm, kHeadDim);
    if (rest == "self_attn.q_proj.weight") return set(L.w_qkv, (uint64_t)qh * kHeadDim * H);
    if (rest == "self_attn.k_proj.weight")
        return set(at(L.w_qkv, (size_t)qh * kHeadDim * H), (uint64_t)kvh * kHeadDim * H);
    if (rest == "self_attn.v_proj.weight")
        return set(at(L.w_qkv, (size_t)(qh + kvh) * kHeadDim * H), (uint64_t)kvh * kHeadDim * H);
    if (rest == "self_attn.o_proj.weight") return set(L.w_o, (uint64_t)H * qh * kHeadDim);
    if (rest == "mlp.down_proj.weight") return set(L.w_down, (uint64_t)H * I);
    if (rest == "mlp.gate_proj.weight") return set(L.w_gu, (uint64_t)I * H, 0);
    if (rest == "mlp.up_proj.weight") return set(L.w_gu, (uint64_t)I * H, 64);
    return qfail(Q, LRM_ERR_ARGUMENT, n + ": not a Qwen3 weight name");
}

// Copies rows [r0, r0 + rows) of a resolved weight from host memory `src` (rows x H bf16, or the whole flat tensor
// when not interleaved: r0 / rows then count elements) on `st`; rows is a multiple of 64 for gate/up.
static cudaError_t copy_weight_part(lrm_qwen Q, const WeightDst &w, uint64_t first, uint64_t n, const void *src,
                                    cudaStream_t st) {
    if (w.interleave < 0) return cudaMemcpyAsync(w.dst + first, src, n * 2, cudaMemcpyHostToDevice, st);
    const size_t H = (size_t)Q->c.hidden;
    const size_t r0 = first / H, rows = n / H;
    return cudaMemcpy2DAsync(w.dst + ((r0 / 64) * 128 + (size_t)w.interleave) * H, 128 * H * 2, src, 64 * H * 2,
                             64 * H * 2, rows / 64, cudaMemcpyHostToDevice, st);
}

lrm_status lrm_qwen_set_weight(lrm_qwen Q, const char *name, const uint16_t *w, uint64_t count) {
    if (!Q || !name || !w) return qfail(Q, LRM_ERR_ARGUMENT, "null argument");
    cudaSetDevice(Q->device);
    WeightDst d;
    LTRY(resolve_weight(Q, name, d));
    if (count != d.count) return qfail(Q, LRM_ERR_ARGUMENT, std::string(name) + ": wrong element count");
    if (!d.dst) return LRM_OK;  // another pipeline stage's weight
    QTRY(Q, copy_weight_part(Q, d, 0, count, w, Q->stream), "set_weight");
    QTRY(Q, cudaStreamSynchronize(Q->stream), "set_weight");
    return LRM_OK;
}

// bf16 bits of x rounded to nearest even (NaN stays a quiet NaN of the same sign).
static inline uint16_t narrow_bf16(uint32_t u) {
    if ((u & 0x7FFFFFFFu) > 0x7F800000u) return (uint16_t)((u >> 16) | 0x40u);
    return (uint16_t)((u + 0x7FFFu + ((u >> 16) & 1u)) >> 16);
}

lrm_status lrm_qwen_load_safetensors(lrm_qwen Q, const char *path, int32_t *loaded) {
    if (!Q || !path) return qfail(Q, LRM_ERR_ARGUMENT, "null argument");
    if (loaded) *loaded = 0;
    cudaSetDevice(Q->device);
    lrm_st_file f = nullptr;
    lrm_status s = lrm_st_open(path, &f);
    if (s != LRM_OK) {
        Q->error = thread_error();
        return s;
    }
    std::unique_ptr<lrm_st_file_s, lrm_status (*)(lrm_st_file)> guard(f, lrm_st_close);
    int64_t count = 0;
    lrm_st_info(f, nullptr, nullptr, &count, nullptr, nullptr);
    // Every tensor is checked before any byte is copied.
    std::vector<WeightDst> dst((size_t)count);
    std::vector<lrm_st_entry> ent((size_t)count);
    for (int64_t i = 0; i < count; ++i) {
        lrm_st_entry_at(f, i, &ent[(size_t)i]);
        const lrm_st_entry &e = ent[(size_t)i];
        LTRY(resolve_weight(Q, e.name, dst[(size_t)i]));
        if (e.dtype != LRM_ST_BF16 && e.dtype != LRM_ST_F32)
            return qfail(Q, LRM_ERR_ARGUMENT, std::string(e.name) + ": only BF16 and F32 weights are loaded");
        const uint64_t elems = (e.end - e.begin) / (e.dtype == LRM_ST_BF16 ? 2 : 4);
        if (elems != dst[(size_t)i].count)
            return qfail(Q, LRM_ERR_ARGUMENT, std::string(e.name) + ": wrong element count");
    }
    // Two pinned 64 MiB buffers: one fills from the mapped file while the other's copy runs.
    constexpr size_t kChunk = 64u << 20;
    uint16_t *pin[2] = {nullptr, nullptr};
    cudaEvent_t done[2] = {nullptr, nullptr};
    auto cleanup = [&]() {
        cudaStreamSynchronize(Q->stream);
        for (int b = 0; b < 2; ++b) {
            if (pin[b]) cudaFreeHost(pin[b]);
            if (done[b]) cudaEventDestroy(done[b]);
        }
    };
    for (int b = 0; b < 2; ++b) {
        cudaError_t e = cudaMallocHost(&pin[b], kChunk);
        if (e == cudaSuccess) e = cudaEventCreateWithFlags(&done[b], cudaEventDisableTiming);
        if (e != cudaSuccess) {
            cleanup();
            return qcuda(Q, e, "pinned staging");
        }
    }
    const size_t H = (size_t)Q->c.hidden;
    uint64_t part = 0;
    for (int64_t i = 0; i < count; ++i) {
        const lrm_st_entry &e = ent[(size_t)i];
        const WeightDst &d = dst[(size_t)i];
        if (!d.dst) continue;  // another pipeline stage's weight
        // elements per chunk; whole 64-row blocks for the interleaved gate/up rows
        uint64_t step = kChunk / 2;
        if (d.interleave >= 0) step = step / (64 * H) * (64 * H);
        for (uint64_t first = 0; first < d.count; first += step, ++part) {
            const uint64_t n = std::min<uint64_t>(step, d.count - first);
            const int b = (int)(part & 1);
            cudaError_t ce = cudaEventSynchronize(done[b]);  // the last copy out of this buffer has finished
            if (ce != cudaSuccess) {
                cleanup();
                return qcuda(Q, ce, "staging");
            }
            if (e.dtype == LRM_ST_BF16) {
                memcpy(pin[b], (const uint16_t *)e.data + first, n * 2);
            } else {
                const uint32_t *src = (const uint32_t *)e.data + first;
                for (uint64_t k = 0; k < n; ++k) {
                    uint32_t u;
                    memcpy(&u, src + k, 4);
                    pin[b][k] = narrow_bf16(u);
                }
            }
            ce = copy_weight_part(Q, d, first, n, pin[b], Q->stream);
            if (ce == cudaSuccess) ce = cudaEventRecord(done[b], Q->stream);
            if (ce != cudaSuccess) {
                cleanup();
                return qcuda(Q, ce, (std::string("loading ") + e.name).c_str());
            }
        }
        if (loaded) *loaded += 1;
    }
    cleanup();
    QTRY(Q, cudaGetLastError(), "loading the checkpoint");
    return LRM_OK;
}

lrm_status lrm_qwen_set_rope(lrm_qwen Q, const float *cs, const float *sn, int32_t rows, int32_t half) {
    if (!Q || !cs || !sn) return qfail(Q, LRM_ERR_ARGUMENT, "null argument");
    if (half != 64 || rows < Q->c.max_pos) return qfail(Q, LRM_ERR_ARGUMENT, "the table must be [>= max_pos, 64]");
    cudaSetDevice(Q->device);
    QTRY(Q, cudaMemcpy(Q->cos_t, cs, sizeof(float) * (size_t)Q->c.max_pos * 64, cudaMemcpyHostToDevice), "rope");
    QTRY(Q, cudaMemcpy(Q->sin_t, sn, sizeof(float) * (size_t)Q->c.max_pos * 64, cudaMemcpyHostToDevice), "rope");
    Q->rope_set = true;
    return LRM_OK;
}

lrm_status lrm_qwen_reset_seq(lrm_qwen Q, int32_t slot) {
    if (!Q || slot < 0 || slot >= Q->c.max_seqs) return qfail(Q, LRM_ERR_ARGUMENT, "slot out of range");
    cudaSetDevice(Q->device);
    for (int32_t pg : Q->slot_pages[slot]) Q->free_pages.push_back(pg);
    Q->slot_pages[slot].clear();
    std::fill(Q->h_pages.begin() + (size_t)slot * Q->maxp, Q->h_pages.begin() + (size_t)(slot + 1) * Q->maxp, 0);
    Q->h_seq_len[slot] = 0;
    int32_t zero = 0;
    QTRY(Q, cudaMemcpyAsync(Q->d_seq_len + slot, &zero, 4, cudaMemcpyHostToDevice, Q->stream), "seq_len");
    return upload_page_row(Q, slot);
}

// Gives `slot` pages for `tokens` in the host copy of its page-table row; *changed says whether the row grew.
static lrm_status reserve_host(lrm_qwen Q, int32_t slot, int32_t tokens, bool *changed) {
    const int need = (tokens + kPageTokens - 1) / kPageTokens;
    auto &pg = Q->slot_pages[slot];
    *changed = false;
    while ((int)pg.size() < need) {
        if (Q->free_pages.empty()) return qfail(Q, LRM_ERR_OUT_OF_MEMORY, "the KV pool has no free page");
        int32_t id = Q->free_pages.back();
        Q->free_pages.pop_back();
        Q->h_pages[(size_t)slot * Q->maxp + pg.size()] = id;
        pg.push_back(id);
        *changed = true;
    }
    return LRM_OK;
}

lrm_status lrm_qwen_reserve(lrm_qwen Q, int32_t slot, int32_t tokens) {
    if (!Q || slot < 0 || slot >= Q->c.max_seqs) return qfail(Q, LRM_ERR_ARGUMENT, "slot out of range");
    if (tokens > Q->c.max_pos) return qfail(Q, LRM_ERR_ARGUMENT, "tokens beyond max_pos");
    cudaSetDevice(Q->device);
    bool changed = false;
    LTRY(reserve_host(Q, slot, tokens, &changed));
    return changed ? upload_page_row(Q, slot) : LRM_OK;
}

// Prefill of `nseq` sequences packed together. Fresh (extend false): each slot is reset first. Extend: each
// sequence's rows continue the tokens its slot already holds (chunked prefill), attending to all of them.
static lrm_status run_prefill(lrm_qwen Q, int32_t nseq, const int32_t *slots, const int32_t *lens,
                              const uint32_t *ids, uint32_t *next_ids, float *logits, bool extend) {
    LTRY(check_ready(Q));
    const lrm_qwen_config &c = Q->c;
    if (nseq < 1 || nseq > c.max_seqs || !slots || !lens || (Q->is_first && !ids) || (Q->is_last && !next_ids))
        return qfail(Q, LRM_ERR_ARGUMENT, "bad prefill arguments");
    std::vector<int32_t> cu(nseq + 1, 0), last(nseq), past(nseq, 0), tslot, tpos;
    int max_len = 0;
    for (int i = 0; i < nseq; ++i) {
        if (slots[i] < 0 || slots[i] >= c.max_seqs) return qfail(Q, LRM_ERR_ARGUMENT, "bad sequence slot");
        for (int i2 = 0; i2 < i; ++i2)
            if (slots[i2] == slots[i]) return qfail(Q, LRM_ERR_ARGUMENT, "a slot appears twice in one prefill");
        past[i] = extend ? Q->h_seq_len[slots[i]] : 0;
        if (lens[i] < 1 || past[i] + lens[i] > c.max_pos)
            return qfail(Q, LRM_ERR_ARGUMENT, "bad sequence length (rows of a call >= 1, cached + rows <= max_pos)");
        cu[i + 1] = cu[i] + lens[i];
        last[i] = cu[i + 1] - 1;
        if (lens[i] > max_len) max_len = lens[i];
    }
    const int T = cu[nseq];
    if (T > c.max_tokens) return qfail(Q, LRM_ERR_ARGUMENT, "more tokens than max_tokens");
    if (Q->is_first)
        for (int i = 0; i < T; ++i)
            if (ids[i] >= (uint32_t)c.vocab) return qfail(Q, LRM_ERR_ARGUMENT, "an id is outside the vocabulary");
    for (int i = 0; i < nseq; ++i) {
        if (!extend) LTRY(lrm_qwen_reset_seq(Q, slots[i]));
        LTRY(lrm_qwen_reserve(Q, slots[i], past[i] + lens[i]));
    }
    for (int i = 0; i < nseq; ++i) {
        for (int t = 0; t < lens[i]; ++t) {
            tslot.push_back(slots[i]);
            tpos.push_back(past[i] + t);
        }
        Q->h_seq_len[slots[i]] = past[i] + lens[i];
    }
    std::vector<int32_t> new_len(nseq);
    for (int i = 0; i < nseq; ++i) new_len[i] = past[i] + lens[i];
    cudaStream_t st = Q->stream;
    if (Q->is_first) {
        Q->ids_slots.clear();
        QTRY(Q, cudaMemcpyAsync(Q->ids, ids, 4 * (size_t)T, cudaMemcpyHostToDevice, st), "ids");
    }
    QTRY(Q, cudaMemcpyAsync(Q->tok_slot, tslot.data(), 4 * (size_t)T, cudaMemcpyHostToDevice, st), "slots");
    QTRY(Q, cudaMemcpyAsync(Q->tok_pos, tpos.data(), 4 * (size_t)T, cudaMemcpyHostToDevice, st), "positions");
    QTRY(Q, cudaMemcpyAsync(Q->cu, cu.data(), 4 * (size_t)(nseq + 1), cudaMemcpyHostToDevice, st), "cu_seqlens");
    QTRY(Q, cudaMemcpyAsync(Q->last_idx, last.data(), 4 * (size_t)nseq, cudaMemcpyHostToDevice, st), "last rows");
    QTRY(Q, cudaMemcpyAsync(Q->pf_slot, slots, 4 * (size_t)nseq, cudaMemcpyHostToDevice, st), "slots");
    QTRY(Q, cudaMemcpyAsync(Q->pf_past, past.data(), 4 * (size_t)nseq, cudaMemcpyHostToDevice, st), "past");
    for (int i = 0; i < nseq; ++i)
        QTRY(Q, cudaMemcpyAsync(Q->d_seq_len + slots[i], &new_len[i], 4, cudaMemcpyHostToDevice, st), "seq_len");
    const int H = c.hidden, qh = c.q_heads, kvh = c.kv_heads, I = c.intermediate;
    const int nss_pair = (H + 255) / 256;  // the residual GEMMs' norm groups (256 columns each)
    PdlScope pdl;
    // RMSNorm fused into the GEMMs: a layer's input is u = bf16(gain * x) (in xn) with the sums of squares of x (ss);
    // the consuming GEMM applies the norm's scale to its output rows. The first layer's inputs come from the embedding
    // on the first stage, from the previous stage's residual (in the residual GEMMs' order) on the others.
    int nss_in;
    if (Q->is_first) {
        KTRY(Q, launch_decode_prep(Q->ids, Q->embed, c.vocab, Q->x, T, H, Q->layers[0].in_norm, Q->xn, Q->ss,
                                   Q->ss_stride, st),
             "norm inputs");
        nss_in = H / 128;
    } else {
        KTRY(Q, launch_pair_prep(Q->x, T, H, Q->layers[0].in_norm, Q->xn, Q->ss, Q->ss_stride, st), "norm inputs");
        nss_in = nss_pair;
    }
    GemmArgs pair;  // every prefill GEMM runs on CTA pairs (the fused norm lives in their epilogues)
    memset(&pair, 0, sizeof pair);
    pair.cta_pair = 2;
    for (int l = 0; l < Q->nl; ++l) {
        const Layer &L = Q->layers[l];
        GemmArgs scaled = pair;  // a consumer of norm inputs: its rows get the norm's scale
        scaled.row_ss = Q->ss;
        scaled.row_nss = nss_in;
        scaled.row_ss_stride = Q->ss_stride;
        scaled.row_hidden = H;
        scaled.row_eps = c.eps;
        // q/k/v GEMM with QK-RMSNorm, RoPE and the paged KV append in its epilogue (no fp32 q/k/v round trip).
        QkvEpilogue qe;
        qe.q_out = Q->q;
        qe.k_out = nullptr;  // attention reads k and v from the cache
        qe.v_out = nullptr;
        qe.pool = Q->pool + (size_t)l * Q->layer_pool_elems;
        qe.pages = Q->d_pages;
        qe.pages_per_seq = Q->maxp;
        qe.q_heads = qh;
        qe.kv_heads = kvh;
        qe.q_norm = L.q_norm;
        qe.k_norm = L.k_norm;
        qe.eps = c.eps;
        qe.cos_t = Q->cos_t;
        qe.sin_t = Q->sin_t;
        qe.tok_slot = Q->tok_slot;
        qe.tok_pos = Q->tok_pos;
        LTRY(gemm(Q, Q->xn, L.w_qkv, T, Q->qkv_rows, H, EPI_QKV, 256, 1, nullptr, Q->qkv_rows, nullptr, 0, 0, &qe,
                  &scaled));
        PrefillAttnArgs pa;
        pa.q = Q->q;
        pa.out = Q->attn;
        pa.cu_seqlens = Q->cu;
        pa.nseq = nseq;
        pa.max_len = max_len;
        pa.q_heads = qh;
        pa.kv_heads = kvh;
        pa.scale_log2 = 1.4426950408889634f / sqrtf((float)kHeadDim);
        pa.pool = qe.pool;
        pa.pages = Q->d_pages;
        pa.seq_slot = Q->pf_slot;
        pa.past = Q->pf_past;
        pa.pages_per_seq = Q->maxp;
        pa.kv_pages = c.kv_pages;
        KTRY(Q, launch_prefill_attention_tc(pa, T, Q->err, st), "prefill_attention");
        // o_proj: x += attn Wo^T, with the post-attention norm's inputs
        GemmArgs post = pair;
        post.norm_gain = L.post_norm;
        post.norm_u = Q->xn;
        post.norm_ss = Q->ss;
        post.norm_ss_stride = Q->ss_stride;
        LTRY(gemm(Q, Q->attn, L.w_o, T, H, qh * kHeadDim, EPI_RESID, 256, 1, Q->x, H, Q->x, H, 0, nullptr, &post));
        scaled.row_nss = nss_pair;
        LTRY(gemm(Q, Q->xn, L.w_gu, T, 2 * I, H, EPI_SWIGLU, 256, 1, Q->act, I, nullptr, 0, 0, nullptr, &scaled));
        // down: x += act Wdown^T, with the next layer's norm inputs (none after a stage's last layer)
        GemmArgs next = pair;
        if (l + 1 < Q->nl) {
            next.norm_gain = Q->layers[l + 1].in_norm;
            next.norm_u = Q->xn;
            next.norm_ss = Q->ss;
            next.norm_ss_stride = Q->ss_stride;
        }
        LTRY(gemm(Q, Q->act, L.w_down, T, H, I, EPI_RESID, 256, 1, Q->x, H, Q->x, H, 0, nullptr, &next));
        nss_in = nss_pair;
    }
    if (!Q->is_last) return sync_check(Q);
    // the final norm of each sequence's last row only (the greedy head reads no other)
    KTRY(Q, launch_norm_rows_block(Q->x, nseq, H, Q->final_norm, c.eps, Q->xl, st, Q->last_idx), "final norm");
    LTRY(gemm(Q, Q->embed, Q->xl, c.vocab, nseq, H, EPI_PARTIAL, 64, 1, Q->partial, c.vocab, nullptr, 0,
              (size_t)nseq * c.vocab));
    KTRY(Q, launch_argmax(Q->partial, nseq, c.vocab, Q->next, st), "argmax");
    QTRY(Q, cudaMemcpyAsync(next_ids, Q->next, 4 * (size_t)nseq, cudaMemcpyDeviceToHost, st), "next ids");
    if (logits)
        QTRY(Q, cudaMemcpyAsync(logits, Q->partial, 4 * (size_t)nseq * c.vocab, cudaMemcpyDeviceToHost, st), "logits");
    return sync_check(Q);
}

lrm_status lrm_qwen_prefill(lrm_qwen Q, int32_t nseq, const int32_t *slots, const int32_t *lens, const uint32_t *ids,
                            uint32_t *next_ids, float *logits) {
    return run_prefill(Q, nseq, slots, lens, ids, next_ids, logits, false);
}

lrm_status lrm_qwen_extend(lrm_qwen Q, int32_t nseq, const int32_t *slots, const int32_t *lens, const uint32_t *ids,
                           uint32_t *next_ids, float *logits) {
    return run_prefill(Q, nseq, slots, lens, ids, next_ids, logits, true);
}

static lrm_status set_slots(lrm_qwen Q, int32_t batch, const int32_t *slots) {
    const lrm_qwen_config &c = Q->c;
    if (batch < 1 || batch > c.max_batch || !slots) return qfail(Q, LRM_ERR_ARGUMENT, "bad batch");
    for (int b = 0; b < batch; ++b) {
        const int s = slots[b];
        if (s < 0 || s >= c.max_seqs) return qfail(Q, LRM_ERR_ARGUMENT, "slot out of range");
        for (int b2 = 0; b2 < b; ++b2)
            if (slots[b2] == s) return qfail(Q, LRM_ERR_ARGUMENT, "a slot appears twice in one step");
    }
    if ((int)Q->dev_slots.size() == batch && std::equal(Q->dev_slots.begin(), Q->dev_slots.end(), slots))
        return LRM_OK;  // d_slots already holds this list (a greedy loop passes the same slots every step)
    Q->dev_slots.clear();
    QTRY(Q, cudaMemcpyAsync(Q->d_slots, slots, 4 * (size_t)batch, cudaMemcpyHostToDevice, Q->stream), "slots");
    Q->dev_slots.assign(slots, slots + batch);
    return LRM_OK;
}

// Host-side checks before a step: every slot must have a page for its next position. The rows that grew go to the
// device table in one asynchronous copy per run of consecutive slots (sequences of equal length cross a page boundary
// on the same step, and a per-row copy with a wait each stalled that step); the copy from pageable memory is staged
// before it returns, and the step's own synchronise reports any error.
static lrm_status ensure_pages(lrm_qwen Q, int32_t batch, const int32_t *slots, int steps) {
    std::vector<int32_t> grown;
    for (int b = 0; b < batch; ++b) {
        const int s = slots[b];
        if (Q->h_seq_len[s] < 1) return qfail(Q, LRM_ERR_STATE, "decode needs a prefilled slot");
        const int need = Q->h_seq_len[s] + steps;
        if (need > Q->c.max_pos) return qfail(Q, LRM_ERR_ARGUMENT, "the sequence would pass max_pos");
        bool changed = false;
        LTRY(reserve_host(Q, s, need, &changed));
        if (changed) grown.push_back(s);
    }
    std::sort(grown.begin(), grown.end());
    for (size_t i = 0; i < grown.size();) {
        size_t j = i + 1;
        while (j < grown.size() && grown[j] == grown[j - 1] + 1) ++j;
        const size_t off = (size_t)grown[i] * Q->maxp, n = (j - i) * (size_t)Q->maxp;
        QTRY(Q, cudaMemcpyAsync(Q->d_pages + off, &Q->h_pages[off], sizeof(int32_t) * n, cudaMemcpyHostToDevice,
                                Q->stream),
             "page table");
        i = j;
    }
    return LRM_OK;
}

lrm_status lrm_qwen_decode(lrm_qwen Q, int32_t batch, const int32_t *slots, const uint32_t *ids, uint32_t *next_ids,
                           float *logits) {
    LTRY(check_ready(Q));
    if ((Q->is_first && !ids) || (Q->is_last && !next_ids)) return qfail(Q, LRM_ERR_ARGUMENT, "null ids");
    if (Q->is_first)
        for (int b = 0; b < batch; ++b)
            if (ids[b] >= (uint32_t)Q->c.vocab) return qfail(Q, LRM_ERR_ARGUMENT, "an id is outside the vocabulary");
    LTRY(set_slots(Q, batch, slots));
    LTRY(ensure_pages(Q, batch, slots, 1));
    cudaStream_t st = Q->stream;
    if (Q->is_first) {
        memcpy(Q->h_pinned, ids, 4 * (size_t)batch);
        QTRY(Q, cudaMemcpyAsync(Q->ids, Q->h_pinned, 4 * (size_t)batch, cudaMemcpyHostToDevice, st), "ids");
    }
    cudaGraphExec_t use_graph = nullptr;  // a kept capture of this exact slot list, if any
    for (const auto &k : Q->kept)
        if ((int)k.slots.size() == batch && std::equal(k.slots.begin(), k.slots.end(), slots)) use_graph = k.exec;
    if (Q->is_first) Q->ids_slots.clear();
    if (use_graph) {
        QTRY(Q, cudaGraphLaunch(use_graph, st), "graph launch");
    } else {
        LTRY(decode_step(Q, batch));
        // as the captured step does: the next ids become the id buffer's contents, the input of a later replay
        if (Q->is_first && Q->is_last)
            QTRY(Q, cudaMemcpyAsync(Q->ids, Q->next, 4 * (size_t)batch, cudaMemcpyDeviceToDevice, st), "feedback");
    }
    if (Q->is_first && Q->is_last) Q->ids_slots.assign(slots, slots + batch);
    if (Q->is_last) {
        QTRY(Q, cudaMemcpyAsync(Q->h_pinned + batch, Q->next, 4 * (size_t)batch, cudaMemcpyDeviceToHost, st),
             "next");
        if (logits)
            QTRY(Q, cudaMemcpyAsync(logits, Q->partial, 4 * (size_t)batch * Q->c.vocab, cudaMemcpyDeviceToHost, st),
                 "logits");
    }
    LTRY(sync_check(Q));
    if (Q->is_last) memcpy(next_ids, Q->h_pinned + batch, 4 * (size_t)batch);
    for (int b = 0; b < batch; ++b) Q->h_seq_len[slots[b]] += 1;
    return LRM_OK;
}

lrm_status lrm_qwen_decode_graph(lrm_qwen Q, int32_t batch, const int32_t *slots, const uint32_t *first_ids,
                                 uint32_t flags) {
    LTRY(check_ready(Q));
    const bool timed = flags & LRM_QWEN_GRAPH_TIME_ATTENTION;
    if (timed && Q->attn_ev.empty()) {
        Q->attn_ev.resize(2 * Q->nl);
        for (auto &e : Q->attn_ev) QTRY(Q, cudaEventCreate(&e), "event");
    }
    LTRY(set_slots(Q, batch, slots));
    if (first_ids) {
        memcpy(Q->h_pinned, first_ids, 4 * (size_t)batch);
        QTRY(Q, cudaMemcpyAsync(Q->ids, Q->h_pinned, 4 * (size_t)batch, cudaMemcpyHostToDevice, Q->stream), "ids");
        Q->ids_slots.assign(slots, slots + batch);
    }
    LTRY(sync_check(Q));
    // a new capture replaces one of the same slot list, else the oldest once kKeptGraphs are kept
    for (size_t i = 0; i < Q->kept.size(); ++i)
        if ((int)Q->kept[i].slots.size() == batch && std::equal(Q->kept[i].slots.begin(), Q->kept[i].slots.end(), slots)) {
            cudaGraphExecDestroy(Q->kept[i].exec);
            Q->kept.erase(Q->kept.begin() + i);
            break;
        }
    if (Q->kept.size() >= lrm_qwen_s::kKeptGraphs) {
        cudaGraphExecDestroy(Q->kept.front().exec);
        Q->kept.erase(Q->kept.begin());
    }
    Q->graph = nullptr;
    cudaGraph_t g;
    QTRY(Q, cudaStreamBeginCapture(Q->stream, cudaStreamCaptureModeThreadLocal), "begin capture");
    lrm_status s = decode_step(Q, batch, timed);
    if (s == LRM_OK && Q->is_first && Q->is_last) {
        cudaError_t e = cudaMemcpyAsync(Q->ids, Q->next, 4 * (size_t)batch, cudaMemcpyDeviceToDevice, Q->stream);
        if (e != cudaSuccess) s = qcuda(Q, e, "feedback copy");
    }
    cudaError_t e = cudaStreamEndCapture(Q->stream, &g);
    if (s != LRM_OK) return s;
    QTRY(Q, e, "end capture");
    size_t nodes = 0;
    cudaGraphGetNodes(g, nullptr, &nodes);
    std::vector<cudaGraphNode_t> list(nodes);
    cudaGraphGetNodes(g, list.data(), &nodes);
    int kernels = 0;
    for (auto n : list) {
        cudaGraphNodeType t;
        if (cudaGraphNodeGetType(n, &t) == cudaSuccess && t == cudaGraphNodeTypeKernel) ++kernels;
    }
    e = cudaGraphInstantiate(&Q->graph, g, 0);
    cudaGraphDestroy(g);
    QTRY(Q, e, "graph instantiate");
    Q->kept.push_back({std::vector<int32_t>(slots, slots + batch), Q->graph});
    Q->graph_kernels = kernels;
    Q->graph_timed = timed;
    Q->graph_batch = batch;
    Q->graph_slots.assign(slots, slots + batch);
    return LRM_OK;
}

lrm_status lrm_qwen_decode_replay(lrm_qwen Q, int32_t steps) {
    LTRY(check_ready(Q));
    if (!Q->graph) return qfail(Q, LRM_ERR_STATE, "no decode graph captured");
    // The graph's input ids are its rows' previous next ids in the id buffer; a prefill or a decode call on other
    // slots since then has replaced them.
    if (Q->is_first && Q->is_last && Q->ids_slots != Q->graph_slots)
        return qfail(Q, LRM_ERR_STATE,
                     "the id buffer holds another call's ids: capture again with first ids, or decode these slots");
    // the graph reads its rows' slots from d_slots, which a decode call with another slot list may have replaced
    LTRY(set_slots(Q, Q->graph_batch, Q->graph_slots.data()));
    LTRY(ensure_pages(Q, Q->graph_batch, Q->graph_slots.data(), steps));
    for (int i = 0; i < steps; ++i) QTRY(Q, cudaGraphLaunch(Q->graph, Q->stream), "graph launch");
    for (int b = 0; b < Q->graph_batch; ++b) Q->h_seq_len[Q->graph_slots[b]] += steps;
    return LRM_OK;
}

lrm_status lrm_qwen_last_ids(lrm_qwen Q, uint32_t *ids) {
    if (!Q || !ids) return qfail(Q, LRM_ERR_ARGUMENT, "null argument");
    cudaSetDevice(Q->device);
    LTRY(sync_check(Q));
    QTRY(Q, cudaMemcpy(ids, Q->next, 4 * (size_t)(Q->graph_batch ? Q->graph_batch : 1), cudaMemcpyDeviceToHost),
         "ids");
    return LRM_OK;
}

lrm_status lrm_qwen_graph_kernels(lrm_qwen Q, int32_t *kernels) {
    if (!Q || !kernels) return LRM_ERR_ARGUMENT;
    if (!Q->graph) return qfail(Q, LRM_ERR_STATE, "no decode graph captured");
    *kernels = Q->graph_kernels;
    return LRM_OK;
}

lrm_status lrm_qwen_attention_ms(lrm_qwen Q, float *ms) {
    if (!Q || !ms) return LRM_ERR_ARGUMENT;
    if (!Q->graph || !Q->graph_timed) return qfail(Q, LRM_ERR_STATE, "no timed decode graph captured");
    cudaSetDevice(Q->device);
    LTRY(sync_check(Q));
    for (int l = 0; l < Q->nl; ++l)
        QTRY(Q, cudaEventElapsedTime(&ms[l], Q->attn_ev[2 * l], Q->attn_ev[2 * l + 1]), "event time");
    return LRM_OK;
}

lrm_status lrm_qwen_truncate(lrm_qwen Q, int32_t slot, int32_t len) {
    if (!Q || slot < 0 || slot >= Q->c.max_seqs) return qfail(Q, LRM_ERR_ARGUMENT, "slot out of range");
    cudaSetDevice(Q->device);
    LTRY(sync_check(Q));
    int32_t cur = 0;
    QTRY(Q, cudaMemcpy(&cur, Q->d_seq_len + slot, 4, cudaMemcpyDeviceToHost), "seq_len");
    if (len < 0 || len > cur) return qfail(Q, LRM_ERR_ARGUMENT, "truncate can only shorten a sequence");
    QTRY(Q, cudaMemcpy(Q->d_seq_len + slot, &len, 4, cudaMemcpyHostToDevice), "seq_len");
    Q->h_seq_len[slot] = len;
    return LRM_OK;
}

lrm_status lrm_qwen_sync(lrm_qwen Q) {
    if (!Q) return LRM_ERR_ARGUMENT;
    cudaSetDevice(Q->device);
    return sync_check(Q);
}

lrm_status lrm_qwen_stream(lrm_qwen Q, void **stream) {
    if (!Q || !stream) return LRM_ERR_ARGUMENT;
    *stream = (void *)Q->stream;
    return LRM_OK;
}

lrm_status lrm_qwen_residual(lrm_qwen Q, float **x, int64_t *rows) {
    if (!Q || !x) return qfail(Q, LRM_ERR_ARGUMENT, "null argument");
    *x = Q->x;
    if (rows) *rows = Q->c.max_tokens > Q->c.max_batch ? Q->c.max_tokens : Q->c.max_batch;
    return LRM_OK;
}

lrm_status lrm_qwen_stage(lrm_qwen Q, int32_t *first_layer, int32_t *end_layer) {
    if (!Q || !first_layer || !end_layer) return qfail(Q, LRM_ERR_ARGUMENT, "null argument");
    *first_layer = Q->first;
    *end_layer = Q->first + Q->nl;
    return LRM_OK;
}

lrm_status lrm_qwen_seq_len(lrm_qwen Q, int32_t slot, int32_t *len) {
    if (!Q || !len || slot < 0 || slot >= Q->c.max_seqs) return LRM_ERR_ARGUMENT;
    cudaSetDevice(Q->device);
    LTRY(sync_check(Q));
    QTRY(Q, cudaMemcpy(len, Q->d_seq_len + slot, 4, cudaMemcpyDeviceToHost), "seq_len");
    return LRM_OK;
}

}  // extern "C"
