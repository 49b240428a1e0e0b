/*
 * lrm_cuda.h -- the C ABI of liblrmcuda.so, the B200 (sm_100a) CUDA device for the LRM Qwen3 forward path.
 *
 * This is the native side of a new `Lrm.Gpu.Cuda` backend. It implements the reference's device/kernel contracts
 * (src/Lrm.Gpu.Core/Backend.fs:104-161: IGpuBackendProvider, IGpuBackend, IGpuHeap, ICommandList, IKernelSet) with
 * plain pointers, sizes and status codes, so a .NET host binds it with blittable P/Invoke (the idiom of
 * src/Lrm.Gpu.D3D12.Interop/Native.fs:11-28) and a Python host with ctypes. No torch or CUDA type crosses the ABI.
 *
 * Rules that hold for every entry point:
 *  - Every function returns an lrm_status; nothing throws across the ABI. LRM_ERR_CONTRACT is the reference's
 *    GpuContractException (Dispatch.fs:149-234 rules, once-only rules); LRM_ERR_CUDA is a device or API failure,
 *    the analogue of D3D12DeviceLostException (D3D12/Backend.fs:109). lrm_cuda_last_error gives the message.
 *  - Calls on one device come from one thread at a time; devices are independent (docs/contracts/gpu-backend.md,
 *    "Threading").
 *  - Host pointers passed in are owned by the caller and only read or written during the call.
 */
#ifndef LRM_CUDA_H
#define LRM_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define LRM_CUDA_ABI_VERSION 1

typedef enum lrm_status {
    LRM_OK = 0,
    LRM_ERR_CONTRACT = 1,      /* a contract rule is broken (GpuContractException) */
    LRM_ERR_CUDA = 2,          /* CUDA runtime/driver failure; the device may be lost */
    LRM_ERR_TIMEOUT = 3,       /* a wait ran past its limit, or a kernel's bounded wait gave up */
    LRM_ERR_ARGUMENT = 4,      /* a null handle/pointer or an impossible size */
    LRM_ERR_OUT_OF_MEMORY = 5, /* device memory allocation failed */
    LRM_ERR_STATE = 6,         /* call out of order: heap/table twice, list reused, ... */
    LRM_ERR_NO_DEVICE = 7,     /* no CUDA device with that index */
    LRM_ERR_FORMAT = 8         /* a file breaks its format (SafetensorsFormatException, Safetensors.fs:16) */
} lrm_status;

typedef struct lrm_device_s *lrm_device;   /* IGpuBackend (+ its IGpuHeap, created once) */
typedef struct lrm_cmdlist_s *lrm_cmdlist; /* ICommandList */

/* DeviceInfo (Backend.fs:9-27). */
typedef struct lrm_device_info {
    int32_t index;
    char name[256];         /* marketing name, e.g. "NVIDIA B200" */
    uint32_t vendor_id;     /* PCI vendor id, 0x10de */
    uint32_t pci_device_id; /* PCI device id from sysfs (0 when unreadable) */
    char driver[64];        /* kernel driver version, e.g. "580.159" */
    int64_t memory_bytes;
    int32_t sm_count;
    int32_t cc_major, cc_minor;
    int32_t accepted;       /* 1 when the device meets the requirements (sm_100 family) */
    char rejection[256];    /* why not, when accepted == 0 */
} lrm_device_info;

/* DeviceOptions flags (Backend.fs:30-55). */
#define LRM_CUDA_DEBUG 0x1u            /* synchronise and check after every dispatch */
#define LRM_CUDA_TIME_DISPATCHES 0x2u  /* time every dispatch; results follow the timers as gpu.dispatch */

/* Completion (Backend.fs:84-92). */
typedef struct lrm_completion {
    uint64_t fence;
    uint32_t dispatches;
    uint32_t timer_count; /* user timers in opening order, then one per dispatch with TIME_DISPATCHES */
} lrm_completion;

/* ---- library ------------------------------------------------------------------------------------------------ */

/* LRM_CUDA_ABI_VERSION of the loaded library. */
int32_t lrm_cuda_abi_version(void);

/* Copies the last error message of `dev` (or of the calling thread when dev is NULL) into buf; returns its length. */
size_t lrm_cuda_last_error(lrm_device dev, char *buf, size_t n);

/* ---- IGpuBackendProvider (Backend.fs:154-161) ---------------------------------------------------------------- */

/* Number of CUDA devices (Enumerate). */
lrm_status lrm_cuda_device_count(int32_t *count);

/* DeviceCandidate for one index: info plus accepted/rejection (Backend.fs:21-27). */
lrm_status lrm_cuda_device_info(int32_t index, lrm_device_info *out);

/* Create: a backend on device `index` with LRM_CUDA_* flags. */
lrm_status lrm_cuda_create(int32_t index, uint32_t flags, lrm_device *out);

/* Dispose: waits for outstanding work and frees every page, list and event. */
lrm_status lrm_cuda_destroy(lrm_device dev);

/* ---- IGpuBackend ---------------------------------------------------------------------------------------------- */

/* CreateHeap (Backend.fs:141, gpu-backend.md "IGpuBackend"): allocates the table (slot 0, 1 MiB) and pages 1..n of a
 * HeapLayout; arenas[i] is the ArenaKind code of page i+1. Exactly once. */
lrm_status lrm_cuda_create_heap(lrm_device dev, int32_t page_count, const uint32_t *arenas, const uint64_t *bytes);

/* LoadKernels (Backend.fs:143): the catalog kernels are compiled into the library for sm_100a; this marks them loaded
 * (exactly once) and returns the SHA-256 of the library's kernel set, the CUDA counterpart of ShaderSetHash. */
lrm_status lrm_cuda_load_kernels(lrm_device dev, uint8_t set_hash[32]);

/* IKernelSet.Contains (Backend.fs:96-100). */
lrm_status lrm_cuda_kernel_present(lrm_device dev, uint32_t kernel_id, int32_t *present);

/* Begin (Backend.fs:145): a new, empty command list. */
lrm_status lrm_cuda_begin(lrm_device dev, lrm_cmdlist *out);

/* Submit (Backend.fs:147): closes the list and enqueues it on the device's stream; *fence = 1, 2, 3, ... A list is
 * submitted once. The list handle stays valid (closed) until lrm_cuda_list_free or lrm_cuda_destroy. */
lrm_status lrm_cuda_submit(lrm_cmdlist list, uint64_t *fence);

/* Frees a command list handle (closed or not). */
lrm_status lrm_cuda_list_free(lrm_cmdlist list);

/* Wait (Backend.fs:149): blocks until `fence` completed or `timeout_ms` passed (LRM_ERR_TIMEOUT, the device stays
 * usable). Waiting again returns the same completion. */
lrm_status lrm_cuda_wait(lrm_device dev, uint64_t fence, uint32_t timeout_ms, lrm_completion *out);

/* One TimerResult of a completed submission (Backend.fs:70-79): the timer id (or 0x80000000 | kernel id for a
 * gpu.dispatch timing), start in ns from the device's creation, duration in ns. */
lrm_status lrm_cuda_timer_result(lrm_device dev, uint64_t fence, uint32_t index, uint32_t *timer_id,
                                 int64_t *start_ns, int64_t *duration_ns);

/* The fp32 denormal probe (Backend.fs:455-531, Fp32Denormals): runs scale_f32 with a = 0.5 over the 7 probe input
 * words on a private buffer and returns the 7 result words for the host to classify (preserve / flush / mixed). */
lrm_status lrm_cuda_denormal_probe(lrm_device dev, const uint32_t inputs[7], uint32_t results[7]);

/* ---- IGpuHeap (Backend.fs:102-116) ---------------------------------------------------------------------------- */

/* WriteTable: the sealed 1 MiB table image into slot 0, exactly once, before the first dispatch. */
lrm_status lrm_cuda_write_table(lrm_device dev, const void *image, uint64_t bytes);

/* Upload: host bytes into a page (slot 1..63); offset and size multiples of 4, inside the page. Waits for all
 * submitted work first and returns when the copy is done. UploadFrom is this call on chunks of at most 64 MiB. */
lrm_status lrm_cuda_upload(lrm_device dev, int32_t slot, uint64_t offset, const void *src, uint64_t bytes);

/* Download: page (or table, slot 0) bytes to the host; waits for all submitted work first. */
lrm_status lrm_cuda_download(lrm_device dev, int32_t slot, uint64_t offset, void *dst, uint64_t bytes);

/* ---- ICommandList (Backend.fs:118-134) ------------------------------------------------------------------------ */

/* Dispatch: records one catalog kernel with its 32-word argument block as Dispatch.prepare returned it (word 0 =
 * the physical groups in x). The library re-checks the block against the sealed table: kernel id, word rules, token
 * rows, dtypes, read-only and contiguity, aliasing, the catalog grid, and every minimum element count of
 * docs/contracts/kernel-abi.md, so a bad block is refused before any launch. */
lrm_status lrm_cuda_dispatch(lrm_cmdlist list, uint32_t kernel_id, const uint32_t words[32]);

/* Barrier: every earlier command's writes are visible to every later command. */
lrm_status lrm_cuda_barrier(lrm_cmdlist list);

/* Copy: bytes between pages (slots 1..63), equal positive sizes, multiples of 4, no overlap; a full barrier. */
lrm_status lrm_cuda_copy(lrm_cmdlist list, int32_t src_slot, uint64_t src_offset, int32_t dst_slot,
                         uint64_t dst_offset, uint64_t bytes);

/* BeginTimer / EndTimer: GPU-timed regions; timers nest and close in reverse order. */
lrm_status lrm_cuda_timer_begin(lrm_cmdlist list, uint32_t *timer_id);
lrm_status lrm_cuda_timer_end(lrm_cmdlist list, uint32_t timer_id);

/* ---- fast-path operators on device memory ------------------------------------------------------------------- */
/*
 * The bf16 forward path's operators, for callers that manage device memory themselves (the Qwen engine below, the
 * tests). Pointers are device addresses as uint64; `stream` is a cudaStream_t (NULL = the legacy default stream).
 * Each call checks its arguments (alignment, sizes) and launches asynchronously; a kernel whose bounded wait gave up
 * writes a nonzero code into the current device's error word (lrm_op_error_word).
 */

/* Makes `device` current for the calling thread and initialises its operator state. */
lrm_status lrm_op_set_device(int32_t device);

/* Reads the current device's error word (0 = no kernel reported an error); clears it when `clear` != 0. Codes:
 * 0x1xxx, 0x2001-0x2003, 0x3001-0x3009 a bounded wait that gave up (GEMM, decode attention, prefill attention);
 * 0x2010 a decode-attention row whose seq_len is below 1 or needs more pages than its page-table row (the row is
 * not read and its output is zeros); 0x3010 a prefill-attention sequence whose cu_seqlens rows fall outside
 * total_tokens or exceed max_len, or whose cached-token count is negative (the sequence is not computed and its
 * output rows are left unwritten). */
lrm_status lrm_op_error_word(uint32_t *code, int32_t clear);

/* Runs one kernel whose bounded in-kernel wait can never complete (an mbarrier nothing arrives on), with a limit of
 * `polls` polls (1 .. 2^24; the kernels' own limit is 2^24): the wait gives up, `code` (nonzero) lands in the error
 * word and the kernel returns, leaving the device usable. It exists to test the path every kernel of this library
 * takes when a wait runs out, the CUDA counterpart of the reference's device wait timeout
 * (src/Lrm.Gpu.D3D12/Backend.fs:109, Context.fs:200-234), without hanging or faulting a GPU. */
lrm_status lrm_op_wait_probe(void *stream, uint32_t polls, uint32_t code);

/* The engine's greedy pick as an operator: out[r] = the lowest index of the maximum of row r of logits (fp32
 * [rows][vocab], device; 16-byte aligned when vocab is a multiple of 4, which the kernel then reads as float4), or
 * 0xFFFFFFFF for a row holding a NaN: the argmax_rows contract (src/Lrm.Tensor.CpuReference/CpuRef.fs:452-466).
 * A row is scanned by a cluster of 8 CTAs; rows is at most 65535. */
lrm_status lrm_op_argmax_rows(void *stream, const float *logits, int32_t rows, int32_t vocab, uint32_t *out);

#define LRM_GEMM_F32 0     /* out_f32[m, n] = acc */
#define LRM_GEMM_RESID 1   /* out_f32[m, n] = resid[m, n] + acc (resid may equal out) */
#define LRM_GEMM_SWIGLU 2  /* b rows interleave gate/up in blocks of 64; out_bf16[m, n/2] = silu(gate) * up */
#define LRM_GEMM_PARTIAL 3 /* split-K partials, transposed: out_f32[split][n][m] */
#define LRM_GEMM_BF16 4    /* out_bf16[m, n] = acc */

/* D = A * B^T with A bf16 [m, k] and B bf16 [n, k] (both K-major) on tcgen05 tensor cores, fp32 accumulation in
 * TMEM, TMA-fed; replaces the reference's matmul_bf16w (src/Lrm.Shaders/hlsl/kernels/matmul/matmul_bf16w.hlsl) on the
 * bf16 path, with its epilogue fusions. */
typedef struct lrm_gemm_desc {
    int32_t m, n, k;
    uint64_t a, b;
    int32_t epilogue; /* LRM_GEMM_* */
    int32_t bn;       /* output tile width 64, 128 or 256; 0 chooses */
    int32_t splits;   /* split-K count; > 1 only with LRM_GEMM_PARTIAL */
    uint64_t out;     /* fp32, bf16 or partial output */
    int32_t ldo;      /* output leading dimension (elements); for PARTIAL the token stride, normally m */
    uint64_t resid;   /* RESID: fp32 [m, ldr] */
    int32_t ldr;
    uint64_t split_stride; /* PARTIAL: elements between split slices */
    int32_t cta_pair;      /* 0 chooses; 1 one CTA per 128-row tile; 2 two-SM clusters sharing 256 x 256 tiles
                              (tcgen05 cta_group::2; needs bn 256, one split, not PARTIAL) */
} lrm_gemm_desc;
lrm_status lrm_op_gemm_bf16(void *stream, const lrm_gemm_desc *desc);

/* A decode step's weight GEMM with its consumer fused, the form the engine's decode step runs: Y = W * B^T for
 * weights w bf16 [m, k] (m a multiple of 128) and n tokens b bf16 [n, k], K split over a thread-block cluster of
 * `splits` CTAs (1, 2, 3, 4, 8 or 16; 0 chooses) whose accumulators are added through distributed shared memory in
 * split order. Replaces the reference's matmul_bf16w (src/Lrm.Shaders/hlsl/kernels/matmul/matmul_bf16w.hlsl) plus the
 * add / rmsnorm_rows / silu_mul dispatches that follow it in a decode step.
 *   LRM_DEC_RESID   x [n][m] fp32 += Y; with gain (bf16 [m]) also u [n][m] = bf16(gain * x) and
 *                   ss_out[m / 128][t] (row stride ss_stride) = the sum of x^2 over each 128-column group: the next
 *                   RMSNorm's inputs;
 *   LRM_DEC_SWIGLU  the norm scale r[t] = 1 / sqrt(sum_g ss[g][t] / hidden + eps) (g < nss) applied to Y's rows, whose
 *                   weight rows interleave gate and up in blocks of 64; act [n][ld_act] bf16 = silu(r g) * (r u).
 * The q/k/v form (norm scale, QK-norm, RoPE, paged KV append) runs inside the engine only. */
#define LRM_DEC_SWIGLU 1
#define LRM_DEC_RESID 2
typedef struct lrm_decode_gemm_desc {
    int32_t m, n, k;
    uint64_t w, b;
    int32_t epilogue; /* LRM_DEC_* */
    int32_t splits;   /* 0 chooses */
    uint64_t ss;      /* SWIGLU: fp32 [nss][ss_stride] */
    int32_t nss, hidden;
    uint64_t ss_stride;
    float eps;
    uint64_t x, gain, u, ss_out; /* RESID */
    uint64_t act;                /* SWIGLU */
    int32_t ld_act;
} lrm_decode_gemm_desc;
lrm_status lrm_op_decode_gemm(void *stream, const lrm_decode_gemm_desc *desc);

/* Causal GQA attention of packed sequences (each starting at position 0), bf16 in/out, fp32 softmax and
 * accumulation: q [T, q_heads, 128], k/v [T, kv_heads, 128] (K after QK-norm and RoPE), cu_seqlens int32 [nseq + 1]
 * (device, cu_seqlens[nseq] = total_tokens = T), out [T, q_heads, 128]. Runs on the tcgen05 tensor cores (TMA tiles,
 * TMEM accumulators). Replaces the reference's attention_gqa_causal
 * (src/Lrm.Shaders/hlsl/kernels/attention/attention_gqa_causal.hlsl) for prefill on the bf16 path. */
typedef struct lrm_prefill_attn_desc {
    uint64_t q, k, v, out, cu_seqlens;
    int32_t nseq, max_len, q_heads, kv_heads, head_dim, total_tokens;
    float scale;
} lrm_prefill_attn_desc;
lrm_status lrm_op_prefill_attention(void *stream, const lrm_prefill_attn_desc *desc);

/* Decode attention, one query per row, over the paged bf16 KV cache: pool [pages][kv_heads][2][16][128] (K then V
 * of a page and head, 8 KiB), page_table int32 [seqs][pages_per_seq], seq_len int32 [seqs] (keys per sequence,
 * the new one included), slots int32 [batch] (device). q/out bf16 [batch][q_heads][128]; q_heads = 2 kv_heads.
 * Each CTA streams pages_per_split pages of one (row, kv head); the splits' partial softmax states go to
 * `workspace` (lrm_op_decode_attention_workspace bytes, 16-byte aligned) and a second kernel merges them; with one
 * split a row (pages_per_split >= pages_per_seq) the attention kernel writes the output itself. The kernels check
 * each row's seq_len against its page-table row (error word 0x2010), but not the values inside the device arrays
 * that index memory: every slots[b] must be a row of page_table, and every page id a row reads (its first
 * ceil(seq_len / 16) entries) a page of pool, as for any pointer the caller passes (neither count is in the
 * descriptor). */
typedef struct lrm_decode_attn_desc {
    uint64_t q, pool, page_table, seq_len, slots, out, workspace;
    int32_t batch, q_heads, kv_heads, head_dim, pages_per_seq, pages_per_split;
    float scale;
} lrm_decode_attn_desc;
uint64_t lrm_op_decode_attention_workspace(int32_t batch, int32_t kv_heads, int32_t pages_per_seq,
                                           int32_t pages_per_split);
lrm_status lrm_op_decode_attention(void *stream, const lrm_decode_attn_desc *desc);

/* Decode attention that allocates nothing. No counterpart in the reference: it is for callers that cannot allocate
 * device memory (a host that sizes all of its device memory once up front and never allocates per call; a serving
 * loop with a fixed memory budget; code inside a stream capture or a host callback, where cudaMalloc is not
 * allowed), and so cannot provide lrm_op_decode_attention's workspace. It runs the same kernels with their split-K scratch in
 * a 16 MiB array built into the library (every GPU that loads the library holds it until the process exits).
 * desc->workspace must be 0. A call needing more than LRM_DECODE_ATTN_STATIC_SCRATCH_BYTES of scratch
 * (lrm_op_decode_attention_workspace) is refused with LRM_ERR_ARGUMENT. The first call on a device looks up the
 * array's device address with that device current; make it before any stream capture. Nothing in the scratch must
 * start at zero. All calls on a device share the array, so calls that overlap on the GPU race on it. The address is
 * kept for the life of the process: after cudaDeviceReset (or any loss of the device's context) it is stale, as is
 * the device's error word, so a process that resets a device must not call the library's operators on it again. */
#define LRM_DECODE_ATTN_STATIC_SCRATCH_BYTES (16u << 20)
lrm_status lrm_op_decode_attention_static(void *stream, const lrm_decode_attn_desc *desc);

/* ---- the Qwen3 forward engine (bf16 fast path) ---------------------------------------------------------------- */
/*
 * The executor the reference plans but does not have (src/Lrm.Gpu.Exec/Placeholder.fs:1,
 * src/Lrm.Models.Qwen/Placeholder.fs:1; schedule of tests/Lrm.Tensor.Tests/TinyModel.fs:144-236): a whole-model
 * Qwen3 decoder forward on one device, bf16 weights and activations, fp32 residual stream and accumulation, bf16
 * paged KV cache (16-token pages) shared by `max_seqs` sequence slots. Prefill runs sequences packed together; a
 * decode step runs one token for each of `batch` slots. Host entry points copy their inputs in and results out;
 * the *_graph / *_replay pair runs decode steps with every input resident on the device (ids fed back on device).
 * Requirements: head_dim 128, q_heads = 2 kv_heads, hidden and intermediate multiples of 128.
 */
typedef struct lrm_qwen_s *lrm_qwen;

typedef struct lrm_qwen_config {
    int32_t layers, hidden, q_heads, kv_heads, head_dim, intermediate, vocab;
    float eps;
    int32_t max_pos;    /* longest sequence (RoPE table rows) */
    int32_t max_seqs;   /* sequence slots */
    int32_t kv_pages;   /* 16-token pages in the KV pool */
    int32_t max_tokens; /* tokens of one prefill call */
    int32_t max_batch;  /* rows of one decode step */
} lrm_qwen_config;

lrm_status lrm_qwen_create(int32_t device, const lrm_qwen_config *config, lrm_qwen *out);

/* A pipeline stage (the reference's stage split, docs/dev-plan.md "StagePipeline": stage 0 runs embed plus layers
 * 0-13, stage 1 layers 14-27 and the head, with the fp32 residual crossing between them): an engine holding layers
 * [first_layer, end_layer) of the `config->layers`-layer model and their KV cache. The first stage (first_layer 0)
 * embeds ids; the last (end_layer == layers) applies the final norm and the tied head; set_weight and
 * load_safetensors skip the weights of other stages. Prefill and decode on a stage:
 *  - a stage that is not the first reads its input residual from rows [0, T) of lrm_qwen_residual (T = the call's
 *    tokens, in the call's order), which the caller writes before the call (ordered on lrm_qwen_stream or
 *    synchronised); `ids` may be NULL;
 *  - a stage that is not the last leaves its output residual in the same rows; `next_ids` and `logits` may be NULL.
 * The split forward is bit-identical to the unsplit one. lrm_qwen_create is lrm_qwen_create_stage(0, layers). */
lrm_status lrm_qwen_create_stage(int32_t device, const lrm_qwen_config *config, int32_t first_layer,
                                 int32_t end_layer, lrm_qwen *out);
/* The stage's layer range. */
lrm_status lrm_qwen_stage(lrm_qwen q, int32_t *first_layer, int32_t *end_layer);
/* The device pointer of the fp32 residual x [rows][hidden] (rows = max(max_tokens, max_batch)). */
lrm_status lrm_qwen_residual(lrm_qwen q, float **x, int64_t *rows);
lrm_status lrm_qwen_destroy(lrm_qwen q);

/* Copies one HF-named bf16 weight (e.g. "model.layers.3.self_attn.q_proj.weight") from host memory into the engine's
 * layout: q/k/v fused into one [q+2kv heads, hidden] matrix, gate/up interleaved in blocks of 64 rows. */
lrm_status lrm_qwen_set_weight(lrm_qwen q, const char *name, const uint16_t *bf16, uint64_t count);

/* The RoPE table (T_spec, lrm_rope_table), float32 [rows, half]. rows >= max_pos, half = head_dim / 2. */
lrm_status lrm_qwen_set_rope(lrm_qwen q, const float *cos_t, const float *sin_t, int32_t rows, int32_t half);

/* Frees a slot's pages and sets its length to 0. */
lrm_status lrm_qwen_reset_seq(lrm_qwen q, int32_t slot);

/* Makes sure slot holds pages for `tokens` positions (so later decode steps need no host work). */
lrm_status lrm_qwen_reserve(lrm_qwen q, int32_t slot, int32_t tokens);

/* Prefill of `nseq` fresh sequences into slots[i] with lens[i] tokens each, ids concatenated (host). Writes each
 * sequence's next greedy id (host, [nseq]) and, when logits is not NULL, its last-row logits (host, [nseq, vocab]). */
lrm_status lrm_qwen_prefill(lrm_qwen q, int32_t nseq, const int32_t *slots, const int32_t *lens, const uint32_t *ids,
                            uint32_t *next_ids, float *logits);

/* Chunked prefill: like lrm_qwen_prefill, but each sequence's lens[i] tokens continue the tokens slots[i] already
 * holds (from a prefill, decode steps or earlier extends; a slot holding none starts at 0), attending to all of them.
 * Splitting a prompt into chunks gives the same ids and logits, bit for bit, as one prefill of the whole prompt. */
lrm_status lrm_qwen_extend(lrm_qwen q, int32_t nseq, const int32_t *slots, const int32_t *lens, const uint32_t *ids,
                           uint32_t *next_ids, float *logits);

/* One decode step: token ids[b] (host) appended to slots[b]; next greedy ids (host, [batch]) and optional logits
 * (host, [batch, vocab]). Uses the captured graph when one exists for the same slots. */
lrm_status lrm_qwen_decode(lrm_qwen q, int32_t batch, const int32_t *slots, const uint32_t *ids, uint32_t *next_ids,
                           float *logits);

/* Captures the decode step for `slots` as a CUDA graph whose input ids are the previous step's outputs (a
 * pipeline stage's graph reads its inputs as lrm_qwen_decode supplies them). The engine keeps the 8 most recent
 * captures by slot list; lrm_qwen_decode replays the one whose slots match its call, and the most recent one is
 * what lrm_qwen_decode_replay, lrm_qwen_last_ids and the attention timers use. With
 * LRM_QWEN_GRAPH_TIME_ATTENTION in flags, the graph also records CUDA events around every layer's decode attention,
 * read back by lrm_qwen_attention_ms after a replay. */
#define LRM_QWEN_GRAPH_TIME_ATTENTION 0x1u
lrm_status lrm_qwen_decode_graph(lrm_qwen q, int32_t batch, const int32_t *slots, const uint32_t *first_ids,
                                 uint32_t flags);

/* Kernel launches in one replay of the captured decode step (its kernel nodes). */
lrm_status lrm_qwen_graph_kernels(lrm_qwen q, int32_t *kernels);

/* After a replay of a graph captured with LRM_QWEN_GRAPH_TIME_ATTENTION: the decode-attention time of each layer
 * (ms, [layers]) in that replay. Waits for the stream. */
lrm_status lrm_qwen_attention_ms(lrm_qwen q, float *ms);

/* Sets a slot's length back to `len` (<= its current length), keeping its pages: later steps overwrite the cache
 * from position len on. */
lrm_status lrm_qwen_truncate(lrm_qwen q, int32_t slot, int32_t len);

/* Replays the captured step `steps` times on the engine's stream (asynchronous; lrm_qwen_sync waits). The step's
 * input ids are its rows' previous next ids, held in the engine's id buffer: after a prefill, or a decode call on
 * other slots, the buffer holds other ids, and a replay is refused (LRM_ERR_STATE) until the graph's slots are
 * decoded again or captured again with first ids. */
lrm_status lrm_qwen_decode_replay(lrm_qwen q, int32_t steps);

/* Device ids of the last replayed step (host copy, [batch]). */
lrm_status lrm_qwen_last_ids(lrm_qwen q, uint32_t *ids);

/* Waits for the engine's stream; returns LRM_ERR_TIMEOUT when a kernel reported a bounded-wait timeout. */
lrm_status lrm_qwen_sync(lrm_qwen q);

/* The engine's CUDA stream (cudaStream_t), for event timing. */
lrm_status lrm_qwen_stream(lrm_qwen q, void **stream);

/* Current length of a slot. */
lrm_status lrm_qwen_seq_len(lrm_qwen q, int32_t slot, int32_t *len);

/* Loads every tensor of a safetensors checkpoint (HF names, as lrm_qwen_set_weight takes them) into the engine,
 * streaming it from the memory-mapped file through two pinned 64 MiB buffers on the engine's stream. BF16 tensors are
 * copied as they are; F32 tensors are narrowed to bf16 (round to nearest even). A name that is not a weight of this
 * model, another dtype or a wrong element count is refused (LRM_ERR_ARGUMENT) before anything of that tensor is
 * copied; a malformed file gives LRM_ERR_FORMAT. `loaded` (may be null) receives the number of tensors loaded.
 * Replaces the reference's streamed SafetensorsFile reads with 64 MiB UploadFrom (Safetensors.fs:504-727,
 * docs/contracts/gpu-backend.md:56). */
lrm_status lrm_qwen_load_safetensors(lrm_qwen q, const char *path, int32_t *loaded);

/* ---- safetensors reader (SafetensorsFile, src/Lrm.Tensor/Safetensors.fs:231-727) --------------------------------
 * Open maps the file read-only and validates the whole header before anything is returned: the 8-byte length
 * (<= 100,000,000 and within the file), strict UTF-8 and JSON (depth <= 8, \u escapes forming valid Unicode), no
 * duplicate key, __metadata__ an object of strings, every tensor with exactly dtype / shape / data_offsets, its byte
 * count equal to the shape's, and the tensors tiling the data section exactly. Failures are LRM_ERR_FORMAT with a
 * message naming the file (lrm_cuda_last_error(NULL, ...)). Entries and metadata come in code point order of their
 * names. Pointers returned (names, shapes, data) stay valid until lrm_st_close. Needs no GPU. */
typedef struct lrm_st_file_s *lrm_st_file;
typedef enum lrm_st_dtype {
    LRM_ST_F32 = 0, LRM_ST_F64 = 1, LRM_ST_BF16 = 2, LRM_ST_F16 = 3,
    LRM_ST_I32 = 4, LRM_ST_U32 = 5, LRM_ST_U8 = 6, LRM_ST_I64 = 7
} lrm_st_dtype;
typedef struct lrm_st_entry {
    const char *name;     /* UTF-8 */
    int32_t dtype;        /* lrm_st_dtype */
    int32_t rank;
    const int64_t *shape; /* [rank] */
    uint64_t begin, end;  /* byte offsets within the data section */
    const void *data;     /* the tensor's bytes in the mapped file */
} lrm_st_entry;

lrm_status lrm_st_open(const char *path, lrm_st_file *out);
lrm_status lrm_st_close(lrm_st_file f);
/* Validates a file image in memory (SafetensorsFile.Validate): header length and tensor count on success. */
lrm_status lrm_st_validate(const void *bytes, uint64_t length, uint64_t *header_len, int64_t *count);
/* File length, header length N (the data section starts at 8 + N), tensor and metadata counts, and whether the data
 * section starts at a multiple of 8 with every tensor at a multiple of its element size (IsAligned). */
lrm_status lrm_st_info(lrm_st_file f, uint64_t *length, uint64_t *header_len, int64_t *count, int64_t *metadata_count,
                       int32_t *aligned);
lrm_status lrm_st_entry_at(lrm_st_file f, int64_t index, lrm_st_entry *out);
/* LRM_ERR_ARGUMENT when the file has no tensor of that name. */
lrm_status lrm_st_find(lrm_st_file f, const char *name, lrm_st_entry *out);
lrm_status lrm_st_metadata_at(lrm_st_file f, int64_t index, const char **key, const char **value);

/* ---- tokenizer (host; needs no GPU) --------------------------------------------------------------------------
 * The Qwen3 byte-level BPE tokenizer on the ends of the path (src/Lrm.Tokenizer/QwenTokenizer.fs:19-235): exact id
 * parity with HF tokenizers 0.23.3 on Qwen3's tokenizer.json. Text crosses the ABI as UTF-8. Calls that produce a
 * variable-length result take (out, cap, count): out null asks for the count only; a cap below the count is
 * LRM_ERR_ARGUMENT with nothing written. A handle is immutable apart from its piece cache, and every call on it is
 * safe from many threads at once. */
typedef struct lrm_tokenizer_s *lrm_tokenizer;

/* QwenTokenizer.fromJson (QwenTokenizer.fs:237-309, TokenizerJson.fs:219-250): parses and checks tokenizer.json.
 * Anything but Qwen3's configuration (NFC, the exact Split regex, ByteLevel without prefix space or regex, plain
 * BPE, added tokens matched on the raw text) is LRM_ERR_FORMAT with the reference's "tokenizer.json: ..." message. */
lrm_status lrm_tok_parse(const void *json, uint64_t json_bytes, lrm_tokenizer *out);
lrm_status lrm_tok_free(lrm_tokenizer t);
/* VocabSize (vocabulary + added tokens), MergeCount, AddedTokens.Length (QwenTokenizer.fs:85-91). */
lrm_status lrm_tok_info(lrm_tokenizer t, int32_t *vocab_size, int32_t *merges, int32_t *added);
/* ClearCache and CachedPieces (QwenTokenizer.fs:218-222): the piece cache holds two generations of at most 32,768
 * pieces or 1 Mi UTF-16 units each; pieces over 65,536 units are never cached; it never changes a result. */
lrm_status lrm_tok_clear_cache(lrm_tokenizer t);
lrm_status lrm_tok_cached_pieces(lrm_tokenizer t, int64_t *pieces);
/* The i-th added token by id; `content` stays valid until lrm_tok_free. */
lrm_status lrm_tok_added_at(lrm_tokenizer t, int32_t i, int32_t *id, const char **content, int32_t *special);
/* Encode (QwenTokenizer.fs:97): LRM_ERR_ARGUMENT when `utf8` is not valid UTF-8 (the reference's lone-surrogate
 * refusal; surrogates cannot be encoded in valid UTF-8). Adds no BOS or EOS. */
lrm_status lrm_tok_encode(lrm_tokenizer t, const char *utf8, uint64_t n, int32_t *ids, uint64_t cap,
                          uint64_t *count);
/* EncodeBytes (QwenTokenizer.fs:130): `bytes` decoded with one U+FFFD per maximal invalid subpart, then Encode. */
lrm_status lrm_tok_encode_bytes(lrm_tokenizer t, const uint8_t *bytes, uint64_t n, int32_t *ids, uint64_t cap,
                                uint64_t *count);
/* DecodeBytes (QwenTokenizer.fs:139): ids from VocabSize to 151,935 add nothing; an id below 0 or at 151,936 and
 * above is LRM_ERR_ARGUMENT. */
lrm_status lrm_tok_decode_bytes(lrm_tokenizer t, const int32_t *ids, uint64_t n, uint8_t *out, uint64_t cap,
                                uint64_t *len);
/* Decode (QwenTokenizer.fs:195): DecodeBytes as UTF-8 with one U+FFFD per maximal invalid subpart. */
lrm_status lrm_tok_decode(lrm_tokenizer t, const int32_t *ids, uint64_t n, char *out, uint64_t cap, uint64_t *len);
/* IdOf (QwenTokenizer.fs:200): an added token's content or a byte-level vocabulary string; -1 when there is none. */
lrm_status lrm_tok_id_of(lrm_tokenizer t, const char *token, int32_t *id);
/* TokenOf (QwenTokenizer.fs:209): `found` 0 for ids that have no token. */
lrm_status lrm_tok_token_of(lrm_tokenizer t, int32_t id, char *out, uint64_t cap, uint64_t *len, int32_t *found);
/* The stages on their own: Nfc.normalize (Nfc.fs), PreTokenizer.split (PreTokenizer.fs) as the byte offsets where
 * pieces end, CharClass.ofScalar (CharClass.fs; 0 letter, 1 number, 2 white space, 3 other, -1 past U+10FFFF), the
 * letter a scalar stands for in (?i:'s|'t|'re|'ve|'m|'ll|'d) (0 for none), and ByteLevel.charOf (ByteLevel.fs). */
lrm_status lrm_tok_nfc(const char *utf8, uint64_t n, char *out, uint64_t cap, uint64_t *len);
lrm_status lrm_tok_split(const char *utf8, uint64_t n, uint64_t *ends, uint64_t cap, uint64_t *count);
int32_t lrm_tok_char_class(uint32_t scalar);
int32_t lrm_tok_contraction_letter(uint32_t scalar);
uint32_t lrm_tok_byte_char(uint8_t byte);

/* ---- host helpers ------------------------------------------------------------------------------------------- */

/* T_spec (src/Lrm.Tensor.CpuReference/Rope.fs:163-251): cos/sin [max_pos, half] float32 with
 * freq = f32(f32(pos) * inv_freq[j]) and the correctly rounded float64 cos/sin rounded to float32. Every rounding is
 * certified; LRM_ERR_ARGUMENT when one cannot be (never seen for the tiny and Qwen3 tables). Needs no GPU. */
lrm_status lrm_rope_table(const uint32_t *inv_freq_bits, int32_t half, int32_t max_pos, float *cos_out,
                          float *sin_out);

#ifdef __cplusplus
}
#endif

#endif /* LRM_CUDA_H */
