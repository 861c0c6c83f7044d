/*
 * laya_gpu.h -- C ABI of the B200 (sm_100a) forward pass for the Laya mmBERT
 * decision encoder (mmBERT-base encoder + 2-layer decision head + option
 * scorer + act/escalate head).
 *
 * This is the boundary at which li-ming1/laya-zig's host program hands its
 * hot path to the GPU. Reference interfaces replaced (paths within the
 * laya-zig project):
 *
 *   laya_gpu_create          loadModel            src/main.zig:2311-2404
 *                            (weights by safetensors name, main.zig:2344-2397;
 *                            errors MissingTensor 1332, UnsupportedDtype 1354,
 *                            BadSafetensors 1359)
 *   laya_gpu_forward         forward(alloc, *FwdCtx) src/main.zig:2641-2817
 *                            (FwdCtx fields ids, L, qtype, markers, logits,
 *                            act, pooled: main.zig:2529-2541; hidden state
 *                            left in f.s.x, main.zig:2266-2294)
 *   laya_gpu_forward_trace   --dumpstats          src/main.zig:113-121, 2651-2777
 *   laya_gpu_forward_dumpstats  (the same, as the reference's [dump] text)
 *   laya_gpu_linear          linear16             src/main.zig:1088-1099
 *                            (checked by --selftest, main.zig:420-536)
 *
 * All pointers are plain host or device pointers; no C++ or framework types
 * cross this boundary. Every call returns a laya_status; after a failure,
 * laya_gpu_last_error() describes it. A context belongs to one device and is
 * externally synchronised (one calling thread at a time), as the reference's
 * forward() is; separate contexts may be driven from separate threads.
 */
#ifndef LAYA_GPU_H
#define LAYA_GPU_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define LAYA_GPU_ABI_VERSION 1

#if defined(__GNUC__)
#define LAYA_API __attribute__((visibility("default")))
#else
#define LAYA_API
#endif

/* Architecture constants (src/main.zig:39-57). */
#define LAYA_HIDDEN 768
#define LAYA_VOCAB 256000
#define LAYA_MAX_LEN 32768        /* longest sequence accepted (RoPE table rows) */
#define LAYA_MAX_MARKERS 1024     /* option markers per sequence */
#define LAYA_TRACE_TAGS 27        /* emb, l0..l21, final, temb, h0, h1 */

typedef enum {
    LAYA_OK = 0,
    LAYA_ERR_ARG = -1,            /* bad argument: id >= vocab, marker >= L, L == 0, qtype > 2 ... */
    LAYA_ERR_MISSING_TENSOR = -2, /* error.MissingTensor (src/main.zig:1332) */
    LAYA_ERR_DTYPE = -3,          /* error.UnsupportedDtype (src/main.zig:1354) */
    LAYA_ERR_SHAPE = -4,          /* element count does not match the architecture */
    LAYA_ERR_OOM = -5,            /* device allocation failed */
    LAYA_ERR_CUDA = -6,           /* CUDA runtime / driver error */
    LAYA_ERR_TIMEOUT = -7,        /* a kernel gave up waiting (bounded device-side wait) */
    LAYA_ERR_NO_DEVICE = -8,      /* no sm_100 device at that index */
} laya_status;

/* Tensor element types, as safetensors names them. */
typedef enum { LAYA_DT_F32 = 0, LAYA_DT_F16 = 1, LAYA_DT_BF16 = 2 } laya_dtype;

/* GEMM operand precision on the device (weights and the activations that
 * feed the tensor cores; the residual stream and every norm stay f32). */
typedef enum { LAYA_PREC_BF16 = 0, LAYA_PREC_F16 = 1 } laya_precision;

/* One checkpoint tensor, borrowed for the duration of laya_gpu_create. */
typedef struct {
    const char* name;   /* safetensors name, e.g. "encoder.layers.3.attn.Wqkv.weight" */
    int32_t dtype;      /* laya_dtype */
    const void* data;   /* host pointer, row-major as stored */
    uint64_t numel;     /* element count */
} laya_tensor;

typedef struct laya_ctx laya_ctx;

/* One sequence of a host batch (the reference's Seq, src/main.zig:2837-2841). */
typedef struct {
    const uint32_t* ids;      /* [len] token ids < LAYA_VOCAB */
    uint32_t len;             /* 1 .. LAYA_MAX_LEN */
    const uint32_t* markers;  /* [n_markers] positions of the option [MASK] tokens, each < len */
    uint32_t n_markers;       /* 0 .. LAYA_MAX_MARKERS */
    uint32_t qtype;           /* 0 choice, 1 score, 2 noul */
} laya_seq;

/* A packed batch whose arrays already live in device memory. */
typedef struct {
    const uint32_t* ids;        /* [n_tokens], sequences back to back */
    const int32_t* cu_seqlens;  /* [n_seqs + 1] token offsets, cu_seqlens[0] = 0 */
    const uint32_t* markers;    /* [n_markers] per-sequence positions, sequences back to back */
    const int32_t* cu_markers;  /* [n_seqs + 1] marker offsets */
    const uint32_t* qtypes;     /* [n_seqs] */
    uint32_t n_seqs, n_tokens, n_markers;
    uint32_t max_len;           /* longest sequence (sizes the attention grid) */
} laya_batch;

LAYA_API int laya_gpu_version(void);

/* Number of CUDA devices visible to this process. */
LAYA_API int laya_gpu_device_count(void);

/* Upload a checkpoint to `device` and build a context. Every tensor that
 * loadModel reads must be present (extra ones are ignored); each may be F16,
 * BF16 or F32. Matrices are converted on the device to `precision`, small
 * tensors (norms, biases, scorer, act head, type embedding) to f32.
 * The host buffers are not retained. */
LAYA_API int laya_gpu_create(int device, const laya_tensor* tensors, int n_tensors, int precision, laya_ctx** out);

LAYA_API void laya_gpu_destroy(laya_ctx* ctx);

/* Text of the last failure on `ctx`; with ctx == NULL, of the last failed
 * context-free call (laya_gpu_create, laya_gpu_linear) on this thread.
 * Never NULL. */
LAYA_API const char* laya_gpu_last_error(const laya_ctx* ctx);

/* The drop-in for forward(): one sequence, host buffers, synchronous.
 * logits[K]; act[2] = (act, escalate) probabilities; pooled[768] = final
 * hidden state of token 0; hidden (nullable) [L][768] = final hidden state. */
LAYA_API int laya_gpu_forward(laya_ctx* ctx, const uint32_t* ids, uint32_t L, uint32_t qtype, const uint32_t* markers,
                     uint32_t K, float* logits, float* act, float* pooled, float* hidden);

/* Many independent sequences in one pass (varlen packed, no padding).
 * logits[sum K]; act[2 * n_seqs]; pooled (nullable) [n_seqs][768];
 * hidden (nullable) [sum L][768]. Synchronous. */
LAYA_API int laya_gpu_forward_batch(laya_ctx* ctx, const laya_seq* seqs, uint32_t n_seqs, float* logits, float* act,
                           float* pooled, float* hidden);

/* Same pass over a batch already in device memory; outputs are device
 * pointers (pooled, hidden nullable). Asynchronous on `stream`, a
 * cudaStream_t of the context's device (NULL = the legacy default stream,
 * as everywhere in CUDA); call laya_gpu_sync to wait and to collect
 * device-side errors. Inputs are not validated on the host; the kernels
 * check what they read: an id >= LAYA_VOCAB, a marker outside its sequence,
 * a qtype > 2, offset tables that are not runs of [0, n_tokens) and
 * [0, n_markers) in order (cu_seqlens[0] = cu_markers[0] = 0,
 * cu_seqlens[n_seqs] = n_tokens, cu_markers[n_seqs] = n_markers), a
 * sequence longer than max_len or with more than LAYA_MAX_MARKERS markers.
 * Such an input is clamped or skipped without any access outside the
 * buffers, and laya_gpu_sync returns LAYA_ERR_ARG. */
LAYA_API int laya_gpu_forward_device(laya_ctx* ctx, const laya_batch* batch, float* logits, float* act, float* pooled,
                            float* hidden, void* stream);

/* Wait for the context's work and report any device-side error. */
LAYA_API int laya_gpu_sync(laya_ctx* ctx);

/* forward() plus the hidden state after every stage the reference's
 * --dumpstats reports: trace[LAYA_TRACE_TAGS][L][768] in tag order emb,
 * l0..l21, final, temb, h0, h1. */
LAYA_API int laya_gpu_forward_trace(laya_ctx* ctx, const uint32_t* ids, uint32_t L, uint32_t qtype, const uint32_t* markers,
                           uint32_t K, float* logits, float* act, float* trace);

/* --dumpstats (src/main.zig:113-130, 2651-2777): forward() of one sequence
 * plus the text the reference prints for it, NUL-terminated, in its line
 * formats: "[dump] meta L=.. qtype=..", the ids eight per "[dump] ids" line,
 * one "[dump] <tag> x0 x1 x2 sum asum" line per tag (emb, l0..l21, final,
 * temb, h0, h1; the first three values of the hidden state and its sum and
 * absolute sum in f64, computed on the device), then "[dump] mark" and
 * "[dump] logit". *text_len (nullable) receives the bytes the text needs,
 * NUL included; if `cap` is smaller, nothing is written and LAYA_ERR_ARG is
 * returned (the forward has run and logits/act are filled). */
LAYA_API int laya_gpu_forward_dumpstats(laya_ctx* ctx, const uint32_t* ids, uint32_t L, uint32_t qtype,
                                        const uint32_t* markers, uint32_t K, float* logits, float* act, char* text,
                                        uint64_t cap, uint64_t* text_len);

/* The text part of laya_gpu_forward_dumpstats, host only (no device, no
 * context): stats[LAYA_TRACE_TAGS][5] = x[0], x[1], x[2], sum, absolute sum
 * per tag, formatted with ids, markers and logits into the reference's
 * `[dump]` lines (src/main.zig:113-130). Same `text`/`cap`/`text_len`
 * contract; a failure is described by laya_gpu_last_error(NULL). */
LAYA_API int laya_gpu_format_dump(const uint32_t* ids, uint32_t L, uint32_t qtype, const uint32_t* markers, uint32_t K,
                                  const float* logits, const double* stats, char* text, uint64_t cap,
                                  uint64_t* text_len);

/* Finer than --dumpstats: every intermediate of encoder layer `layer`
 * (0..21) for one sequence, as the GPU holds it. 16-bit buffers are raw
 * element bits of the context's precision. xn_attn[L][768] (attn_norm
 * output; layer 0: the embedding output), qkv[L][2304] (after RoPE),
 * ctx[L][768] (attention output), x_mid[L][768] f32 (after the attention
 * residual), xn_mlp[L][768] (mlp_norm output), glu[L][1152] (gelu(gate) *
 * up). Any output may be NULL. */
LAYA_API int laya_gpu_forward_dump(laya_ctx* ctx, const uint32_t* ids, uint32_t L, uint32_t qtype,
                                   const uint32_t* markers, uint32_t K, int layer, uint16_t* xn_attn, uint16_t* qkv,
                                   uint16_t* ctx_out, float* x_mid, uint16_t* xn_mlp, uint16_t* glu);

/* Stages of the forward, as the reference's --profile buckets them
 * (src/main.zig:132-198): one entry per kernel family. */
typedef enum {
    LAYA_STAGE_EMBED = 0,     /* embedding gather + norm */
    LAYA_STAGE_NORM = 1,      /* LayerNorms between projections */
    LAYA_STAGE_GEMM_QKV = 2,  /* QKV / in_proj projections (+ RoPE epilogue) */
    LAYA_STAGE_ATTN = 3,      /* attention */
    LAYA_STAGE_GEMM_OUT = 4,  /* attention-out projections (+ residual) */
    LAYA_STAGE_GEMM_UP = 5,   /* GLU Wi / head linear1 (+ GLU or ReLU) */
    LAYA_STAGE_GEMM_DOWN = 6, /* FFN-out / head linear2 (+ residual) */
    LAYA_STAGE_FINAL = 7,     /* final norm + type embedding (+ head norm1) */
    LAYA_STAGE_TAIL = 8,      /* scorer + act/escalate head */
    LAYA_N_STAGES = 9
} laya_stage;

/* --profile: capture one forward of a device batch as a CUDA graph with an
 * external event record node on either side of every kernel, then launch it
 * `iters` times on `stream` (a cudaStream_t, NULL = the legacy default
 * stream), so the kernels run back to back as in the timed path.
 * stage_ms[LAYA_N_STAGES] receives the summed kernel time per stage over all
 * iterations, stage_launches[LAYA_N_STAGES] the launches per forward.
 * Synchronous. */
LAYA_API int laya_gpu_forward_profile(laya_ctx* ctx, const laya_batch* batch, float* logits, float* act, int iters,
                                      void* stream, float* stage_ms, int* stage_launches);

/* The same capture, per launch: launch_ms[i] receives the summed time of the
 * forward's i-th timed launch (in launch order; the decision tail's three
 * kernels count as one) over all iterations, launch_stage[i] its laya_stage.
 * *n_launches (nullable) receives the count; at most `cap` are written.
 * Synchronous. */
LAYA_API int laya_gpu_forward_profile_launches(laya_ctx* ctx, const laya_batch* batch, float* logits, float* act,
                                               int iters, void* stream, float* launch_ms, int* launch_stage, int cap,
                                               int* n_launches);

/* The decision tail alone (option scorer + act/escalate head) over final
 * hidden states the caller already holds in device memory, allocating
 * nothing. No counterpart in the reference: it is for callers that cannot
 * let a library call cudaMalloc at decision time (a process that gives all
 * device memory to its own caching allocator, or a serving loop with a fixed
 * memory budget), which the other entry points may do when a batch outgrows
 * their workspace. Its scratch is a static device array sized for
 * LAYA_NOALLOC_MAX_MARKERS markers (6.4 MB, held by every GPU that loads
 * the library until exit); larger calls are rejected with LAYA_ERR_ARG.
 * hidden[cu_seqlens[n_seqs]][768] f32, cu_seqlens/cu_markers[n_seqs + 1],
 * markers[n_markers]; outputs logits[n_markers], act[2 * n_seqs],
 * pooled[n_seqs][768], all device pointers. As in laya_gpu_forward_device,
 * each sequence holds at most LAYA_MAX_MARKERS (1024) markers, and the
 * device-resident tables are checked by the kernels, not the host: a marker
 * outside its sequence, a sequence with more than 1024 markers or offsets
 * out of order (cu_markers[0] = 0, cu_markers[n_seqs] = n_markers) make
 * laya_gpu_sync return LAYA_ERR_ARG, with nothing read or written outside
 * the buffers. Asynchronous on `stream` (NULL = the legacy default stream);
 * the caller's current device is left as it was.
 * The first call on a device resolves the array's device address
 * (cudaGetSymbolAddress, which may load the module): make it before any
 * stream capture. Calls share the array: calls that overlap on the GPU race. */
#define LAYA_NOALLOC_MAX_MARKERS 2048
LAYA_API int laya_gpu_decision_tail_noalloc(laya_ctx* ctx, const float* hidden, const int32_t* cu_seqlens,
                                            const uint32_t* markers, const int32_t* cu_markers, uint32_t n_seqs,
                                            uint32_t n_markers, float* logits, float* act, float* pooled,
                                            void* stream);

/* One projection, device pointers: out[M][N] (f32) = x[M][K] . w[N][K]^T
 * (+ bias[N]); x and w 16-bit of `elem_dtype` (LAYA_DT_BF16 or LAYA_DT_F16).
 * N a multiple of 128, K a multiple of 128; device pointers 16-byte aligned.
 * Runs on `stream` (NULL = default stream) of the current device, ordered
 * after the work before it on that stream: x, w and bias may come from the
 * kernel just before. */
LAYA_API int laya_gpu_linear(const void* x, const void* w, const float* bias, float* out, int M, int N, int K,
                    int elem_dtype, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* LAYA_GPU_H */
