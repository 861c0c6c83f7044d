// laya_gpu.cu -- context, weight upload, forward driver and the C ABI.
//
// The forward pass is the reference's forward() (src/main.zig:2641-2817)
// restructured for the GPU: all sequences of a batch are packed back to back
// (varlen, no padding); every projection is one tcgen05 GEMM whose epilogue
// performs the elementwise job that follows it; one CUDA graph per batch
// shape replays the ~170 launches of a forward.
//
// Per encoder layer l (sliding = l % 3 != 0, main.zig:2366):
//   [ln]       xn  = LN(x; attn_norm)          (layer 0: xn = x, main.zig:2660-2665)
//   [gemm]     qkv = rope(xn Wqkv^T)           (2666-2671)
//   [attn]     ctx = attention(qkv, window)    (2673-2684)
//   [gemm]     x  += ctx Wo^T                  (2686-2688)
//   [ln]       xn  = LN(x; mlp_norm)           (2691)
//   [gemm]     g   = glu(xn Wi^T)              (2693-2695)
//   [gemm]     x  += g Wo2^T                   (2697-2699)
// then x = LN_final(x) + type_emb[qtype] with head norm1 fused (2708-2716),
// the two head layers (2714-2754: biases, no RoPE, full attention, ReLU FFN),
// and the tail (scorer, act head; 2756-2814).
#include <algorithm>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <string>
#include <tuple>
#include <vector>

#include "../../include/laya_gpu.h"
#include "attention.cuh"
#include "gemm.cuh"
#include "kernels.cuh"

using namespace laya;

namespace {

thread_local std::string g_create_error = "no error";

struct EncW {
    void *wqkv, *wo, *wi, *wo2;
    float *attn_norm, *mlp_norm;
    CUtensorMap m_qkv, m_wo, m_wi, m_wo2;
};

struct HeadW {
    float *n1w, *n1b, *n2w, *n2b, *in_b, *out_b, *l1_b, *l2_b;
    void *in_w, *out_w, *l1_w, *l2_w;
    CUtensorMap m_in, m_out, m_l1, m_l2;
};

struct GraphKey {
    int M, S, G, maxlen;
    const void *ids, *cu, *mk, *cum, *qt, *lg, *act, *pooled, *hidden;
    bool operator<(const GraphKey& o) const {
        return std::tie(M, S, G, maxlen, ids, cu, mk, cum, qt, lg, act, pooled, hidden) <
               std::tie(o.M, o.S, o.G, o.maxlen, o.ids, o.cu, o.mk, o.cum, o.qt, o.lg, o.act, o.pooled, o.hidden);
    }
};

}  // namespace

struct laya_ctx {
    int device = 0;
    bool bf16 = true;
    int num_sms = 148;
    size_t l2_persist = 0;     // persisting L2 set aside for this context (bytes)
    size_t l2_max_window = 0;  // largest access-policy window
    cudaStream_t stream = nullptr;
    std::string err = "no error";
    std::vector<void*> allocs;

    // weights
    void* emb = nullptr;
    float *emb_norm = nullptr, *final_norm = nullptr, *type_emb = nullptr;
    EncW enc[NL];
    HeadW head[HEAD_LAYERS];
    TailWeights tail{};
    float2* rope = nullptr;

    // workspace (capacities in tokens / sequences / markers)
    int capM = 0, capS = 0, capG = 0;
    std::vector<void*> ws;
    float* x = nullptr;
    void *xn = nullptr, *qkv = nullptr, *ctxb = nullptr, *mlp = nullptr, *ff = nullptr;
    float4* rope_tok = nullptr;  // [16][capM]: per-token RoPE pairs, frequency-major
    int* seq_of = nullptr;
    float *mv = nullptr, *partial = nullptr;
    // Staged batch inputs / outputs of the host-buffer entry points. d_in
    // holds ids | cu_seqlens | qtypes | markers | cu_markers packed for the
    // batch at hand, the same layout as the pinned staging buffer, so one
    // copy moves them; d_out holds act | logits, read back in one copy.
    uint32_t* d_in = nullptr;
    float* d_out = nullptr;
    float* d_pooled = nullptr;
    int* d_err = nullptr;
    int* h_err = nullptr;  // pinned
    double* d_stats = nullptr;  // [LAYA_TRACE_TAGS][5] --dumpstats fingerprints
    void* h_stage = nullptr;
    size_t h_stage_bytes = 0;

    std::map<GraphKey, cudaGraphExec_t> graphs;
};

namespace {

int fail(laya_ctx* c, int code, const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    if (c) c->err = buf;
    else g_create_error = buf;
    return code;
}

#define CK(call)                                                                                      \
    do {                                                                                              \
        cudaError_t e_ = (call);                                                                      \
        if (e_ != cudaSuccess)                                                                        \
            return fail(c, e_ == cudaErrorMemoryAllocation ? LAYA_ERR_OOM : LAYA_ERR_CUDA, "%s: %s (%s:%d)", \
                        #call, cudaGetErrorString(e_), __FILE__, __LINE__);                           \
    } while (0)

// Makes a context's device current for one entry point and gives the
// caller's current device back on return, so a call never changes which
// device the calling thread works on.
struct DeviceGuard {
    int prev = -1;
    cudaError_t set(int dev) {
        if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
        return cudaSetDevice(dev);
    }
    ~DeviceGuard() {
        if (prev >= 0) cudaSetDevice(prev);
    }
};

size_t elem_size(int dt) { return dt == LAYA_DT_F32 ? 4 : 2; }

const laya_tensor* find(const laya_tensor* t, int n, const char* name) {
    for (int i = 0; i < n; i++)
        if (t[i].name && strcmp(t[i].name, name) == 0) return &t[i];
    return nullptr;
}

int check_tensor(laya_ctx* c, const laya_tensor* t, int n, const char* name, uint64_t numel, const laya_tensor** out) {
    const laya_tensor* e = find(t, n, name);
    if (!e) return fail(c, LAYA_ERR_MISSING_TENSOR, "missing tensor: %s", name);
    if (e->dtype != LAYA_DT_F32 && e->dtype != LAYA_DT_F16 && e->dtype != LAYA_DT_BF16)
        return fail(c, LAYA_ERR_DTYPE, "tensor %s has dtype %d, expected F16, BF16 or F32", name, (int)e->dtype);
    if (e->numel != numel)
        return fail(c, LAYA_ERR_SHAPE, "tensor %s has %llu elements, expected %llu", name,
                    (unsigned long long)e->numel, (unsigned long long)numel);
    if (!e->data) return fail(c, LAYA_ERR_ARG, "tensor %s has no data", name);
    *out = e;
    return LAYA_OK;
}

int dev_alloc(laya_ctx* c, void** p, size_t bytes, std::vector<void*>& list) {
    cudaError_t e = cudaMalloc(p, bytes < 256 ? 256 : bytes);
    if (e != cudaSuccess) return fail(c, LAYA_ERR_OOM, "cudaMalloc(%zu): %s", bytes, cudaGetErrorString(e));
    list.push_back(*p);
    return LAYA_OK;
}

// Upload one tensor through a device staging buffer; matrices -> 16-bit
// (optionally GLU-interleaved), vectors -> f32.
int upload(laya_ctx* c, const laya_tensor* t, int n, const char* name, uint64_t rows, uint64_t cols, bool matrix,
           int glu_tile, void** dst, void* staging) {
    const laya_tensor* e;
    int rc = check_tensor(c, t, n, name, rows * cols, &e);
    if (rc) return rc;
    rc = dev_alloc(c, dst, rows * cols * (matrix ? 2 : 4), c->allocs);
    if (rc) return rc;
    // On the context's stream: a cudaMemcpy from pageable memory may return
    // before its DMA lands, and c->stream does not wait on the legacy stream.
    CK(cudaMemcpyAsync(staging, e->data, rows * cols * elem_size(e->dtype), cudaMemcpyHostToDevice, c->stream));
    if (matrix)
        CK(launch_convert16(*dst, c->bf16, staging, e->dtype, rows, cols, glu_tile, c->stream));
    else
        CK(launch_convert_f32(static_cast<float*>(*dst), staging, e->dtype, rows * cols, c->stream));
    CK(cudaStreamSynchronize(c->stream));
    return LAYA_OK;
}

int weight_map(laya_ctx* c, CUtensorMap* m, const void* w, uint64_t rows, uint64_t cols) {
    CUresult r = make_tmap_2d(m, w, cols, rows, 128, c->bf16);  // B operand box: 128 rows
    if (r != CUDA_SUCCESS) return fail(c, LAYA_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
    return LAYA_OK;
}

// Words of the packed batch inputs (ids, cu_seqlens, qtypes, markers,
// cu_markers) and outputs (act, logits); host outputs start at out_offset.
size_t in_words(int M, int S, int G) { return (size_t)M + (S + 1) + S + G + (S + 1); }
size_t out_words(int S, int G) { return (size_t)S * 2 + G; }
size_t out_offset(const laya_ctx* c) { return (in_words(c->capM, c->capS, c->capG) * 4 + 63) & ~(size_t)63; }

void free_workspace(laya_ctx* c) {
    for (auto& g : c->graphs) cudaGraphExecDestroy(g.second);
    c->graphs.clear();
    for (void* p : c->ws) cudaFree(p);
    c->ws.clear();
    c->capM = c->capS = c->capG = 0;
}

int ensure_workspace(laya_ctx* c, int M, int S, int G) {
    if (M <= c->capM && S <= c->capS && G <= c->capG) return LAYA_OK;
    const int nM = std::max(M, c->capM), nS = std::max(S, c->capS), nG = std::max(std::max(G, c->capG), 1);
    CK(cudaDeviceSynchronize());  // device-path work may be pending on a caller's stream
    free_workspace(c);
    const size_t e16 = 2;
    int rc = 0;
    auto A = [&](void** p, size_t bytes) { if (!rc) rc = dev_alloc(c, p, bytes, c->ws); };
    A((void**)&c->x, (size_t)nM * D * 4);
    A(&c->xn, (size_t)nM * D * e16);
    A(&c->qkv, (size_t)nM * 3 * D * e16);
    A(&c->ctxb, (size_t)nM * D * e16);
    A(&c->mlp, (size_t)nM * INTER * e16);
    A(&c->ff, (size_t)nM * HEAD_FF * e16);
    A((void**)&c->rope_tok, (size_t)nM * 16 * sizeof(float4));
    A((void**)&c->seq_of, (size_t)nM * 4);
    A((void**)&c->mv, (size_t)nG * D * 4);
    A((void**)&c->partial, (size_t)nG * SCORER_GROUPS * 4);
    A((void**)&c->d_in, in_words(nM, nS, nG) * 4);
    A((void**)&c->d_out, out_words(nS, nG) * 4);
    A((void**)&c->d_pooled, (size_t)nS * D * 4);
    if (rc) {
        free_workspace(c);
        return rc;
    }
    c->capM = nM;
    c->capS = nS;
    c->capG = nG;
    const size_t stage = out_offset(c) + out_words(nS, nG) * 4;
    if (stage > c->h_stage_bytes) {
        if (c->h_stage) cudaFreeHost(c->h_stage);
        c->h_stage = nullptr;
        CK(cudaMallocHost(&c->h_stage, stage));
        c->h_stage_bytes = stage;
    }
    return LAYA_OK;
}

struct Batch {  // device pointers + host-side shape
    const uint32_t* ids;
    const int* cu;
    const uint32_t* mk;
    const int* cum;
    const uint32_t* qt;
    int S, M, G, maxlen;
};

struct Outs {
    float *logits, *act, *pooled, *hidden;
};

// Tensor maps over the workspace for a batch of exactly M tokens: GEMM
// operand loads (zero-filled past M) and epilogue stores (clipped at M).
struct ActMaps {
    CUtensorMap a_xn, a_ctx, a_mlp, a_ff;  // A operands, box 128 x 64
    CUtensorMap o_qkv, o_mlp, o_ff, o_x;   // outputs, box 32 rows x 128 bytes
    CUtensorMap a_qkv;                     // tcgen05 attention's Q, K, V boxes, 128 x 64
    CUtensorMap a_qkv64;                   // mma.sync attention's Q, K, V boxes, 64 x 64
};

int build_maps(laya_ctx* c, int M, ActMaps* m) {
    CUresult r = make_tmap_2d(&m->a_xn, c->xn, D, M, 128, c->bf16);
    if (r == CUDA_SUCCESS) r = make_tmap_2d(&m->a_ctx, c->ctxb, D, M, 128, c->bf16);
    if (r == CUDA_SUCCESS) r = make_tmap_2d(&m->a_mlp, c->mlp, INTER, M, 128, c->bf16);
    if (r == CUDA_SUCCESS) r = make_tmap_2d(&m->a_ff, c->ff, HEAD_FF, M, 128, c->bf16);
    if (r == CUDA_SUCCESS) r = make_out_map(&m->o_qkv, c->qkv, 3 * D, M, 2, c->bf16);
    if (r == CUDA_SUCCESS) r = make_out_map(&m->o_mlp, c->mlp, INTER, M, 2, c->bf16);
    if (r == CUDA_SUCCESS) r = make_out_map(&m->o_ff, c->ff, HEAD_FF, M, 2, c->bf16);
    if (r == CUDA_SUCCESS) r = make_out_map(&m->o_x, c->x, D, M, 4, c->bf16);
    if (r == CUDA_SUCCESS) r = make_tmap_2d(&m->a_qkv, c->qkv, 3 * D, M, 128, c->bf16);
    if (r == CUDA_SUCCESS) r = make_tmap_2d(&m->a_qkv64, c->qkv, 3 * D, M, 64, c->bf16);
    if (r != CUDA_SUCCESS) return fail(c, LAYA_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
    return LAYA_OK;
}

cudaError_t gemm(laya_ctx* c, int epi, const CUtensorMap& a, const CUtensorMap& b, const CUtensorMap& out, int M,
                 int N, int K, const float* bias, int rope_cols, cudaStream_t s) {
    GemmArgs g{};
    g.M = M;
    g.N = N;
    g.K = K;
    g.bias = bias;
    g.rope_tok = c->rope_tok;
    g.rope_ld = c->capM;
    g.rope_cols = rope_cols;
    g.err = c->d_err;
    g.b_const = 1;  // B is one of the context's weights, written once at create
    return launch_gemm(epi, 256, c->bf16, a, b, out, g, c->num_sms, s);
}

// One attention layer. Global layers hand sequences of at least
// attention_tc_min_len() tokens to the tcgen05 kernel and the rest to the
// mma.sync kernel (per sequence, so a sequence's result does not depend on
// the batch it is in); sliding layers run the mma.sync kernel.
cudaError_t attention(laya_ctx* c, const Batch& b, const ActMaps& am, int window, cudaStream_t s) {
    const int tc_len = attention_tc_min_len();
    const bool tc = window < 0 && b.maxlen >= tc_len;
    cudaError_t e = launch_attention(c->bf16, am.a_qkv64, c->ctxb, b.cu, b.S, b.M, b.maxlen, window, c->d_err, s,
                                     tc ? tc_len : 0x7fffffff);
    if (e == cudaSuccess && tc)
        e = launch_attention_tc(c->bf16, am.a_qkv, c->ctxb, b.cu, b.S, b.M, b.maxlen, tc_len, c->d_err, s);
    return e;
}

// The whole forward on stream `s`. The hook sees begin(stage)/end(stage)
// around every kernel launch and tap(tag) after each --dumpstats point.
template <typename Hook>
cudaError_t run_forward(laya_ctx* c, const Batch& b, const Outs& o, const ActMaps& am, cudaStream_t s, Hook& hook) {
    cudaError_t e;
#define RUN(stage, x)                           \
    do {                                        \
        hook.begin(stage);                      \
        e = (x);                                \
        hook.end(stage);                        \
        if (e != cudaSuccess) return e;         \
    } while (0)
    const int M = b.M;
    L2Window l2w;
    if (c->l2_persist) {  // the residual stream x persists in L2 across the whole forward
        l2w.base = c->x;
        l2w.bytes = std::min((size_t)M * D * 4, c->l2_max_window);
        l2w.hit_ratio = std::min(1.0f, (float)c->l2_persist / (float)l2w.bytes);
    }
    L2WindowScope l2scope(l2w);
    RUN(LAYA_STAGE_EMBED,
        launch_embed(c->bf16, b.ids, b.cu, b.S, M, c->emb, c->emb_norm, c->x, c->xn, c->rope, c->rope_tok, c->capM,
                     c->seq_of, c->d_err, s));
    hook.tap(0);
    for (int l = 0; l < NL; l++) {
        const EncW& w = c->enc[l];
        if (w.attn_norm) RUN(LAYA_STAGE_NORM, launch_ln(c->bf16, c->x, c->xn, w.attn_norm, nullptr, M, c->num_sms, s));
        RUN(LAYA_STAGE_GEMM_QKV,
            gemm(c, EPI_QKV, am.a_xn, w.m_qkv, am.o_qkv, M, 3 * D, D, nullptr, 2 * D, s));
        RUN(LAYA_STAGE_ATTN, attention(c, b, am, (l % 3) ? WINDOW : -1, s));
        RUN(LAYA_STAGE_GEMM_OUT, gemm(c, EPI_RESID, am.a_ctx, w.m_wo, am.o_x, M, D, D, nullptr, 0, s));
        RUN(LAYA_STAGE_NORM, launch_ln(c->bf16, c->x, c->xn, w.mlp_norm, nullptr, M, c->num_sms, s));
        RUN(LAYA_STAGE_GEMM_UP,
            gemm(c, EPI_GLU, am.a_xn, w.m_wi, am.o_mlp, M, 2 * INTER, D, nullptr, 0, s));
        RUN(LAYA_STAGE_GEMM_DOWN, gemm(c, EPI_RESID, am.a_mlp, w.m_wo2, am.o_x, M, D, INTER, nullptr, 0, s));
        hook.tap(1 + l);
    }
    float* pre_temb = hook.pre_temb();
    RUN(LAYA_STAGE_FINAL, launch_final(c->bf16, c->x, c->xn, c->final_norm, c->type_emb, b.qt, c->seq_of,
                                       c->head[0].n1w, c->head[0].n1b, M, pre_temb, c->d_err, s));
    hook.tap(23, pre_temb);
    hook.tap(24);
    for (int l = 0; l < HEAD_LAYERS; l++) {
        const HeadW& w = c->head[l];
        if (l > 0) RUN(LAYA_STAGE_NORM, launch_ln(c->bf16, c->x, c->xn, w.n1w, w.n1b, M, c->num_sms, s));
        RUN(LAYA_STAGE_GEMM_QKV, gemm(c, EPI_QKV, am.a_xn, w.m_in, am.o_qkv, M, 3 * D, D, w.in_b, 0, s));
        RUN(LAYA_STAGE_ATTN, attention(c, b, am, -1, s));
        RUN(LAYA_STAGE_GEMM_OUT, gemm(c, EPI_RESID, am.a_ctx, w.m_out, am.o_x, M, D, D, w.out_b, 0, s));
        RUN(LAYA_STAGE_NORM, launch_ln(c->bf16, c->x, c->xn, w.n2w, w.n2b, M, c->num_sms, s));
        RUN(LAYA_STAGE_GEMM_UP,
            gemm(c, EPI_RELU, am.a_xn, w.m_l1, am.o_ff, M, HEAD_FF, D, w.l1_b, 0, s));
        RUN(LAYA_STAGE_GEMM_DOWN,
            gemm(c, EPI_RESID, am.a_ff, w.m_l2, am.o_x, M, D, HEAD_FF, w.l2_b, 0, s));
        hook.tap(25 + l);
    }
    RUN(LAYA_STAGE_TAIL, launch_tail(c->x, b.cu, b.mk, b.cum, b.S, b.G, M, c->tail, c->mv, c->partial, o.logits,
                                     o.act, o.pooled ? o.pooled : c->d_pooled, c->d_err, s));
    hook.extra(LAYA_STAGE_TAIL, b.G > 0 ? 2 : 0);  // launch_tail issues 3 kernels when there are markers
    if (o.hidden) {
        e = cudaMemcpyAsync(o.hidden, c->x, (size_t)M * D * 4, cudaMemcpyDeviceToDevice, s);
        if (e != cudaSuccess) return e;
    }
    return cudaSuccess;
#undef RUN
}

struct NoHook {
    void begin(int) {}
    void end(int) {}
    void tap(int, const float* = nullptr) {}
    void extra(int, int) {}
    float* pre_temb() { return nullptr; }
};

// Copies x to the host after every --dumpstats point. The "final" point
// (the final LayerNorm before the type embedding) is written by the final
// kernel into the qkv buffer, free between the last encoder layer and the
// first head layer (M x 768 f32 fits in its M x 2304 16-bit elements).
struct TraceHook {
    laya_ctx* c;
    float* trace;
    size_t LD;
    void begin(int) {}
    void end(int) {}
    void extra(int, int) {}
    float* pre_temb() { return reinterpret_cast<float*>(c->qkv); }
    void tap(int tag, const float* src = nullptr) {
        cudaMemcpyAsync(trace + (size_t)tag * LD, src ? src : c->x, LD * 4, cudaMemcpyDeviceToHost, c->stream);
    }
};

// --dumpstats on the device: after every dump point, the first three values,
// the sum and the absolute sum of the [M][768] state (f64), into
// c->d_stats[tag][5].
struct StatsHook {
    laya_ctx* c;
    size_t n;
    cudaError_t err = cudaSuccess;
    void begin(int) {}
    void end(int) {}
    void extra(int, int) {}
    float* pre_temb() { return reinterpret_cast<float*>(c->qkv); }
    void tap(int tag, const float* src = nullptr) {
        const cudaError_t e = launch_dump_stats(src ? src : c->x, n, c->d_stats + (size_t)tag * 5, c->stream);
        if (err == cudaSuccess) err = e;
    }
};

// Copies every intermediate of one encoder layer to the host.
struct DumpHook {
    laya_ctx* c;
    int target, M;
    uint16_t *xn_attn, *qkv, *ctx, *xn_mlp, *glu;
    float* x_mid;
    int cur = -1, norms = 0;
    void get(void* dst, const void* src, size_t bytes) {
        if (dst) cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToHost, c->stream);
    }
    void begin(int) {}
    void extra(int, int) {}
    float* pre_temb() { return nullptr; }
    void end(int st) {
        if (cur != target) return;
        const size_t M16 = (size_t)M * 2;
        switch (st) {
            case LAYA_STAGE_NORM:
                if (norms++ == 0 && target > 0) get(xn_attn, c->xn, M16 * D);
                else get(xn_mlp, c->xn, M16 * D);
                break;
            case LAYA_STAGE_GEMM_QKV: get(qkv, c->qkv, M16 * 3 * D); break;
            case LAYA_STAGE_ATTN: get(ctx, c->ctxb, M16 * D); break;
            case LAYA_STAGE_GEMM_OUT: get(x_mid, c->x, (size_t)M * D * 4); break;
            case LAYA_STAGE_GEMM_UP: get(glu, c->mlp, M16 * INTER); break;
            default: break;
        }
    }
    void tap(int tag, const float* = nullptr) {
        cur = tag;  // tag 0 follows the embedding, tag 1 + l follows layer l
        norms = 0;
        if (tag == 0 && target == 0) get(xn_attn, c->xn, (size_t)M * 2 * D);
    }
};

// An event pair around every launch. Recorded while the forward is being
// captured, the events become external event-record nodes of the graph, so
// the times are those of the graph's back-to-back kernels.
struct ProfileHook {
    cudaStream_t s;
    std::vector<cudaEvent_t> ev;  // created before capture
    std::vector<int> stage;
    size_t used = 0;
    int launches[LAYA_N_STAGES] = {0};
    cudaError_t reserve(size_t pairs) {
        while (ev.size() < 2 * pairs) {
            cudaEvent_t e;
            cudaError_t r = cudaEventCreate(&e);
            if (r != cudaSuccess) return r;
            ev.push_back(e);
        }
        stage.resize(pairs);
        return cudaSuccess;
    }
    void begin(int st) {
        if (used + 2 > ev.size()) return;  // more launches than reserved: left untimed
        stage[used / 2] = st;
        cudaEventRecordWithFlags(ev[used], s, cudaEventRecordExternal);
    }
    void end(int st) {
        launches[st]++;
        if (used + 2 > ev.size()) return;
        cudaEventRecordWithFlags(ev[used + 1], s, cudaEventRecordExternal);
        used += 2;
    }
    void tap(int, const float* = nullptr) {}
    float* pre_temb() { return nullptr; }
    void extra(int st, int n) { launches[st] += n; }
    // adds each timed launch's milliseconds to acc[launch]
    void collect_each(std::vector<float>& acc) const {
        for (size_t i = 0; i + 1 < used && i / 2 < acc.size(); i += 2) {
            float ms = 0.f;
            cudaEventElapsedTime(&ms, ev[i], ev[i + 1]);
            acc[i / 2] += ms;
        }
    }
    ~ProfileHook() {
        for (cudaEvent_t e : ev) cudaEventDestroy(e);
    }
};

// Run on stream s (any stream, the legacy default one included), capturing
// a graph on the context's own stream on first use of this shape.
// Batches above this many tokens run for milliseconds on the GPU, so
// launching their 171 kernels directly costs under 1%; each distinct shape
// would otherwise capture a graph that is rarely replayed (a length-bucketed
// sweep has a new shape almost every bucket).
constexpr int EAGER_TOKENS = 16384;

int launch_forward(laya_ctx* c, const Batch& b, const Outs& o, cudaStream_t s) {
    if (b.M > EAGER_TOKENS) {
        ActMaps am;
        int rc = build_maps(c, b.M, &am);
        if (rc) return rc;
        NoHook hook;
        cudaError_t e = run_forward(c, b, o, am, s, hook);
        if (e != cudaSuccess) return fail(c, LAYA_ERR_CUDA, "forward launch: %s", cudaGetErrorString(e));
        return LAYA_OK;
    }
    GraphKey k{b.M, b.S, b.G, b.maxlen, b.ids, b.cu, b.mk, b.cum, b.qt, o.logits, o.act, o.pooled, o.hidden};
    auto it = c->graphs.find(k);
    if (it == c->graphs.end()) {
        if (c->graphs.size() >= 16) {
            for (auto& g : c->graphs) cudaGraphExecDestroy(g.second);
            c->graphs.clear();
        }
        cudaGraph_t graph;
        ActMaps am;
        int rc = build_maps(c, b.M, &am);
        if (rc) return rc;
        NoHook hook;
        CK(cudaStreamBeginCapture(c->stream, cudaStreamCaptureModeThreadLocal));
        cudaError_t e = run_forward(c, b, o, am, c->stream, hook);
        cudaError_t e2 = cudaStreamEndCapture(c->stream, &graph);
        if (e != cudaSuccess) return fail(c, LAYA_ERR_CUDA, "launch during capture: %s", cudaGetErrorString(e));
        if (e2 != cudaSuccess) return fail(c, LAYA_ERR_CUDA, "cudaStreamEndCapture: %s", cudaGetErrorString(e2));
        cudaGraphExec_t exec;
        e = cudaGraphInstantiate(&exec, graph, 0);
        cudaGraphDestroy(graph);
        if (e != cudaSuccess) return fail(c, LAYA_ERR_CUDA, "cudaGraphInstantiate: %s", cudaGetErrorString(e));
        it = c->graphs.emplace(k, exec).first;
    }
    CK(cudaGraphLaunch(it->second, s));
    return LAYA_OK;
}

int check_seqs(laya_ctx* c, const laya_seq* seqs, uint32_t n, int* M, int* G, int* maxlen) {
    long long m = 0, g = 0;
    int ml = 0;
    for (uint32_t s = 0; s < n; s++) {
        const laya_seq& q = seqs[s];
        if (q.len == 0 || q.len > LAYA_MAX_LEN)
            return fail(c, LAYA_ERR_ARG, "sequence %u: length %u outside [1, %d]", s, q.len, LAYA_MAX_LEN);
        if (!q.ids) return fail(c, LAYA_ERR_ARG, "sequence %u: ids is NULL", s);
        if (q.qtype > 2) return fail(c, LAYA_ERR_ARG, "sequence %u: qtype %u (expected 0, 1 or 2)", s, q.qtype);
        if (q.n_markers > LAYA_MAX_MARKERS)
            return fail(c, LAYA_ERR_ARG, "sequence %u: %u markers (max %d)", s, q.n_markers, LAYA_MAX_MARKERS);
        if (q.n_markers && !q.markers) return fail(c, LAYA_ERR_ARG, "sequence %u: markers is NULL", s);
        for (uint32_t i = 0; i < q.len; i++)
            if (q.ids[i] >= (uint32_t)LAYA_VOCAB)
                return fail(c, LAYA_ERR_ARG, "sequence %u: token %u has id %u >= vocab %d", s, i, q.ids[i], LAYA_VOCAB);
        for (uint32_t r = 0; r < q.n_markers; r++)
            if (q.markers[r] >= q.len)
                return fail(c, LAYA_ERR_ARG, "sequence %u: marker %u at %u >= length %u", s, r, q.markers[r], q.len);
        m += q.len;
        g += q.n_markers;
        ml = std::max(ml, (int)q.len);
    }
    if (m > (1LL << 30)) return fail(c, LAYA_ERR_ARG, "batch of %lld tokens is too large", m);
    *M = (int)m;
    *G = (int)g;
    *maxlen = ml;
    return LAYA_OK;
}

int read_err(laya_ctx* c) {
    const int e = *c->h_err;
    if (e == 0) return LAYA_OK;
    *c->h_err = 0;
    cudaMemsetAsync(c->d_err, 0, 4, c->stream);
    cudaStreamSynchronize(c->stream);
    if (e & ERR_WAIT_TIMEOUT) return fail(c, LAYA_ERR_TIMEOUT, "a kernel gave up waiting (device error word %d)", e);
    return fail(c, LAYA_ERR_ARG, "a kernel rejected an index (device error word %d)", e);
}

// Stage a host batch into the workspace; returns the device-side view.
int stage_batch(laya_ctx* c, const laya_seq* seqs, uint32_t n, int M, int G, int maxlen, Batch* b) {
    const int S = (int)n;
    int rc = ensure_workspace(c, M, S, G);
    if (rc) return rc;
    uint8_t* h = static_cast<uint8_t*>(c->h_stage);
    uint32_t* h_ids = reinterpret_cast<uint32_t*>(h);
    int* h_cu = reinterpret_cast<int*>(h_ids + M);
    uint32_t* h_qt = reinterpret_cast<uint32_t*>(h_cu + S + 1);
    uint32_t* h_mk = h_qt + S;
    int* h_cum = reinterpret_cast<int*>(h_mk + G);
    int tok = 0, g = 0;
    h_cu[0] = 0;
    h_cum[0] = 0;
    for (int s = 0; s < S; s++) {
        memcpy(h_ids + tok, seqs[s].ids, seqs[s].len * 4);
        if (seqs[s].n_markers) memcpy(h_mk + g, seqs[s].markers, seqs[s].n_markers * 4);
        tok += seqs[s].len;
        g += seqs[s].n_markers;
        h_cu[s + 1] = tok;
        h_cum[s + 1] = g;
        h_qt[s] = seqs[s].qtype;
    }
    CK(cudaMemcpyAsync(c->d_in, h, in_words(M, S, G) * 4, cudaMemcpyHostToDevice, c->stream));
    uint32_t* d = c->d_in;  // the same offsets on the device
    *b = Batch{d, reinterpret_cast<const int*>(d + M), d + M + (S + 1) + S,
               reinterpret_cast<const int*>(d + M + (S + 1) + S + G), d + M + (S + 1), S, M, G, maxlen};
    return LAYA_OK;
}

// Device outputs of a staged batch of S sequences and G markers.
Outs staged_outs(laya_ctx* c, int S, float* pooled, float* hidden) {
    return Outs{c->d_out + 2 * S, c->d_out, pooled, hidden};
}

// After the forward: the error word and act | logits into pinned memory,
// one copy each (optional pooled / hidden straight to the caller).
int read_back(laya_ctx* c, int S, int G, float* logits, float* act) {
    float* h_out = reinterpret_cast<float*>(static_cast<uint8_t*>(c->h_stage) + out_offset(c));
    CK(cudaMemcpyAsync(c->h_err, c->d_err, 4, cudaMemcpyDeviceToHost, c->stream));
    CK(cudaMemcpyAsync(h_out, c->d_out, out_words(S, G) * 4, cudaMemcpyDeviceToHost, c->stream));
    CK(cudaStreamSynchronize(c->stream));
    memcpy(act, h_out, (size_t)S * 8);
    if (G) memcpy(logits, h_out + 2 * S, (size_t)G * 4);
    return LAYA_OK;
}

void rope_table(std::vector<float2>& t) {
    // inv_freq (src/main.zig:2399-2401) and f32 cos/sin of inv*pos (2503-2506)
    float inv[32];
    for (int j = 0; j < 32; j++) inv[j] = 1.0f / powf(ROPE_THETA, (float)j / 32.0f);
    t.resize((size_t)MAX_POS * 32);
    for (int p = 0; p < MAX_POS; p++)
        for (int j = 0; j < 32; j++) {
            const float f = inv[j] * (float)p;
            t[(size_t)p * 32 + j] = make_float2(cosf(f), sinf(f));
        }
}

int create_impl(laya_ctx* c, const laya_tensor* t, int n) {
    CK(cudaSetDevice(c->device));
    cudaDeviceProp prop;
    CK(cudaGetDeviceProperties(&prop, c->device));
    if (prop.major != 10)
        return fail(c, LAYA_ERR_NO_DEVICE, "device %d is sm_%d%d; this library is built for sm_100a", c->device,
                    prop.major, prop.minor);
    c->num_sms = prop.multiProcessorCount;
    // 40 MB of L2 set aside for the residual stream (a limit of this
    // process's context on the device, released with it). Measured on the
    // 64 x 180 batch (x = 35 MB): 16-48 MB all gain 2.5-3%, 40 MB the most;
    // 64 MB or the device maximum starve the other activations and lose.
    if (prop.persistingL2CacheMaxSize > 0 && prop.accessPolicyMaxWindowSize > 0) {
        c->l2_persist = std::min((size_t)prop.persistingL2CacheMaxSize, (size_t)40 << 20);
        c->l2_max_window = (size_t)prop.accessPolicyMaxWindowSize;
        CK(cudaDeviceSetLimit(cudaLimitPersistingL2CacheSize, c->l2_persist));
    }
    CK(cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking));
    CK(cudaMalloc(&c->d_err, 4));
    c->allocs.push_back(c->d_err);
    CK(cudaMemsetAsync(c->d_err, 0, 4, c->stream));
    CK(cudaMallocHost(&c->h_err, 4));
    *c->h_err = 0;
    CK(cudaMalloc(&c->d_stats, LAYA_TRACE_TAGS * 5 * sizeof(double)));
    c->allocs.push_back(c->d_stats);

    // one device staging buffer, as large as the largest tensor given
    size_t stage_bytes = 0;
    for (int i = 0; i < n; i++) stage_bytes = std::max(stage_bytes, (size_t)t[i].numel * elem_size(t[i].dtype));
    void* staging = nullptr;
    CK(cudaMalloc(&staging, stage_bytes ? stage_bytes : 256));
    int rc = 0;
    char nm[160];
    auto MAT = [&](const char* name, uint64_t rows, uint64_t cols, void** dst, int glu) {
        if (!rc) rc = upload(c, t, n, name, rows, cols, true, glu, dst, staging);
    };
    auto VEC = [&](const char* name, uint64_t numel, float** dst) {
        if (!rc) rc = upload(c, t, n, name, 1, numel, false, 0, reinterpret_cast<void**>(dst), staging);
    };
    MAT("encoder.embeddings.tok_embeddings.weight", VOCAB, D, &c->emb, 0);
    VEC("encoder.embeddings.norm.weight", D, &c->emb_norm);
    VEC("encoder.final_norm.weight", D, &c->final_norm);
    VEC("type_emb.weight", 3 * D, &c->type_emb);
    for (int l = 0; l < NL && !rc; l++) {
        EncW& w = c->enc[l];
        w.attn_norm = nullptr;
        if (l > 0) {
            snprintf(nm, sizeof nm, "encoder.layers.%d.attn_norm.weight", l);
            VEC(nm, D, &w.attn_norm);
        }
        snprintf(nm, sizeof nm, "encoder.layers.%d.attn.Wqkv.weight", l);
        MAT(nm, 3 * D, D, &w.wqkv, 0);
        snprintf(nm, sizeof nm, "encoder.layers.%d.attn.Wo.weight", l);
        MAT(nm, D, D, &w.wo, 0);
        snprintf(nm, sizeof nm, "encoder.layers.%d.mlp.Wi.weight", l);
        MAT(nm, 2 * INTER, D, &w.wi, 256);
        snprintf(nm, sizeof nm, "encoder.layers.%d.mlp.Wo.weight", l);
        MAT(nm, D, INTER, &w.wo2, 0);
        snprintf(nm, sizeof nm, "encoder.layers.%d.mlp_norm.weight", l);
        VEC(nm, D, &w.mlp_norm);
        if (!rc) rc = weight_map(c, &w.m_qkv, w.wqkv, 3 * D, D);
        if (!rc) rc = weight_map(c, &w.m_wo, w.wo, D, D);
        if (!rc) rc = weight_map(c, &w.m_wi, w.wi, 2 * INTER, D);
        if (!rc) rc = weight_map(c, &w.m_wo2, w.wo2, D, INTER);
    }
    for (int l = 0; l < HEAD_LAYERS && !rc; l++) {
        HeadW& w = c->head[l];
        auto N = [&](const char* s) {
            snprintf(nm, sizeof nm, "head.layers.%d.%s", l, s);
            return nm;
        };
        VEC(N("norm1.weight"), D, &w.n1w);
        VEC(N("norm1.bias"), D, &w.n1b);
        VEC(N("norm2.weight"), D, &w.n2w);
        VEC(N("norm2.bias"), D, &w.n2b);
        MAT(N("self_attn.in_proj_weight"), 3 * D, D, &w.in_w, 0);
        VEC(N("self_attn.in_proj_bias"), 3 * D, &w.in_b);
        MAT(N("self_attn.out_proj.weight"), D, D, &w.out_w, 0);
        VEC(N("self_attn.out_proj.bias"), D, &w.out_b);
        MAT(N("linear1.weight"), HEAD_FF, D, &w.l1_w, 0);
        VEC(N("linear1.bias"), HEAD_FF, &w.l1_b);
        MAT(N("linear2.weight"), D, HEAD_FF, &w.l2_w, 0);
        VEC(N("linear2.bias"), D, &w.l2_b);
        if (!rc) rc = weight_map(c, &w.m_in, w.in_w, 3 * D, D);
        if (!rc) rc = weight_map(c, &w.m_out, w.out_w, D, D);
        if (!rc) rc = weight_map(c, &w.m_l1, w.l1_w, HEAD_FF, D);
        if (!rc) rc = weight_map(c, &w.m_l2, w.l2_w, D, HEAD_FF);
    }
    float *s0w, *s0b, *s1w, *s1b, *s3w, *s3b, *a0w, *a0b, *a2w, *a2b;
    VEC("scorer.0.weight", D, &s0w);
    VEC("scorer.0.bias", D, &s0b);
    VEC("scorer.1.weight", (uint64_t)D * D, &s1w);
    VEC("scorer.1.bias", D, &s1b);
    VEC("scorer.3.weight", D, &s3w);
    VEC("scorer.3.bias", 1, &s3b);
    VEC("act_head.0.weight", 256 * (D + 4), &a0w);
    VEC("act_head.0.bias", 256, &a0b);
    VEC("act_head.2.weight", 2 * 256, &a2w);
    VEC("act_head.2.bias", 2, &a2b);
    cudaFree(staging);
    if (rc) return rc;
    // the act head reads act_head.0.weight column-wise: keep it transposed, [772][256]
    float* a0t = nullptr;
    rc = dev_alloc(c, reinterpret_cast<void**>(&a0t), (size_t)256 * (D + 4) * 4, c->allocs);
    if (rc) return rc;
    CK(launch_transpose_f32(a0t, a0w, 256, D + 4, c->stream));
    CK(cudaStreamSynchronize(c->stream));
    c->tail = TailWeights{s0w, s0b, s1w, s1b, s3w, s3b, a0t, a0b, a2w, a2b};

    std::vector<float2> rt;
    rope_table(rt);
    rc = dev_alloc(c, reinterpret_cast<void**>(&c->rope), rt.size() * sizeof(float2), c->allocs);
    if (rc) return rc;
    CK(cudaMemcpyAsync(c->rope, rt.data(), rt.size() * sizeof(float2), cudaMemcpyHostToDevice, c->stream));
    CK(cudaStreamSynchronize(c->stream));
    CK(gemm_prepare());
    CK(attention_prepare());
    return LAYA_OK;
}

}  // namespace

// For tail_noalloc.cu: the tail weights, device and error word of a context,
// and a way to record a failure on it.
int laya_ctx_tail_view(laya_ctx* c, TailWeights* w, int* device, int** d_err) {
    if (!c) return LAYA_ERR_ARG;
    *w = c->tail;
    *device = c->device;
    *d_err = c->d_err;
    return LAYA_OK;
}

int laya_ctx_fail(laya_ctx* c, int code, const char* msg) { return fail(c, code, "%s", msg); }

extern "C" {

int laya_gpu_version(void) { return LAYA_GPU_ABI_VERSION; }

int laya_gpu_device_count(void) {
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess) return 0;
    return n;
}

const char* laya_gpu_last_error(const laya_ctx* ctx) { return ctx ? ctx->err.c_str() : g_create_error.c_str(); }

void laya_gpu_destroy(laya_ctx* c) {
    if (!c) return;
    DeviceGuard dg;
    dg.set(c->device);
    if (c->stream) cudaStreamSynchronize(c->stream);
    free_workspace(c);
    for (void* p : c->allocs) cudaFree(p);
    if (c->h_err) cudaFreeHost(c->h_err);
    if (c->h_stage) cudaFreeHost(c->h_stage);
    if (c->stream) cudaStreamDestroy(c->stream);
    delete c;
}

int laya_gpu_create(int device, const laya_tensor* tensors, int n_tensors, int precision, laya_ctx** out) {
    if (!out) return fail(nullptr, LAYA_ERR_ARG, "out is NULL");
    *out = nullptr;
    if (!tensors || n_tensors <= 0) return fail(nullptr, LAYA_ERR_ARG, "no tensors given");
    if (precision != LAYA_PREC_BF16 && precision != LAYA_PREC_F16)
        return fail(nullptr, LAYA_ERR_ARG, "precision %d (expected LAYA_PREC_BF16 or LAYA_PREC_F16)", precision);
    const int ndev = laya_gpu_device_count();
    if (device < 0 || device >= ndev)
        return fail(nullptr, LAYA_ERR_NO_DEVICE, "device %d requested, %d visible", device, ndev);
    DeviceGuard dg;  // create_impl makes `device` current
    dg.prev = -1;
    if (cudaGetDevice(&dg.prev) != cudaSuccess) dg.prev = -1;
    laya_ctx* c = new laya_ctx();
    c->device = device;
    c->bf16 = precision == LAYA_PREC_BF16;
    const int rc = create_impl(c, tensors, n_tensors);
    if (rc) {
        g_create_error = c->err;
        laya_gpu_destroy(c);
        return rc;
    }
    *out = c;
    return LAYA_OK;
}

int laya_gpu_forward_batch(laya_ctx* c, const laya_seq* seqs, uint32_t n, float* logits, float* act, float* pooled,
                           float* hidden) {
    if (!c) return fail(nullptr, LAYA_ERR_ARG, "ctx is NULL");
    if (!seqs || n == 0) return fail(c, LAYA_ERR_ARG, "empty batch");
    if (!act) return fail(c, LAYA_ERR_ARG, "act is NULL");
    DeviceGuard dg;
    CK(dg.set(c->device));
    int M, G, maxlen;
    int rc = check_seqs(c, seqs, n, &M, &G, &maxlen);
    if (rc) return rc;
    if (G && !logits) return fail(c, LAYA_ERR_ARG, "logits is NULL");
    Batch b;
    rc = stage_batch(c, seqs, n, M, G, maxlen, &b);
    if (rc) return rc;
    float* d_hidden = nullptr;
    if (hidden) d_hidden = reinterpret_cast<float*>(c->qkv);  // free after the forward; M*D*4 <= M*3*D*2
    const Outs o = staged_outs(c, (int)n, pooled ? c->d_pooled : nullptr, d_hidden);
    rc = launch_forward(c, b, o, c->stream);
    if (rc) return rc;
    if (pooled) CK(cudaMemcpyAsync(pooled, c->d_pooled, (size_t)n * D * 4, cudaMemcpyDeviceToHost, c->stream));
    if (hidden) CK(cudaMemcpyAsync(hidden, d_hidden, (size_t)M * D * 4, cudaMemcpyDeviceToHost, c->stream));
    rc = read_back(c, (int)n, G, logits, act);
    if (rc) return rc;
    return read_err(c);
}

int laya_gpu_forward(laya_ctx* c, const uint32_t* ids, uint32_t L, uint32_t qtype, const uint32_t* markers,
                     uint32_t K, float* logits, float* act, float* pooled, float* hidden) {
    if (!pooled) return fail(c, LAYA_ERR_ARG, "pooled is NULL");
    laya_seq s{ids, L, markers, K, qtype};
    return laya_gpu_forward_batch(c, &s, 1, logits, act, pooled, hidden);
}

int laya_gpu_forward_device(laya_ctx* c, const laya_batch* bt, float* logits, float* act, float* pooled,
                            float* hidden, void* stream) {
    if (!c) return fail(nullptr, LAYA_ERR_ARG, "ctx is NULL");
    if (!bt || bt->n_seqs == 0 || bt->n_tokens == 0) return fail(c, LAYA_ERR_ARG, "empty batch");
    if (bt->max_len == 0 || bt->max_len > LAYA_MAX_LEN)
        return fail(c, LAYA_ERR_ARG, "max_len %u outside [1, %d]", bt->max_len, LAYA_MAX_LEN);
    if (!bt->ids || !bt->cu_seqlens || !bt->cu_markers || !bt->qtypes || !act || (bt->n_markers && (!bt->markers || !logits)))
        return fail(c, LAYA_ERR_ARG, "NULL input or output pointer");
    DeviceGuard dg;
    CK(dg.set(c->device));
    int rc = ensure_workspace(c, (int)bt->n_tokens, (int)bt->n_seqs, (int)bt->n_markers);
    if (rc) return rc;
    cudaStream_t s = static_cast<cudaStream_t>(stream);  // 0 = the legacy default stream
    Batch b{bt->ids, bt->cu_seqlens, bt->markers, bt->cu_markers, bt->qtypes, (int)bt->n_seqs, (int)bt->n_tokens,
            (int)bt->n_markers, (int)bt->max_len};
    Outs o{logits, act, pooled, hidden};
    return launch_forward(c, b, o, s);
}

int laya_gpu_sync(laya_ctx* c) {
    if (!c) return fail(nullptr, LAYA_ERR_ARG, "ctx is NULL");
    DeviceGuard dg;
    CK(dg.set(c->device));
    CK(cudaDeviceSynchronize());
    CK(cudaMemcpy(c->h_err, c->d_err, 4, cudaMemcpyDeviceToHost));
    return read_err(c);
}

int laya_gpu_forward_trace(laya_ctx* c, const uint32_t* ids, uint32_t L, uint32_t qtype, const uint32_t* markers,
                           uint32_t K, float* logits, float* act, float* trace) {
    if (!c) return fail(nullptr, LAYA_ERR_ARG, "ctx is NULL");
    if (!trace || !act) return fail(c, LAYA_ERR_ARG, "NULL output");
    DeviceGuard dg;
    CK(dg.set(c->device));
    laya_seq sq{ids, L, markers, K, qtype};
    int M, G, maxlen;
    int rc = check_seqs(c, &sq, 1, &M, &G, &maxlen);
    if (rc) return rc;
    if (G && !logits) return fail(c, LAYA_ERR_ARG, "logits is NULL");
    Batch b;
    rc = stage_batch(c, &sq, 1, M, G, maxlen, &b);
    if (rc) return rc;
    const Outs o = staged_outs(c, 1, nullptr, nullptr);
    const size_t LD = (size_t)L * D;
    ActMaps am;
    rc = build_maps(c, M, &am);
    if (rc) return rc;
    TraceHook hook{c, trace, LD};
    cudaError_t e = run_forward(c, b, o, am, c->stream, hook);
    if (e != cudaSuccess) return fail(c, LAYA_ERR_CUDA, "forward: %s", cudaGetErrorString(e));
    rc = read_back(c, 1, G, logits, act);
    if (rc) return rc;
    return read_err(c);
}

int laya_gpu_format_dump(const uint32_t* ids, uint32_t L, uint32_t qtype, const uint32_t* markers, uint32_t K,
                         const float* logits, const double* stats, char* text, uint64_t cap, uint64_t* text_len) {
    if (text_len) *text_len = 0;
    if (!stats || (L && !ids) || (K && (!markers || !logits)))
        return fail(nullptr, LAYA_ERR_ARG, "format_dump: NULL input");
    // The lines the reference's forward prints with --dumpstats, in its
    // order and formats (src/main.zig:113-130, 2651-2655, 2679-2683,
    // 2708-2711, 2749-2753, 2771-2777).
    static const char* const tags[LAYA_TRACE_TAGS] = {
        "emb", "l0", "l1", "l2", "l3", "l4", "l5", "l6", "l7", "l8", "l9", "l10", "l11", "l12",
        "l13", "l14", "l15", "l16", "l17", "l18", "l19", "l20", "l21", "final", "temb", "h0", "h1"};
    std::string out;
    char line[256];
    snprintf(line, sizeof line, "[dump] meta L=%u qtype=%u\n", L, qtype);
    out += line;
    for (uint32_t i = 0; i < L; i += 8) {
        out += "[dump] ids";
        for (uint32_t j = i; j < L && j < i + 8; j++) {
            snprintf(line, sizeof line, " %u", ids[j]);
            out += line;
        }
        out += "\n";
    }
    for (int t = 0; t < LAYA_TRACE_TAGS; t++) {
        const double* st = stats + 5 * t;  // x[0..2] are f32 values, printed as the reference prints an f32
        snprintf(line, sizeof line, "[dump] %-5s %.5f %.5f %.5f %.3f %.3f\n", tags[t], (double)(float)st[0],
                 (double)(float)st[1], (double)(float)st[2], st[3], st[4]);
        out += line;
    }
    out += "[dump] mark";
    for (uint32_t r = 0; r < K; r++) {
        snprintf(line, sizeof line, " %u", markers[r]);
        out += line;
    }
    out += "\n[dump] logit";
    for (uint32_t r = 0; r < K; r++) {
        snprintf(line, sizeof line, " %.5f", (double)logits[r]);
        out += line;
    }
    out += "\n";
    if (text_len) *text_len = out.size() + 1;
    if (!text || cap < out.size() + 1)
        return fail(nullptr, LAYA_ERR_ARG, "dumpstats: the text needs %zu bytes, %llu given", out.size() + 1,
                    (unsigned long long)cap);
    memcpy(text, out.c_str(), out.size() + 1);
    return LAYA_OK;
}

int laya_gpu_forward_dumpstats(laya_ctx* c, const uint32_t* ids, uint32_t L, uint32_t qtype, const uint32_t* markers,
                               uint32_t K, float* logits, float* act, char* text, uint64_t cap, uint64_t* text_len) {
    if (text_len) *text_len = 0;
    if (!c) return fail(nullptr, LAYA_ERR_ARG, "ctx is NULL");
    if (!act) return fail(c, LAYA_ERR_ARG, "act is NULL");
    DeviceGuard dg;
    CK(dg.set(c->device));
    laya_seq sq{ids, L, markers, K, qtype};
    int M, G, maxlen;
    int rc = check_seqs(c, &sq, 1, &M, &G, &maxlen);
    if (rc) return rc;
    if (G && !logits) return fail(c, LAYA_ERR_ARG, "logits is NULL");
    Batch b;
    rc = stage_batch(c, &sq, 1, M, G, maxlen, &b);
    if (rc) return rc;
    const Outs o = staged_outs(c, 1, nullptr, nullptr);
    ActMaps am;
    rc = build_maps(c, M, &am);
    if (rc) return rc;
    StatsHook hook{c, (size_t)M * D};
    cudaError_t e = run_forward(c, b, o, am, c->stream, hook);
    if (e == cudaSuccess) e = hook.err;
    if (e != cudaSuccess) return fail(c, LAYA_ERR_CUDA, "forward: %s", cudaGetErrorString(e));
    double st[LAYA_TRACE_TAGS][5];
    CK(cudaMemcpyAsync(st, c->d_stats, sizeof st, cudaMemcpyDeviceToHost, c->stream));
    rc = read_back(c, 1, G, logits, act);
    if (rc) return rc;
    rc = read_err(c);
    if (rc) return rc;
    return laya_gpu_format_dump(ids, L, qtype, markers, K, logits, &st[0][0], text, cap, text_len) == LAYA_OK
               ? LAYA_OK
               : fail(c, LAYA_ERR_ARG, "%s", laya_gpu_last_error(nullptr));
}

int laya_gpu_forward_dump(laya_ctx* c, const uint32_t* ids, uint32_t L, uint32_t qtype, const uint32_t* markers,
                          uint32_t K, int layer, uint16_t* xn_attn, uint16_t* qkv, uint16_t* ctx_out, float* x_mid,
                          uint16_t* xn_mlp, uint16_t* glu) {
    if (!c) return fail(nullptr, LAYA_ERR_ARG, "ctx is NULL");
    if (layer < 0 || layer >= NL) return fail(c, LAYA_ERR_ARG, "layer %d outside [0, %d)", layer, NL);
    DeviceGuard dg;
    CK(dg.set(c->device));
    laya_seq sq{ids, L, markers, K, qtype};
    int M, G, maxlen;
    int rc = check_seqs(c, &sq, 1, &M, &G, &maxlen);
    if (rc) return rc;
    Batch b;
    rc = stage_batch(c, &sq, 1, M, G, maxlen, &b);
    if (rc) return rc;
    const Outs o = staged_outs(c, 1, nullptr, nullptr);
    ActMaps am;
    rc = build_maps(c, M, &am);
    if (rc) return rc;
    DumpHook hook{c, layer, M, xn_attn, qkv, ctx_out, xn_mlp, glu, x_mid};
    cudaError_t e = run_forward(c, b, o, am, c->stream, hook);
    if (e != cudaSuccess) return fail(c, LAYA_ERR_CUDA, "forward: %s", cudaGetErrorString(e));
    CK(cudaMemcpyAsync(c->h_err, c->d_err, 4, cudaMemcpyDeviceToHost, c->stream));
    CK(cudaStreamSynchronize(c->stream));
    return read_err(c);
}

int laya_gpu_forward_profile_launches(laya_ctx* c, const laya_batch* bt, float* logits, float* act, int iters,
                                      void* stream, float* launch_ms, int* launch_stage, int cap, int* n_launches) {
    if (!c) return fail(nullptr, LAYA_ERR_ARG, "ctx is NULL");
    if (!bt || bt->n_seqs == 0 || bt->n_tokens == 0 || bt->max_len == 0 || bt->max_len > LAYA_MAX_LEN || iters <= 0 ||
        !act || (bt->n_markers && !logits) || cap < 0 || (cap > 0 && (!launch_ms || !launch_stage)))
        return fail(c, LAYA_ERR_ARG, "profile: bad batch or NULL output");
    DeviceGuard dg;
    CK(dg.set(c->device));
    int rc = ensure_workspace(c, (int)bt->n_tokens, (int)bt->n_seqs, (int)bt->n_markers);
    if (rc) return rc;
    cudaStream_t s = static_cast<cudaStream_t>(stream);  // 0 = the legacy default stream
    Batch b{bt->ids, bt->cu_seqlens, bt->markers, bt->cu_markers, bt->qtypes, (int)bt->n_seqs, (int)bt->n_tokens,
            (int)bt->n_markers, (int)bt->max_len};
    Outs o{logits, act, nullptr, nullptr};
    ActMaps am;
    rc = build_maps(c, (int)bt->n_tokens, &am);
    if (rc) return rc;
    ProfileHook hook;
    hook.s = c->stream;
    CK(hook.reserve(512));
    cudaGraph_t graph;
    CK(cudaStreamBeginCapture(c->stream, cudaStreamCaptureModeThreadLocal));
    cudaError_t e = run_forward(c, b, o, am, c->stream, hook);
    cudaError_t e2 = cudaStreamEndCapture(c->stream, &graph);
    if (e != cudaSuccess) return fail(c, LAYA_ERR_CUDA, "profile capture: %s", cudaGetErrorString(e));
    if (e2 != cudaSuccess) return fail(c, LAYA_ERR_CUDA, "profile capture: %s", cudaGetErrorString(e2));
    cudaGraphExec_t exec;
    e = cudaGraphInstantiate(&exec, graph, 0);
    cudaGraphDestroy(graph);
    if (e != cudaSuccess) return fail(c, LAYA_ERR_CUDA, "profile instantiate: %s", cudaGetErrorString(e));
    const int pairs = (int)(hook.used / 2);
    std::vector<float> acc(pairs, 0.f);
    for (int it = 0; it < iters && e == cudaSuccess; it++) {
        e = cudaGraphLaunch(exec, s);
        if (e == cudaSuccess) e = cudaStreamSynchronize(s);
        if (e == cudaSuccess) hook.collect_each(acc);
    }
    cudaGraphExecDestroy(exec);
    if (e != cudaSuccess) return fail(c, LAYA_ERR_CUDA, "profile run: %s", cudaGetErrorString(e));
    if (n_launches) *n_launches = pairs;
    for (int i = 0; i < pairs && i < cap; i++) {
        launch_ms[i] = acc[i];
        launch_stage[i] = hook.stage[i];
    }
    CK(cudaMemcpy(c->h_err, c->d_err, 4, cudaMemcpyDeviceToHost));
    return read_err(c);
}

int laya_gpu_forward_profile(laya_ctx* c, const laya_batch* bt, float* logits, float* act, int iters, void* stream,
                             float* stage_ms, int* stage_launches) {
    if (!stage_ms) return fail(c, LAYA_ERR_ARG, "profile: stage_ms is NULL");
    std::vector<float> ms(512);
    std::vector<int> st(512);
    int n = 0;
    const int rc = laya_gpu_forward_profile_launches(c, bt, logits, act, iters, stream, ms.data(), st.data(), 512, &n);
    if (rc) return rc;
    for (int i = 0; i < LAYA_N_STAGES; i++) {
        stage_ms[i] = 0.f;
        if (stage_launches) stage_launches[i] = 0;
    }
    for (int i = 0; i < n && i < 512; i++) {
        stage_ms[st[i]] += ms[i];
        if (stage_launches) stage_launches[st[i]] += st[i] == LAYA_STAGE_TAIL && bt->n_markers ? 3 : 1;
    }
    return LAYA_OK;
}

int laya_gpu_linear(const void* x, const void* w, const float* bias, float* out, int M, int N, int K, int elem_dtype,
                    void* stream) {
    laya_ctx* c = nullptr;
    if (!x || !w || !out || M <= 0 || N <= 0 || K <= 0 || N % 128 || K % 128)
        return fail(c, LAYA_ERR_ARG, "linear: bad shape or NULL pointer (M=%d N=%d K=%d)", M, N, K);
    if (elem_dtype != LAYA_DT_BF16 && elem_dtype != LAYA_DT_F16)
        return fail(c, LAYA_ERR_DTYPE, "linear: elem_dtype %d", elem_dtype);
    if (((uintptr_t)x | (uintptr_t)w | (uintptr_t)out | (uintptr_t)bias) & 15)
        return fail(c, LAYA_ERR_ARG, "linear: pointers must be 16-byte aligned");
    const bool bf16 = elem_dtype == LAYA_DT_BF16;
    const int bn = N % 256 == 0 ? 256 : 128;
    int dev = 0, sms = 148;
    CK(cudaGetDevice(&dev));
    CK(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
    CK(gemm_prepare());
    static int* d_err[64] = {nullptr};
    if (dev < 64 && !d_err[dev]) {
        CK(cudaMalloc(&d_err[dev], 4));
        CK(cudaMemset(d_err[dev], 0, 4));
        CK(cudaDeviceSynchronize());  // the launch below may be on a stream that does not wait on this one
    }
    CUtensorMap am, bm, om;
    if (make_tmap_2d(&am, x, K, M, 128, bf16) != CUDA_SUCCESS || make_tmap_2d(&bm, w, K, N, 128, bf16) != CUDA_SUCCESS ||
        make_out_map(&om, out, N, M, 4, bf16) != CUDA_SUCCESS)
        return fail(c, LAYA_ERR_CUDA, "linear: cuTensorMapEncodeTiled failed");
    GemmArgs g{};
    g.M = M;
    g.N = N;
    g.K = K;
    g.bias = bias;
    g.err = d_err[dev < 64 ? dev : 0];
    CK(launch_gemm(EPI_F32, bn, bf16, am, bm, om, g, sms, static_cast<cudaStream_t>(stream)));
    return LAYA_OK;
}

}  // extern "C"
