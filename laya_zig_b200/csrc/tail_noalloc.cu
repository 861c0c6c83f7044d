// tail_noalloc.cu -- the decision tail (scorer + act/escalate head) for
// callers that must not allocate device memory at decision time.
//
// Who needs it: a host that hands all of a GPU's memory to its own caching
// allocator up front (a serving process with a fixed memory budget, or a
// PyTorch process whose allocator already holds the device) cannot have a
// library call cudaMalloc mid-request: the call fails or stalls the whole
// device with an implicit synchronisation. The regular entry points keep
// their scratch in a per-context workspace that grows with cudaMalloc when a
// batch is larger than any before. This entry point scores the options of
// hidden states the caller already holds, with its scratch in the static
// array below instead.
//
// The scratch is `g_tail_scratch`: room for LAYA_NOALLOC_MAX_MARKERS marker
// rows (the LayerNorm'd marker vectors, 768 f32 each, plus 12 partial scorer
// sums each), 6.4 MB. Every GPU that loads this library holds it until the
// process exits. All calls share it and it keeps the last call's contents;
// every element a call reads is first written by the same call, so nothing
// needs clearing, but calls that overlap on the GPU (on different streams,
// or from different threads) race on it.
#include <atomic>
#include <cstdio>

#include "../../include/laya_gpu.h"
#include "kernels.cuh"

using namespace laya;

constexpr size_t MV_FLOATS = (size_t)LAYA_NOALLOC_MAX_MARKERS * D;
constexpr size_t SCRATCH_FLOATS = MV_FLOATS + (size_t)LAYA_NOALLOC_MAX_MARKERS * SCORER_GROUPS;

static __device__ __align__(256) float g_tail_scratch[SCRATCH_FLOATS];

// Device address of g_tail_scratch per device, resolved on the first call on
// that device with that device current (in host code the symbol is only a
// stand-in, not an address a kernel could use). Atomic, because two host
// threads may make their first calls on one device at the same time; both
// then resolve and store the same address.
static std::atomic<float*> g_scratch_ptr[64];

// Context pieces the tail needs (defined with the context in laya_gpu.cu).
int laya_ctx_tail_view(laya_ctx* c, TailWeights* w, int* device, int** d_err);
int laya_ctx_fail(laya_ctx* c, int code, const char* msg);

extern "C" LAYA_API int laya_gpu_decision_tail_noalloc(laya_ctx* ctx, const float* hidden, const int32_t* cu_seqlens,
                                                       const uint32_t* markers, const int32_t* cu_markers,
                                                       uint32_t n_seqs, uint32_t n_markers, float* logits,
                                                       float* act, float* pooled, void* stream) {
    if (!ctx) return laya_ctx_fail(nullptr, LAYA_ERR_ARG, "decision tail: ctx is NULL");
    TailWeights w;
    int device = 0;
    int* d_err = nullptr;
    if (laya_ctx_tail_view(ctx, &w, &device, &d_err) != LAYA_OK)
        return laya_ctx_fail(ctx, LAYA_ERR_ARG, "decision tail: the context has no tail weights");
    if (!hidden || !cu_seqlens || !cu_markers || !act || !pooled || (n_markers && (!markers || !logits)))
        return laya_ctx_fail(ctx, LAYA_ERR_ARG, "decision tail: NULL input or output pointer");
    if (n_seqs == 0) return laya_ctx_fail(ctx, LAYA_ERR_ARG, "decision tail: no sequences");
    if (n_markers > (uint32_t)LAYA_NOALLOC_MAX_MARKERS) {
        char msg[160];
        snprintf(msg, sizeof msg, "decision tail: %u markers exceed the no-allocation limit of %d", n_markers,
                 LAYA_NOALLOC_MAX_MARKERS);
        return laya_ctx_fail(ctx, LAYA_ERR_ARG, msg);
    }
    if (device < 0 || device >= 64) return laya_ctx_fail(ctx, LAYA_ERR_NO_DEVICE, "decision tail: device index");
    // The context's device is made current for the call and the caller's
    // current device given back before returning.
    int prev = -1;
    if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
    struct Restore {
        int dev;
        ~Restore() {
            if (dev >= 0) cudaSetDevice(dev);
        }
    } restore{prev};
    cudaError_t e = cudaSetDevice(device);
    if (e != cudaSuccess) return laya_ctx_fail(ctx, LAYA_ERR_CUDA, cudaGetErrorString(e));
    float* mv = g_scratch_ptr[device].load(std::memory_order_relaxed);
    if (!mv) {
        void* p = nullptr;
        e = cudaGetSymbolAddress(&p, g_tail_scratch);
        if (e != cudaSuccess || !p) return laya_ctx_fail(ctx, LAYA_ERR_CUDA, "cudaGetSymbolAddress(g_tail_scratch) failed");
        mv = static_cast<float*>(p);
        g_scratch_ptr[device].store(mv, std::memory_order_relaxed);
    }
    float* partial = mv + MV_FLOATS;
    e = launch_tail(hidden, cu_seqlens, markers, reinterpret_cast<const int*>(cu_markers), (int)n_seqs,
                    (int)n_markers, -1, w, mv, partial, logits, act, pooled, d_err, static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return laya_ctx_fail(ctx, LAYA_ERR_CUDA, cudaGetErrorString(e));
    return LAYA_OK;
}
