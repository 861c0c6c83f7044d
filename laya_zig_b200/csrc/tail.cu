// tail.cu -- option-marker scorer and act/escalate head (src/main.zig:2756-2814).
//
// Three small kernels over all sequences of a batch at once:
//   marker_ln   x[marker token] -> LayerNorm(scorer.0 w, b)        (2761-2763)
//   scorer      h = gelu(scorer.1 . v + b); partial dot with scorer.3 over
//               each group of 64 outputs, summed later in a fixed order
//               (2764-2767), so the result does not depend on scheduling
//   act         per sequence: logits, pooled = x[CLS], untempered softmax,
//               [top1, top1-top2, entropy/ln(max(K,2)), max(K,2)/255],
//               [pooled | features] -> 256 -> gelu -> 2 -> softmax (2787-2814)
// Everything here is f32 with the scalar erf/gelu of src/main.zig:60-70.
#include "kernels.cuh"

namespace laya {
namespace {

__device__ __forceinline__ float erf_as(float x) {
    const float s = x < 0 ? -1.0f : 1.0f;
    const float a = fabsf(x);
    const float t = 1.0f / (1.0f + 0.3275911f * a);
    const float poly = ((((1.061405429f * t - 1.453152027f) * t + 1.421413741f) * t - 0.284496736f) * t + 0.254829592f) * t;
    return s * (1.0f - poly * expf(-a * a));
}
__device__ __forceinline__ float gelu_scalar(float x) { return 0.5f * x * (1.0f + erf_as(x * 0.70710678118654752440f)); }

__device__ __forceinline__ int find_seq(const int* cu, int n, int t) {
    int lo = 0, hi = n;
    while (hi - lo > 1) {
        const int mid = (lo + hi) >> 1;
        if (cu[mid] <= t) lo = mid;
        else hi = mid;
    }
    return lo;
}

// one warp per marker
__global__ void marker_ln_kernel(const float* __restrict__ x, const int* __restrict__ cu_seqlens,
                                 const uint32_t* __restrict__ markers, const int* __restrict__ cu_markers, int n_seqs,
                                 int G, const float* __restrict__ w, const float* __restrict__ b,
                                 float* __restrict__ mv, int* err) {
    const int g = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (g >= G) return;
    const int s = find_seq(cu_markers, n_seqs, g);
    const int L = cu_seqlens[s + 1] - cu_seqlens[s];
    uint32_t m = markers[g];
    if (m >= (uint32_t)L) {
        if (lane == 0) atomicOr(err, ERR_BAD_INDEX);
        m = 0;
    }
    const float* row = x + (size_t)(cu_seqlens[s] + m) * D;
    float v[24];
#pragma unroll
    for (int i = 0; i < 24; i++) v[i] = row[i * 32 + lane];
    float sum = 0.f;
#pragma unroll
    for (int i = 0; i < 24; i++) sum += v[i];
    const float mean = warp_sum(sum) * (1.0f / D);
    float q = 0.f;
#pragma unroll
    for (int i = 0; i < 24; i++) q += (v[i] - mean) * (v[i] - mean);
    const float rs = 1.0f / sqrtf(warp_sum(q) * (1.0f / D) + LN_EPS);
#pragma unroll
    for (int i = 0; i < 24; i++) {
        const int c = i * 32 + lane;
        mv[(size_t)g * D + c] = (v[i] - mean) * rs * w[c] + b[c];
    }
}

// CTA: 16 markers x 64 scorer outputs; 256 threads, each 1 marker x 4 outputs.
constexpr int SM_ROWS = 16, SM_COLS = 64, SM_K = 64;
__global__ void __launch_bounds__(256) scorer_kernel(const float* __restrict__ mv, int G, const float* __restrict__ w1,
                                                     const float* __restrict__ b1, const float* __restrict__ w3,
                                                     float* __restrict__ partial) {
    __shared__ float As[SM_ROWS][SM_K + 1];
    __shared__ float Bs[SM_COLS][SM_K + 1];
    const int g0 = blockIdx.x * SM_ROWS, j0 = blockIdx.y * SM_COLS;
    const int tid = threadIdx.x, mr = tid >> 4, jc = (tid & 15) * 4;
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    for (int k0 = 0; k0 < D; k0 += SM_K) {
#pragma unroll
        for (int i = 0; i < (SM_ROWS * SM_K) / 256; i++) {
            const int e = tid + i * 256, r = e / SM_K, c = e % SM_K;
            As[r][c] = (g0 + r < G) ? mv[(size_t)(g0 + r) * D + k0 + c] : 0.f;
        }
#pragma unroll
        for (int i = 0; i < (SM_COLS * SM_K) / 256; i++) {
            const int e = tid + i * 256, r = e / SM_K, c = e % SM_K;
            Bs[r][c] = w1[(size_t)(j0 + r) * D + k0 + c];
        }
        __syncthreads();
#pragma unroll 8
        for (int k = 0; k < SM_K; k++) {
            const float a = As[mr][k];
#pragma unroll
            for (int i = 0; i < 4; i++) acc[i] = fmaf(a, Bs[jc + i][k], acc[i]);
        }
        __syncthreads();
    }
    float p = 0.f;
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const int j = j0 + jc + i;
        p += gelu_scalar(acc[i] + b1[j]) * w3[j];
    }
    // the 16 threads of one marker are lanes 0-15 or 16-31 of a warp
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) p += __shfl_xor_sync(0xffffffffu, p, o);
    if ((tid & 15) == 0 && g0 + mr < G) partial[(size_t)(g0 + mr) * SCORER_GROUPS + blockIdx.y] = p;
}

// one CTA (256 threads) per sequence
__global__ void __launch_bounds__(256) act_kernel(const float* __restrict__ x, const int* __restrict__ cu_seqlens,
                                                  const int* __restrict__ cu_markers,
                                                  const float* __restrict__ partial, TailWeights w,
                                                  float* __restrict__ logits, float* __restrict__ act,
                                                  float* __restrict__ pooled) {
    __shared__ float lg[MAX_MARKERS_PER_SEQ];
    __shared__ float act_in[D + 4];
    __shared__ float h256[256];
    __shared__ float a2[2];
    const int s = blockIdx.x, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int gb = cu_markers[s], K = min(cu_markers[s + 1] - gb, MAX_MARKERS_PER_SEQ);
    for (int r = tid; r < K; r += 256) {
        float v = 0.f;
        for (int c = 0; c < SCORER_GROUPS; c++) v += partial[(size_t)(gb + r) * SCORER_GROUPS + c];
        v += w.s3b[0];
        lg[r] = v;
        logits[gb + r] = v;
    }
    const float* cls = x + (size_t)cu_seqlens[s] * D;
    for (int c = tid; c < D; c += 256) {
        act_in[c] = cls[c];
        pooled[(size_t)s * D + c] = cls[c];
    }
    __syncthreads();
    if (tid == 0) {
        // softmax (src/main.zig:72-81) and the features (2789-2807)
        float mx = -INFINITY;
        for (int r = 0; r < K; r++) mx = fmaxf(mx, lg[r]);
        float sum = 0.f;
        for (int r = 0; r < K; r++) {
            lg[r] = expf(lg[r] - mx);
            sum += lg[r];
        }
        for (int r = 0; r < K; r++) lg[r] /= sum;
        const float kk = (float)(K > 2 ? K : 2);
        float ent = 0.f;
        for (int r = 0; r < K; r++)
            if (lg[r] > 1e-12f) ent -= lg[r] * logf(lg[r]);
        ent /= logf(kk);
        float t0 = 0.f, t1 = 0.f;
        for (int r = 0; r < K; r++) {
            const float v = lg[r];
            if (v > t0) {
                t1 = t0;
                t0 = v;
            } else if (v > t1) {
                t1 = v;
            }
        }
        act_in[D] = t0;
        act_in[D + 1] = t0 - t1;
        act_in[D + 2] = ent;
        act_in[D + 3] = kk / 255.0f;
    }
    __syncthreads();
    for (int i = warp; i < 256; i += 8) {
        const float* wr = w.a0w + (size_t)i * (D + 4);
        float p = 0.f;
        for (int k = lane; k < D + 4; k += 32) p = fmaf(act_in[k], wr[k], p);
        p = warp_sum(p);
        if (lane == 0) h256[i] = gelu_scalar(p + w.a0b[i]);
    }
    __syncthreads();
    if (warp < 2) {
        float p = 0.f;
        for (int k = lane; k < 256; k += 32) p = fmaf(h256[k], w.a2w[warp * 256 + k], p);
        p = warp_sum(p);
        if (lane == 0) a2[warp] = p + w.a2b[warp];
    }
    __syncthreads();
    if (tid == 0) {
        const float a0 = a2[0], a1 = a2[1];
        const float mx = fmaxf(a0, a1);
        const float e0 = expf(a0 - mx), e1 = expf(a1 - mx);
        const float sum = e0 + e1;
        act[2 * s] = e0 / sum;
        act[2 * s + 1] = e1 / sum;
    }
}

}  // namespace

cudaError_t launch_tail(const float* x, const int* cu_seqlens, const uint32_t* markers, const int* cu_markers,
                        int n_seqs, int G, const TailWeights& w, float* mv, float* partial, float* logits, float* act,
                        float* pooled, int* err, cudaStream_t s) {
    if (n_seqs <= 0) return cudaSuccess;
    if (G > 0) {
        marker_ln_kernel<<<(G + 7) / 8, 256, 0, s>>>(x, cu_seqlens, markers, cu_markers, n_seqs, G, w.s0w, w.s0b, mv,
                                                     err);
        scorer_kernel<<<dim3((G + SM_ROWS - 1) / SM_ROWS, D / SM_COLS), 256, 0, s>>>(mv, G, w.s1w, w.s1b, w.s3w,
                                                                                      partial);
    }
    act_kernel<<<n_seqs, 256, 0, s>>>(x, cu_seqlens, cu_markers, partial, w, logits, act, pooled);
    return cudaGetLastError();
}

}  // namespace laya
