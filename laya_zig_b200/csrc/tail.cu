// tail.cu -- option-marker scorer and act/escalate head (src/main.zig:2756-2814).
//
// Three small kernels over all sequences of a batch at once:
//   marker_ln   x[marker token] -> LayerNorm(scorer.0 w, b)        (2761-2763)
//   scorer      h = gelu(scorer.1 . v + b); partial dot with scorer.3 over
//               each group of 64 outputs, summed later in a fixed order
//               (2764-2767), so the result does not depend on scheduling;
//               K split over a cluster of 4 CTAs, reduced in rank order
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
                                 int G, int M, const float* __restrict__ w, const float* __restrict__ b,
                                 float* __restrict__ mv, int* err) {
    griddep_wait();
    griddep_launch();
    const int g = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (g >= G) return;
    // Device-resident offsets are not checked on the host. The marker must
    // lie in its sequence's marker run and inside the sequence, and the
    // sequence inside the M rows of x; otherwise the marker is flagged and
    // its vector zeroed, and no row outside x is read.
    const int s = find_seq(cu_markers, n_seqs, g);
    const int rows = M >= 0 ? M : cu_seqlens[n_seqs];
    const int cs = cu_seqlens[s], L = cu_seqlens[s + 1] - cs;
    const uint32_t m = markers[g];
    if (g < cu_markers[s] || g >= cu_markers[s + 1] || cs < 0 || L <= 0 || cs > rows - L || m >= (uint32_t)L) {
        if (lane == 0) atomicOr(err, ERR_BAD_INDEX);
#pragma unroll
        for (int i = 0; i < 24; i++) mv[(size_t)g * D + i * 32 + lane] = 0.f;
        return;
    }
    const float* row = x + (size_t)(cs + m) * D;
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

// scorer.1 + gelu + dot with scorer.3, as an f32 tile GEMM: a cluster of
// SC_SPLIT CTAs takes 32 markers x 64 scorer outputs, CTA z of the cluster
// the K range [z*192, z*192 + 192), each of its 256 threads 2 markers x 4
// outputs; k-chunks of 32 are staged in shared memory and the next chunk's
// loads are issued before the current chunk's FMAs. The partial tiles meet
// in rank 0 through distributed shared memory, summed in rank order (a fixed
// order, so results do not depend on scheduling), and rank 0 sums the
// tile's 64 outputs of a marker (after gelu and the scorer.3 weights) into
// one partial sum. Splitting K gives SC_SPLIT times the CTAs of a 32 x 64
// tiling (768 for 512 markers), enough warps per SM to hide the shared
// memory and FMA latencies.
constexpr int SC_M = 32, SC_N = 64, SC_K = 32, SC_SPLIT = 4, SC_KR = D / SC_SPLIT;
static_assert(SC_KR % SC_K == 0, "scorer K split");

__device__ __forceinline__ float4 ld_cluster_f4(uint32_t addr) {
    float4 v;
    asm volatile("ld.shared::cluster.v4.f32 {%0, %1, %2, %3}, [%4];"
                 : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
                 : "r"(addr)
                 : "memory");
    return v;
}

__global__ void __cluster_dims__(1, 1, SC_SPLIT) __launch_bounds__(256)
    scorer_kernel(const float* __restrict__ mv, int G, const float* __restrict__ w1, const float* __restrict__ b1,
                  const float* __restrict__ w3, float* __restrict__ partial) {
    __shared__ float As[SC_K][SC_M + 4];  // [k][marker]
    __shared__ float Bs[SC_K][SC_N + 4];  // [k][output]
    __shared__ float4 red[2][256];        // this CTA's partial tile, by thread
    const int g0 = blockIdx.x * SC_M, j0 = blockIdx.y * SC_N, kbeg = blockIdx.z * SC_KR;
    const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;  // outputs tx*4.., markers ty*2..
    // loads: A 32x32 -> 4 floats per thread, B 64x32 -> 8 floats per thread
    const int ar = tid >> 3, ac = (tid & 7) * 4;        // A row (marker) 0..31, k offset
    const int br = tid >> 2, bc = (tid & 3) * 8;        // B row (output) 0..63, k offset
    const bool a_ok = g0 + ar < G;
    const float* ap = mv + (size_t)(a_ok ? g0 + ar : 0) * D + kbeg + ac;
    const float* bp = w1 + (size_t)(j0 + br) * D + kbeg + bc;
    griddep_launch();
    float4 rb0 = *reinterpret_cast<const float4*>(bp), rb1 = *reinterpret_cast<const float4*>(bp + 4);  // weights
    griddep_wait();  // mv comes from the marker LayerNorm
    float4 ra = a_ok ? *reinterpret_cast<const float4*>(ap) : make_float4(0.f, 0.f, 0.f, 0.f);
    float acc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
    for (int k0 = 0; k0 < SC_KR; k0 += SC_K) {
        __syncthreads();
        As[ac + 0][ar] = ra.x; As[ac + 1][ar] = ra.y; As[ac + 2][ar] = ra.z; As[ac + 3][ar] = ra.w;
        Bs[bc + 0][br] = rb0.x; Bs[bc + 1][br] = rb0.y; Bs[bc + 2][br] = rb0.z; Bs[bc + 3][br] = rb0.w;
        Bs[bc + 4][br] = rb1.x; Bs[bc + 5][br] = rb1.y; Bs[bc + 6][br] = rb1.z; Bs[bc + 7][br] = rb1.w;
        __syncthreads();
        if (k0 + SC_K < SC_KR) {  // next chunk in flight while this one is consumed
            ra = a_ok ? *reinterpret_cast<const float4*>(ap + k0 + SC_K) : make_float4(0.f, 0.f, 0.f, 0.f);
            rb0 = *reinterpret_cast<const float4*>(bp + k0 + SC_K);
            rb1 = *reinterpret_cast<const float4*>(bp + k0 + SC_K + 4);
        }
#pragma unroll
        for (int k = 0; k < SC_K; k++) {
            const float2 av = *reinterpret_cast<const float2*>(&As[k][ty * 2]);
            const float4 bv = *reinterpret_cast<const float4*>(&Bs[k][tx * 4]);
            acc[0][0] = fmaf(av.x, bv.x, acc[0][0]); acc[0][1] = fmaf(av.x, bv.y, acc[0][1]);
            acc[0][2] = fmaf(av.x, bv.z, acc[0][2]); acc[0][3] = fmaf(av.x, bv.w, acc[0][3]);
            acc[1][0] = fmaf(av.y, bv.x, acc[1][0]); acc[1][1] = fmaf(av.y, bv.y, acc[1][1]);
            acc[1][2] = fmaf(av.y, bv.z, acc[1][2]); acc[1][3] = fmaf(av.y, bv.w, acc[1][3]);
        }
    }
    red[0][tid] = make_float4(acc[0][0], acc[0][1], acc[0][2], acc[0][3]);
    red[1][tid] = make_float4(acc[1][0], acc[1][1], acc[1][2], acc[1][3]);
    cluster_sync();
    if (cluster_rank() == 0) {
#pragma unroll
        for (int r = 1; r < SC_SPLIT; r++) {
#pragma unroll
            for (int i = 0; i < 2; i++) {
                const float4 v = ld_cluster_f4(mapa_shared(smem_u32(&red[i][tid]), r));
                acc[i][0] += v.x;
                acc[i][1] += v.y;
                acc[i][2] += v.z;
                acc[i][3] += v.w;
            }
        }
#pragma unroll
        for (int i = 0; i < 2; i++) {
            float p = 0.f;
#pragma unroll
            for (int c = 0; c < 4; c++) {
                const int j = j0 + tx * 4 + c;
                p += gelu_scalar(acc[i][c] + b1[j]) * w3[j];
            }
            // the 16 threads sharing a marker are 16 consecutive lanes
#pragma unroll
            for (int o = 8; o > 0; o >>= 1) p += __shfl_xor_sync(0xffffffffu, p, o);
            const int g = g0 + ty * 2 + i;
            if (tx == 0 && g < G) partial[(size_t)g * SCORER_GROUPS + blockIdx.y] = p;
        }
    }
    cluster_sync();  // the other ranks keep their shared memory until rank 0 has read it
}

// One CTA (1024 threads) per sequence: logits from the partial sums, pooled
// = x[CLS], the act features, then [pooled | features] (772) -> 256 with the
// transposed act_head.0 weight (thread j of each 256-thread slice reads
// column j: coalesced), gelu, -> 2, softmax.
constexpr int ACT_THREADS = 1024, ACT_SLICES = ACT_THREADS / 256, ACT_IN = D + 4;
__global__ void __launch_bounds__(ACT_THREADS) act_kernel(const float* __restrict__ x,
                                                          const int* __restrict__ cu_seqlens,
                                                          const int* __restrict__ cu_markers, int G, int M,
                                                          const float* __restrict__ partial, TailWeights w,
                                                          float* __restrict__ logits, float* __restrict__ act,
                                                          float* __restrict__ pooled, int* err) {
    __shared__ float lg[MAX_MARKERS_PER_SEQ];
    __shared__ float act_in[ACT_IN];
    __shared__ float hpart[ACT_SLICES][256];
    __shared__ float a2[2];
    griddep_wait();
    griddep_launch();
    const int s = blockIdx.x, n_seqs = gridDim.x, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    // Device-resident offsets are not checked on the host. A marker run that
    // is not inside [0, G) or is longer than MAX_MARKERS_PER_SEQ is flagged
    // and scored as empty (its logits are not written); a [CLS] row outside
    // the M rows of x is flagged and read as zeros.
    const int gb = cu_markers[s], ge = cu_markers[s + 1];
    const int rows = M >= 0 ? M : cu_seqlens[n_seqs];
    const int cs = cu_seqlens[s];
    const bool bad_k = gb < 0 || ge < gb || ge > G || ge - gb > MAX_MARKERS_PER_SEQ;
    const bool bad_cls = cs < 0 || cs >= rows;
    const bool bad_tab = s == 0 && (cu_markers[0] != 0 || cu_markers[n_seqs] != G || cu_seqlens[0] != 0);
    if (tid == 0 && (bad_k || bad_cls || bad_tab)) atomicOr(err, ERR_BAD_INDEX);
    const int K = bad_k ? 0 : ge - gb;
    for (int r = tid; r < K; r += ACT_THREADS) {
        float v = 0.f;
        for (int c = 0; c < SCORER_GROUPS; c++) v += partial[(size_t)(gb + r) * SCORER_GROUPS + c];
        v += w.s3b[0];
        lg[r] = v;
        logits[gb + r] = v;
    }
    const float* cls = x + (size_t)(bad_cls ? 0 : cs) * D;
    for (int c = tid; c < D; c += ACT_THREADS) {
        const float v = bad_cls ? 0.f : cls[c];
        act_in[c] = v;
        pooled[(size_t)s * D + c] = v;
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
    {
        const int j = tid & 255, sl = tid >> 8;
        const int k0 = sl * ((ACT_IN + ACT_SLICES - 1) / ACT_SLICES);
        const int k1 = min(ACT_IN, k0 + (ACT_IN + ACT_SLICES - 1) / ACT_SLICES);
        float p0 = 0.f, p1 = 0.f;
        int k = k0;
#pragma unroll 4
        for (; k + 1 < k1; k += 2) {
            p0 = fmaf(act_in[k], w.a0t[(size_t)k * 256 + j], p0);
            p1 = fmaf(act_in[k + 1], w.a0t[(size_t)(k + 1) * 256 + j], p1);
        }
        if (k < k1) p0 = fmaf(act_in[k], w.a0t[(size_t)k * 256 + j], p0);
        hpart[sl][j] = p0 + p1;
    }
    __syncthreads();
    if (tid < 256) {
        float h = 0.f;
#pragma unroll
        for (int sl = 0; sl < ACT_SLICES; sl++) h += hpart[sl][tid];
        hpart[0][tid] = gelu_scalar(h + w.a0b[tid]);
    }
    __syncthreads();
    if (warp < 2) {
        float p = 0.f;
        for (int k = lane; k < 256; k += 32) p = fmaf(hpart[0][k], w.a2w[warp * 256 + k], p);
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
                        int n_seqs, int G, int M, const TailWeights& w, float* mv, float* partial, float* logits,
                        float* act, float* pooled, int* err, cudaStream_t s) {
    if (n_seqs <= 0) return cudaSuccess;
    if (G > 0) {
        cudaError_t e = launch_k(marker_ln_kernel, (G + 7) / 8, 256, 0, s, x, cu_seqlens, markers, cu_markers, n_seqs,
                                 G, M, w.s0w, w.s0b, mv, err);
        if (e != cudaSuccess) return e;
        e = launch_k(scorer_kernel, dim3((G + SC_M - 1) / SC_M, D / SC_N, SC_SPLIT), 256, 0, s, mv, G, w.s1w, w.s1b,
                     w.s3w, partial);
        if (e != cudaSuccess) return e;
    }
    return launch_k(act_kernel, n_seqs, ACT_THREADS, 0, s, x, cu_seqlens, cu_markers, G, M, partial, w, logits, act,
                    pooled, err);
}

}  // namespace laya
