// norm.cu -- LayerNorm, embedding gather and the final-norm/type-embedding
// step, one warp per 768-wide row with 16-byte loads and stores.
//
// LayerNorm is the reference's two-pass form (src/main.zig:83-95): mean,
// then the mean of squared deviations, r = 1/sqrt(var + 1e-5), out =
// (x - mean) * r * w (+ b). The sums run as warp reductions instead of one
// sequential f32 chain.
#include "kernels.cuh"

namespace laya {
namespace {

// Lane `lane` owns elements [i*256 + lane*8, +8) for i = 0..2.
struct Row {
    float v[24];
};

__device__ __forceinline__ void load_f32_row(Row& r, const float* src, int lane) {
#pragma unroll
    for (int i = 0; i < 3; i++) {
        const float4* p = reinterpret_cast<const float4*>(src + i * 256 + lane * 8);
        const float4 a = p[0], b = p[1];
        r.v[8 * i + 0] = a.x; r.v[8 * i + 1] = a.y; r.v[8 * i + 2] = a.z; r.v[8 * i + 3] = a.w;
        r.v[8 * i + 4] = b.x; r.v[8 * i + 5] = b.y; r.v[8 * i + 6] = b.z; r.v[8 * i + 7] = b.w;
    }
}

__device__ __forceinline__ void store_f32_row(float* dst, const Row& r, int lane) {
#pragma unroll
    for (int i = 0; i < 3; i++) {
        float4* p = reinterpret_cast<float4*>(dst + i * 256 + lane * 8);
        p[0] = make_float4(r.v[8 * i + 0], r.v[8 * i + 1], r.v[8 * i + 2], r.v[8 * i + 3]);
        p[1] = make_float4(r.v[8 * i + 4], r.v[8 * i + 5], r.v[8 * i + 6], r.v[8 * i + 7]);
    }
}

template <typename T>
__device__ __forceinline__ float to_f(T x);
template <>
__device__ __forceinline__ float to_f<__nv_bfloat16>(__nv_bfloat16 x) { return __bfloat162float(x); }
template <>
__device__ __forceinline__ float to_f<__half>(__half x) { return __half2float(x); }

template <typename T>
__device__ __forceinline__ void load16_row(Row& r, const T* src, int lane) {
#pragma unroll
    for (int i = 0; i < 3; i++) {
        const uint4 u = *reinterpret_cast<const uint4*>(src + i * 256 + lane * 8);
        const T* e = reinterpret_cast<const T*>(&u);
#pragma unroll
        for (int j = 0; j < 8; j++) r.v[8 * i + j] = to_f<T>(e[j]);
    }
}

template <typename T>
__device__ __forceinline__ uint32_t pk(float a, float b);
template <>
__device__ __forceinline__ uint32_t pk<__nv_bfloat16>(float a, float b) {
    __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
}
template <>
__device__ __forceinline__ uint32_t pk<__half>(float a, float b) {
    __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
}

template <typename T>
__device__ __forceinline__ void store16_row(T* dst, const Row& r, int lane) {
#pragma unroll
    for (int i = 0; i < 3; i++) {
        uint4 u;
        u.x = pk<T>(r.v[8 * i + 0], r.v[8 * i + 1]);
        u.y = pk<T>(r.v[8 * i + 2], r.v[8 * i + 3]);
        u.z = pk<T>(r.v[8 * i + 4], r.v[8 * i + 5]);
        u.w = pk<T>(r.v[8 * i + 6], r.v[8 * i + 7]);
        *reinterpret_cast<uint4*>(dst + i * 256 + lane * 8) = u;
    }
}

// In-place LayerNorm of the row held across the warp.
__device__ __forceinline__ void layer_norm(Row& r, const float* w, const float* b, int lane) {
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < 24; i++) s += r.v[i];
    const float mean = warp_sum(s) * (1.0f / D);
    float q = 0.f;
#pragma unroll
    for (int i = 0; i < 24; i++) {
        const float d = r.v[i] - mean;
        q += d * d;
    }
    const float rs = 1.0f / sqrtf(warp_sum(q) * (1.0f / D) + LN_EPS);
#pragma unroll
    for (int i = 0; i < 3; i++) {
        // plain loads: w and b may point to global or to shared memory
        const float4* wp = reinterpret_cast<const float4*>(w + i * 256 + lane * 8);
        const float4 w0 = wp[0], w1 = wp[1];
        const float ww[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
        float bb[8] = {0, 0, 0, 0, 0, 0, 0, 0};
        if (b) {
            const float4* bp = reinterpret_cast<const float4*>(b + i * 256 + lane * 8);
            const float4 b0 = bp[0], b1 = bp[1];
            bb[0] = b0.x; bb[1] = b0.y; bb[2] = b0.z; bb[3] = b0.w;
            bb[4] = b1.x; bb[5] = b1.y; bb[6] = b1.z; bb[7] = b1.w;
        }
#pragma unroll
        for (int j = 0; j < 8; j++) r.v[8 * i + j] = (r.v[8 * i + j] - mean) * rs * ww[j] + bb[j];
    }
}

__device__ __forceinline__ int find_seq(const int* cu, int n, int t) {
    int lo = 0, hi = n;  // cu[lo] <= t < cu[hi]
    while (hi - lo > 1) {
        const int mid = (lo + hi) >> 1;
        if (cu[mid] <= t) lo = mid;
        else hi = mid;
    }
    return lo;
}

// embedJob + normJob (src/main.zig:2543-2555): x = LN(E[id]); also writes the
// 16-bit copy layer 0 multiplies (its attn_norm is the identity), the
// sequence index of each token, and the RoPE (cos, sin) pairs of the token's
// position (src/main.zig:2503-2506) transposed to frequency-major rows
// rope_tok[i][t], so the QKV projection's epilogue, where lane l holds
// token m0 + l, reads them with coalesced loads and no position lookup.
template <typename T>
__global__ void embed_kernel(const uint32_t* __restrict__ ids, const int* __restrict__ cu, int n_seqs, int M,
                             const T* __restrict__ emb, const float* __restrict__ w, float* __restrict__ x,
                             T* __restrict__ xn, const float2* __restrict__ rope, float4* __restrict__ rope_tok,
                             int rope_ld, int* __restrict__ seq_of, int* err) {
    griddep_wait();
    griddep_launch();
    const int t = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (t >= M) return;
    uint32_t id = ids[t];
    if (id >= (uint32_t)VOCAB) {
        if (lane == 0) atomicOr(err, ERR_BAD_INDEX);
        id = 0;
    }
    int p = 0;
    if (lane == 0) {
        const int s = find_seq(cu, n_seqs, t);
        seq_of[t] = s;
        p = t - cu[s];
        // A device-resident offset table is not checked on the host: a token
        // outside its sequence's run [cu[s], cu[s+1]) (offsets out of order,
        // cu[0] != 0 or cu[n_seqs] != M) is flagged; its position is taken as
        // 0 so the RoPE table is never read out of range.
        if (p < 0 || p >= MAX_POS || t >= cu[s + 1]) {
            atomicOr(err, ERR_BAD_INDEX);
            p = 0;
        }
    }
    p = __shfl_sync(0xffffffffu, p, 0);
    if (lane < 16)
        rope_tok[(size_t)lane * rope_ld + t] = reinterpret_cast<const float4*>(rope + (size_t)p * 32)[lane];
    Row r;
    load16_row<T>(r, emb + (size_t)id * D, lane);
    layer_norm(r, w, nullptr, lane);
    store_f32_row(x + (size_t)t * D, r, lane);
    store16_row<T>(xn + (size_t)t * D, r, lane);
}

// normIntoJob (src/main.zig:2596-2603): xn = LN(x), x untouched. The grid
// is sized to the SMs' resident blocks and each warp strides over rows,
// loading its next row while it normalises the current one, so every warp
// keeps a row's loads in flight; the block stages the gain and bias in
// shared memory once.
template <typename T>
__global__ void __launch_bounds__(256) ln_kernel(const float* __restrict__ x, T* __restrict__ xn,
                                                 const float* __restrict__ w, const float* __restrict__ b, int M) {
    __shared__ __align__(16) float sw[D];
    __shared__ __align__(16) float sb[D];
    griddep_launch();
    const int lane = threadIdx.x & 31;
    const int nw = gridDim.x * (blockDim.x >> 5);
    int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    for (int i = threadIdx.x; i < D; i += blockDim.x) {  // weights: no earlier kernel writes them
        sw[i] = w[i];
        sb[i] = b ? b[i] : 0.0f;
    }
    griddep_wait();
    Row ra, rb;
    if (row < M) load_f32_row(ra, x + (size_t)row * D, lane);
    __syncthreads();
    // two row buffers used in turn: no register copies between iterations
    while (row < M) {
        int next = row + nw;
        if (next < M) load_f32_row(rb, x + (size_t)next * D, lane);
        layer_norm(ra, sw, sb, lane);
        store16_row<T>(xn + (size_t)row * D, ra, lane);
        row = next;
        if (row >= M) break;
        next = row + nw;
        if (next < M) load_f32_row(ra, x + (size_t)next * D, lane);
        layer_norm(rb, sw, sb, lane);
        store16_row<T>(xn + (size_t)row * D, rb, lane);
        row = next;
    }
}

// final LN + typeEmbJob (src/main.zig:2708-2711) fused with the first head
// layer's norm1 (2716): x = LN_final(x) + type_emb[qtype of the row's
// sequence]; xn = LN(x; w1, b1).
template <typename T>
__global__ void final_kernel(float* __restrict__ x, T* __restrict__ xn, const float* __restrict__ wf,
                             const float* __restrict__ type_emb, const uint32_t* __restrict__ qtypes,
                             const int* __restrict__ seq_of, const float* __restrict__ w1,
                             const float* __restrict__ b1, int M, float* __restrict__ pre_temb, int* err) {
    griddep_wait();
    griddep_launch();
    const int t = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (t >= M) return;
    Row r;
    load_f32_row(r, x + (size_t)t * D, lane);
    layer_norm(r, wf, nullptr, lane);
    if (pre_temb) store_f32_row(pre_temb + (size_t)t * D, r, lane);  // the "final" --dumpstats point
    uint32_t qt = qtypes[seq_of[t]];
    if (qt >= 3) {  // device-resident qtypes are not checked on the host
        if (lane == 0) atomicOr(err, ERR_BAD_INDEX);
        qt = 0;
    }
    Row te;
    load_f32_row(te, type_emb + (size_t)qt * D, lane);
#pragma unroll
    for (int i = 0; i < 24; i++) r.v[i] += te.v[i];
    store_f32_row(x + (size_t)t * D, r, lane);
    layer_norm(r, w1, b1, lane);
    store16_row<T>(xn + (size_t)t * D, r, lane);
}

constexpr int ROWS_PER_BLOCK = 8;  // 256 threads

// dumpStats (src/main.zig:113-121): x[0], x[1], x[2], and the sum and the
// absolute sum of all n values in f64. One 1024-thread block: coalesced
// strided partial sums per thread, then a fixed-order tree, so the result
// does not depend on scheduling.
constexpr int STATS_THREADS = 1024;
__global__ void __launch_bounds__(STATS_THREADS) dump_stats_kernel(const float* __restrict__ x, size_t n,
                                                                   double* __restrict__ out) {
    __shared__ double ss[STATS_THREADS], sa[STATS_THREADS];
    griddep_wait();
    griddep_launch();
    double sum = 0.0, asum = 0.0;
    for (size_t i = threadIdx.x; i < n; i += STATS_THREADS) {
        const double v = x[i];
        sum += v;
        asum += fabs(v);
    }
    ss[threadIdx.x] = sum;
    sa[threadIdx.x] = asum;
    __syncthreads();
#pragma unroll 1
    for (int w = STATS_THREADS / 2; w > 0; w >>= 1) {
        if ((int)threadIdx.x < w) {
            ss[threadIdx.x] += ss[threadIdx.x + w];
            sa[threadIdx.x] += sa[threadIdx.x + w];
        }
        __syncthreads();
    }
    if (threadIdx.x == 0) {
        out[0] = n > 0 ? x[0] : 0.0;
        out[1] = n > 1 ? x[1] : 0.0;
        out[2] = n > 2 ? x[2] : 0.0;
        out[3] = ss[0];
        out[4] = sa[0];
    }
}

}  // namespace

cudaError_t launch_dump_stats(const float* x, size_t n, double* out5, cudaStream_t s) {
    return launch_k(dump_stats_kernel, 1, STATS_THREADS, 0, s, x, n, out5);
}

cudaError_t launch_embed(bool bf16, const uint32_t* ids, const int* cu, int n_seqs, int M, const void* emb,
                         const float* w, float* x, void* xn, const float2* rope, float4* rope_tok, int rope_ld,
                         int* seq_of, int* err, cudaStream_t s) {
    if (M <= 0) return cudaSuccess;
    const int grid = (M + ROWS_PER_BLOCK - 1) / ROWS_PER_BLOCK;
    if (bf16)
        return launch_k(embed_kernel<__nv_bfloat16>, grid, 32 * ROWS_PER_BLOCK, 0, s, ids, cu, n_seqs, M,
                        static_cast<const __nv_bfloat16*>(emb), w, x, static_cast<__nv_bfloat16*>(xn), rope, rope_tok,
                        rope_ld, seq_of, err);
    else
        return launch_k(embed_kernel<__half>, grid, 32 * ROWS_PER_BLOCK, 0, s, ids, cu, n_seqs, M,
                        static_cast<const __half*>(emb), w, x, static_cast<__half*>(xn), rope, rope_tok, rope_ld, seq_of,
                        err);
    return cudaGetLastError();
}

cudaError_t launch_ln(bool bf16, const float* x, void* xn, const float* w, const float* b, int M, int num_sms,
                      cudaStream_t s) {
    if (M <= 0) return cudaSuccess;
    // resident blocks per SM, once per process (every device here is a B200)
    static const int per_sm = [] {
        int n = 0;
        if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, ln_kernel<__nv_bfloat16>, 32 * ROWS_PER_BLOCK, 0) !=
                cudaSuccess ||
            n < 1)
            n = 1;
        return n;
    }();
    const int blocks_for_rows = (M + ROWS_PER_BLOCK - 1) / ROWS_PER_BLOCK;  // one row per warp
    const int grid = blocks_for_rows < num_sms * per_sm ? blocks_for_rows : num_sms * per_sm;
    if (bf16)
        return launch_k(ln_kernel<__nv_bfloat16>, grid, 32 * ROWS_PER_BLOCK, 0, s, x,
                        static_cast<__nv_bfloat16*>(xn), w, b, M);
    else
        return launch_k(ln_kernel<__half>, grid, 32 * ROWS_PER_BLOCK, 0, s, x, static_cast<__half*>(xn), w, b, M);
    return cudaGetLastError();
}

cudaError_t launch_final(bool bf16, float* x, void* xn, const float* wf, const float* type_emb,
                         const uint32_t* qtypes, const int* seq_of, const float* w1, const float* b1, int M,
                         float* pre_temb, int* err, cudaStream_t s) {
    if (M <= 0) return cudaSuccess;
    const int grid = (M + ROWS_PER_BLOCK - 1) / ROWS_PER_BLOCK;
    if (bf16)
        return launch_k(final_kernel<__nv_bfloat16>, grid, 32 * ROWS_PER_BLOCK, 0, s, x,
                        static_cast<__nv_bfloat16*>(xn), wf, type_emb, qtypes, seq_of, w1, b1, M, pre_temb, err);
    else
        return launch_k(final_kernel<__half>, grid, 32 * ROWS_PER_BLOCK, 0, s, x, static_cast<__half*>(xn), wf,
                        type_emb, qtypes, seq_of, w1, b1, M, pre_temb, err);
    return cudaGetLastError();
}

}  // namespace laya
