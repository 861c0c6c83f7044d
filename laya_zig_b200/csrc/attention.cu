// attention.cu -- bidirectional multi-head attention over packed sequences.
//
// Replaces attWorker (src/main.zig:2431-2489): per query row i and head h,
// softmax(q_i . k_j / 8) over j in [klo, khi) -- all keys of the sequence on
// global layers, |i - j| <= 64 on sliding layers -- then the weighted sum of
// v_j. Here one CTA takes 64 query rows of one head of one sequence; four
// warps hold 16 rows each. Scores and P.V run on the tensor cores
// (mma.sync m16n8k16, f32 accumulate); the softmax is the online
// (running max / running sum) form in f32 with exp2, normalised once at the
// end as the reference does (2479-2486). Q and the key/value tiles of 64
// keys arrive by TMA (one thread issues cp.async.bulk.tensor boxes of 64
// rows x 128 bytes; the 128-byte swizzle is the XOR layout the ldmatrix
// addressing below reads) into a 3-deep ring, each slot completing on its
// own mbarrier; the prologue requests Q and the first three tiles at once,
// which is every tile a 64-row block of a sequence of up to 192 tokens
// needs. Rows past the sequence end hold the next sequence's keys (masked
// below) or, past the batch, the TMA's zero fill.
//
// Inputs come straight from the QKV projection's output: row r of `qkv`
// holds q | k | v (each 12 heads x 64, RoPE already applied to q and k),
// which is the reference's split layout (splitJob 2626-2634).
#include "attention.cuh"

namespace laya {
namespace {

constexpr int QB = 64;   // query rows per CTA
constexpr int KB = 64;   // keys per tile
constexpr int NST = 3;   // key/value tiles in flight
constexpr int THREADS = 128;
constexpr int TILE_BYTES = KB * 64 * 2;                            // 8 KB: 64 rows x 64 16-bit
constexpr int BAR_OFFSET = (QB + 2 * NST * KB) * 64 * 2;               // 56 KB of tiles
constexpr int SMEM_BYTES = BAR_OFFSET + 64 + 1024;                     // barriers, 1 KB alignment slack

// element offset of (row, col) in a 64x64 16-bit tile whose 16-byte chunks
// are XOR-swizzled by row, so ldmatrix row fetches never share a bank.
__device__ __forceinline__ int swz(int r, int c) { return r * 64 + ((((c >> 3) ^ (r & 7))) << 3) + (c & 7); }

// 2^x with the SFU's approximate exp2 (relative error ~2^-22; -inf -> 0),
// far below the bf16 rounding P gets for the tensor-core P.V product.
__device__ __forceinline__ float ex2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], const void* p) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(smem_u32(p)));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t (&r)[4], const void* p) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(smem_u32(p)));
}

template <typename T>
__device__ __forceinline__ void mma16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1);
template <>
__device__ __forceinline__ void mma16816<__nv_bfloat16>(float (&c)[4], const uint32_t (&a)[4], uint32_t b0,
                                                        uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
template <>
__device__ __forceinline__ void mma16816<__half>(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

template <typename T>
__device__ __forceinline__ uint32_t pack2(float a, float b);
template <>
__device__ __forceinline__ uint32_t pack2<__nv_bfloat16>(float a, float b) {
    __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
}
template <>
__device__ __forceinline__ uint32_t pack2<__half>(float a, float b) {
    __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
}

template <typename T>
__global__ void __launch_bounds__(THREADS, 3) attention_kernel(const __grid_constant__ CUtensorMap qkv_map,
                                                            T* __restrict__ out, const int* __restrict__ cu_seqlens,
                                                            int M, int max_len, int window, int* err, int long_len) {
    // Q tile, then NST K tiles, then NST V tiles, 1 KB aligned (the TMA
    // swizzle pattern is anchored to 1 KB); then the slots' barriers
    extern __shared__ uint8_t att_smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(att_smem_raw) + 1023) & ~uintptr_t(1023));
    T* sQ = reinterpret_cast<T*>(smem);
    T* sK = sQ + QB * 64;
    T* sV = sK + NST * KB * 64;
    uint64_t* bar = reinterpret_cast<uint64_t*>(smem + BAR_OFFSET);  // [0] Q, [1 + slot] K/V
    __shared__ int abort_flag;

    griddep_launch();
    const int seq = blockIdx.z, h = blockIdx.y;
    const int start = cu_seqlens[seq];  // batch offsets: written before the forward starts
    const int L = cu_seqlens[seq + 1] - start;
    // A device-resident offset table is not checked on the host: a sequence
    // that is not a run of [0, M) no longer than max_len (the grid's extent)
    // is flagged and left alone, so no row outside the batch is touched.
    if (start < 0 || L < 0 || L > max_len || start > M - L) {
        if (blockIdx.x == 0 && threadIdx.x == 0) atomicOr(err, ERR_BAD_INDEX);
        griddep_exit();
        return;
    }
    const int q0 = blockIdx.x * QB;
    if (q0 >= L || L >= long_len) {  // past the sequence end, or the tcgen05 kernel's sequence
        griddep_exit();
        return;
    }
    if (threadIdx.x == 0) {
        for (int i = 0; i <= NST; i++) mbar_init(&bar[i], 1);
        abort_flag = 0;
        fence_barrier_init();
        prefetch_tmap(&qkv_map);
    }
    __syncthreads();
    griddep_wait();  // qkv comes from the preceding projection

    int klo = 0, khi = L;
    if (window >= 0) {
        klo = max(0, q0 - window);
        khi = min(L, q0 + QB - 1 + window + 1);
    }
    const int kt0 = klo / KB, kt1 = (khi + KB - 1) / KB;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    // Prologue: Q and the first NST key/value tiles all requested at once
    // (a 64-row block of a <= 192-token sequence needs at most 3).
    int issued[NST];  // thread 0: phase of each slot's last request, -1 if none
    if (threadIdx.x == 0) {
        mbar_arrive_expect_tx(&bar[0], TILE_BYTES);
        tma_load_2d(sQ, &qkv_map, &bar[0], h * HD, start + q0);
#pragma unroll
        for (int i = 0; i < NST; i++) {
            issued[i] = -1;
            if (kt0 + i < kt1) {
                mbar_arrive_expect_tx(&bar[1 + i], 2 * TILE_BYTES);
                tma_load_2d(sK + i * KB * 64, &qkv_map, &bar[1 + i], D + h * HD, start + (kt0 + i) * KB);
                tma_load_2d(sV + i * KB * 64, &qkv_map, &bar[1 + i], 2 * D + h * HD, start + (kt0 + i) * KB);
                issued[i] = 0;
            }
        }
    }

    const float sl2 = 0.125f * 1.4426950408889634f;  // 1/sqrt(64) * log2(e)
    const int qi0 = q0 + warp * 16 + (lane >> 2), qi1 = qi0 + 8;
    float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
    float o[8][4];
#pragma unroll
    for (int j = 0; j < 8; j++) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
    uint32_t qa[4][4];

    bool ok = true;
    for (int kt = kt0; kt < kt1; kt++) {
        const int slot = (kt - kt0) % NST;
        ok = mbar_wait(&bar[1 + slot], ((kt - kt0) / NST) & 1, err, &abort_flag);
        if (kt == kt0 && ok) ok = mbar_wait(&bar[0], 0, err, &abort_flag);
        if (__syncthreads_or(!ok)) {  // every thread leaves together
            ok = false;
            break;
        }
        if (kt == kt0) {
#pragma unroll
            for (int ks = 0; ks < 4; ks++) {
                const int r = warp * 16 + (lane & 15), c = ks * 16 + (lane >> 4) * 8;
                ldsm_x4(qa[ks], sQ + swz(r, c));
            }
        }
        // S = Q K^T for 64 keys: 8 n-tiles of 8 keys
        float s[8][4];
#pragma unroll
        for (int j = 0; j < 8; j++) s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.f;
        const T* K = sK + slot * KB * 64;
#pragma unroll
        for (int ks = 0; ks < 4; ks++) {
#pragma unroll
            for (int np = 0; np < 4; np++) {
                uint32_t b[4];
                const int mi = lane >> 3;
                const int r = np * 16 + (lane & 7) + (mi >> 1) * 8, c = ks * 16 + (mi & 1) * 8;
                ldsm_x4(b, K + swz(r, c));
                mma16816<T>(s[2 * np], qa[ks], b[0], b[1]);
                mma16816<T>(s[2 * np + 1], qa[ks], b[2], b[3]);
            }
        }
        // Masks only on tiles that cross the sequence end or a window edge
        // (keys j of the tile, rows i of the block: j < L and |i - j| <= window).
        const int klo = kt * KB, khi = kt * KB + KB - 1;
        const bool need_mask = khi >= L || (window >= 0 && (q0 + QB - 1 - klo > window || khi - q0 > window));
        if (need_mask) {
            // row qi sees keys [lo, hi]; element (j, e) of this thread holds
            // key klo + 8j + 2(lane & 3) + e, so one unsigned compare of its
            // offset from lo against hi - lo tests both ends
            int lo0 = 0, hi0 = L - 1, lo1 = 0, hi1 = L - 1;
            if (window >= 0) {
                lo0 = max(0, qi0 - window);
                hi0 = min(L - 1, qi0 + window);
                lo1 = max(0, qi1 - window);
                hi1 = min(L - 1, qi1 + window);
            }
            const int kb = klo + 2 * (lane & 3);
            const int d0 = kb - lo0, d1 = kb - lo1;
            // an empty range (a row past the sequence end, never stored) masks everything
            const bool e0 = hi0 < lo0, e1 = hi1 < lo1;
            const unsigned r0 = e0 ? 0u : (unsigned)(hi0 - lo0), r1 = e1 ? 0u : (unsigned)(hi1 - lo1);
#pragma unroll
            for (int j = 0; j < 8; j++) {
#pragma unroll
                for (int e = 0; e < 2; e++) {
                    if (e0 || (unsigned)(d0 + j * 8 + e) > r0) s[j][e] = -INFINITY;
                    if (e1 || (unsigned)(d1 + j * 8 + e) > r1) s[j][2 + e] = -INFINITY;
                }
            }
        }
        // online softmax over raw scores, two rows per thread (qi0, qi1);
        // p = 2^(s * log2(e)/8 - max * log2(e)/8)
        // row maxima as balanced trees (depth 4, not a 16-long chain)
        float ta[8], tb[8];
#pragma unroll
        for (int j = 0; j < 8; j++) {
            ta[j] = fmaxf(s[j][0], s[j][1]);
            tb[j] = fmaxf(s[j][2], s[j][3]);
        }
#pragma unroll
        for (int w = 4; w > 0; w >>= 1) {
#pragma unroll
            for (int j = 0; j < w; j++) {
                ta[j] = fmaxf(ta[j], ta[j + w]);
                tb[j] = fmaxf(tb[j], tb[j + w]);
            }
        }
        float mx0 = ta[0], mx1 = tb[0];
        mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
        mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
        mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
        mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
        const float n0 = fmaxf(m0, mx0), n1 = fmaxf(m1, mx1);
        const float u0 = n0 == -INFINITY ? 0.f : n0 * sl2, u1 = n1 == -INFINITY ? 0.f : n1 * sl2;
        const float a0 = ex2(m0 * sl2 - u0), a1 = ex2(m1 * sl2 - u1);
        m0 = n0;
        m1 = n1;
        float rs0 = 0.f, rs1 = 0.f;
#pragma unroll
        for (int j = 0; j < 8; j++) {
            s[j][0] = ex2(fmaf(s[j][0], sl2, -u0));
            s[j][1] = ex2(fmaf(s[j][1], sl2, -u0));
            s[j][2] = ex2(fmaf(s[j][2], sl2, -u1));
            s[j][3] = ex2(fmaf(s[j][3], sl2, -u1));
            rs0 += s[j][0] + s[j][1];
            rs1 += s[j][2] + s[j][3];
        }
        l0 = l0 * a0 + rs0;
        l1 = l1 * a1 + rs1;
#pragma unroll
        for (int j = 0; j < 8; j++) {
            o[j][0] *= a0;
            o[j][1] *= a0;
            o[j][2] *= a1;
            o[j][3] *= a1;
        }
        // O += P V: P as the A operand straight from the score registers
        const T* V = sV + slot * KB * 64;
#pragma unroll
        for (int kk = 0; kk < 4; kk++) {
            uint32_t pa[4];
            pa[0] = pack2<T>(s[2 * kk][0], s[2 * kk][1]);
            pa[1] = pack2<T>(s[2 * kk][2], s[2 * kk][3]);
            pa[2] = pack2<T>(s[2 * kk + 1][0], s[2 * kk + 1][1]);
            pa[3] = pack2<T>(s[2 * kk + 1][2], s[2 * kk + 1][3]);
#pragma unroll
            for (int dp = 0; dp < 4; dp++) {
                uint32_t b[4];
                const int r = kk * 16 + (lane & 7) + ((lane >> 3) & 1) * 8, c = dp * 16 + (lane >> 4) * 8;
                ldsm_x4_t(b, V + swz(r, c));
                mma16816<T>(o[2 * dp], pa, b[0], b[1]);
                mma16816<T>(o[2 * dp + 1], pa, b[2], b[3]);
            }
        }
        __syncthreads();  // every warp is done with this slot before it is refilled
        if (threadIdx.x == 0 && kt + NST < kt1) {
            mbar_arrive_expect_tx(&bar[1 + slot], 2 * TILE_BYTES);
            tma_load_2d(sK + slot * KB * 64, &qkv_map, &bar[1 + slot], D + h * HD, start + (kt + NST) * KB);
            tma_load_2d(sV + slot * KB * 64, &qkv_map, &bar[1 + slot], 2 * D + h * HD, start + (kt + NST) * KB);
            issued[slot] = ((kt + NST - kt0) / NST) & 1;
        }
    }
    if (!ok) {
        // a wait gave up: every box requested lands before the CTA (and its
        // shared memory) goes away; nothing is stored
        if (threadIdx.x == 0) {
            const unsigned long long t0 = globaltimer();
            while (!mbar_try_wait(&bar[0], 0) && globaltimer() - t0 < WAIT_LIMIT_NS) {
            }
            for (int i = 0; i < NST; i++)
                if (issued[i] >= 0)
                    while (!mbar_try_wait(&bar[1 + i], (uint32_t)issued[i]) && globaltimer() - t0 < WAIT_LIMIT_NS) {
                    }
        }
        return;
    }

    l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
    l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
    l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
    l1 += __shfl_xor_sync(0xffffffffu, l1, 2);
    const float i0 = 1.0f / l0, i1 = 1.0f / l1;
    T* dst = out + (size_t)start * D + h * HD + 2 * (lane & 3);
#pragma unroll
    for (int j = 0; j < 8; j++) {
        if (qi0 < L) *reinterpret_cast<uint32_t*>(dst + (size_t)qi0 * D + j * 8) = pack2<T>(o[j][0] * i0, o[j][1] * i0);
        if (qi1 < L) *reinterpret_cast<uint32_t*>(dst + (size_t)qi1 * D + j * 8) = pack2<T>(o[j][2] * i1, o[j][3] * i1);
    }
}

}  // namespace

cudaError_t launch_attention(bool bf16, const CUtensorMap& qkv_map, void* out, const int* cu_seqlens, int n_seqs,
                             int M, int max_len, int window, int* err, cudaStream_t stream, int long_len) {
    if (n_seqs <= 0 || max_len <= 0) return cudaSuccess;
    dim3 grid((max_len + QB - 1) / QB, H, n_seqs);
    if (bf16)
        return launch_k(attention_kernel<__nv_bfloat16>, grid, THREADS, SMEM_BYTES, stream, qkv_map,
                        static_cast<__nv_bfloat16*>(out), cu_seqlens, M, max_len, window, err, long_len);
    return launch_k(attention_kernel<__half>, grid, THREADS, SMEM_BYTES, stream, qkv_map, static_cast<__half*>(out),
                    cu_seqlens, M, max_len, window, err, long_len);
}

int attention_tc_min_len() {
    static const int v = [] {
        const char* e = getenv("LAYA_ATTN_TC_MIN_LEN");
        if (e && *e) {
            const int x = atoi(e);
            return x <= 0 ? 0x7fffffff : x;
        }
        return 2048;  // measured: 1,024 tokens run faster on mma.sync, 2,048 on tcgen05
    }();
    return v;
}

cudaError_t attention_prepare() {
    cudaError_t e = cudaFuncSetAttribute(attention_kernel<__nv_bfloat16>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         SMEM_BYTES);
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(attention_kernel<__half>, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
    if (e == cudaSuccess) e = attention_tc_prepare();
    return e;
}

}  // namespace laya
