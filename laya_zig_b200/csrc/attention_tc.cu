// attention_tc.cu -- tensor-core (tcgen05) attention for long sequences.
//
// Replaces attWorker (src/main.zig:2431-2489) on global-attention layers for
// sequences of at least attention_tc_min_len() tokens. Each CTA takes two
// 128-row query tiles of one head of one sequence and streams the
// sequence's keys and values through shared memory in tiles of 128:
//
//   warp 8      TMA producer: both Q tiles once, then K_j and V_j (128 x 64
//               16-bit boxes, 128-byte swizzle) into a KV_STAGES-deep ring.
//   warp 9      TMEM owner and MMA issuer: S_q = Q_q K_j^T (M 128, N 128,
//               K 64) into TMEM, then O_q += P_q V_j (M 128, N 64, K 128)
//               accumulated in TMEM across key tiles, with P from shared
//               memory and V read MN-major.
//   warps 0-7   two softmax warpgroups, one per query tile; thread t of a
//               group owns query row t (its TMEM lane). Per key tile it
//               copies its 128 scores from TMEM to registers (S_q is then
//               free for the next tile's MMA), takes the row maximum, and
//               writes p = 2^(s*log2(e)/8 - m*log2(e)/8) rounded to 16 bits
//               into one of two P buffers (K-major swizzled, as the MMA
//               reads it), keeping the row sum in f32.
//
// The reference point m of a row moves only when the row's maximum grows by
// more than 8 in the exponent (p then stays below 2^8): the warp rescales
// its rows of the TMEM accumulator and the row sum by 2^(m_old - m_new)
// before the next P.V accumulates. Softmax is invariant to the reference
// point, so the result is that of the online softmax of the mma.sync
// kernel (attention.cu: same scale, same exp2 argument, normalised once at
// the end as the reference does, 2479-2486) up to rounding. Keys past the
// sequence end are masked to -inf; query rows past it are computed and not
// stored. Every wait is bounded (common.cuh): a CTA that gives up sets the
// error word, drains its own TMA loads and MMAs, frees TMEM and exits.
#include <type_traits>

#include "attention.cuh"

namespace laya {
namespace {

constexpr int TQ = 128;        // query rows per tile (one TMEM lane each)
constexpr int TK = 128;        // keys per tile
constexpr int NQT = 2;         // query tiles per CTA
constexpr int KV_STAGES = 2;
constexpr int TC_THREADS = 320;
constexpr int TILE_BYTES = TQ * HD * 2;            // 16 KB: a 128 x 64 16-bit box
constexpr int SMEM_Q = 0;
constexpr int SMEM_K = SMEM_Q + NQT * TILE_BYTES;
constexpr int SMEM_V = SMEM_K + KV_STAGES * TILE_BYTES;
constexpr int SMEM_BAR = SMEM_V + KV_STAGES * TILE_BYTES;  // P lives in TMEM
constexpr int SMEM_TC = SMEM_BAR + 256 + 1024;     // barriers, TMEM slot, 1 KB alignment slack
constexpr uint32_t TMEM_COLS = 512;  // S_0, S_1 [0,256), O_0, O_1 [256,384), P_0, P_1 [384,512)
constexpr uint32_t P_COL = 384;
constexpr uint32_t IDESC_S_BF16 = idesc_f16(TQ, TK, true);
constexpr uint32_t IDESC_S_F16 = idesc_f16(TQ, TK, false);
// P . V: B (= V) is MN-major (head dim contiguous): transpose-B bit 16.
constexpr uint32_t IDESC_O_BF16 = idesc_f16(TQ, HD, true) | (1u << 16);
constexpr uint32_t IDESC_O_F16 = idesc_f16(TQ, HD, false) | (1u << 16);

struct Bars {
    uint64_t q_full;
    uint64_t kv_full[KV_STAGES], kv_empty[KV_STAGES];
    uint64_t s_full[NQT], s_free[NQT], p_full[NQT], o_full[NQT];
    uint64_t drain;
    uint32_t tmem;
    int abort;
};
static_assert(sizeof(Bars) <= 256, "barrier block");

// Named barriers 1 and 2 pass a token between the two softmax warpgroups:
// warpgroup q computes its exponentials only while it holds the token, so
// the SFU serves one group at a time and each group's score loads and row
// maxima overlap the other group's exponentials.
__device__ __forceinline__ void token_wait(int q) {
    asm volatile("bar.sync %0, 256;" ::"r"(1 + q) : "memory");
}
__device__ __forceinline__ void token_pass(int q) {
    asm volatile("bar.arrive %0, 256;" ::"r"(2 - q) : "memory");
}

__device__ __forceinline__ float ex2f(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

template <typename T>
__device__ __forceinline__ uint32_t pack16(float a, float b);
template <>
__device__ __forceinline__ uint32_t pack16<__nv_bfloat16>(float a, float b) {
    __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
}
template <>
__device__ __forceinline__ uint32_t pack16<__half>(float a, float b) {
    __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
}

// P's rounding to 16 bits, two values packed. For bf16 on the integer pipe
// (the SFU, which also converts, is busy with the exponentials): add half a
// bf16 ulp and keep the high halves, round to nearest with ties away from
// zero, for the non-negative finite p here; f16 by conversion.
template <typename T>
__device__ __forceinline__ uint32_t pack_p(float a, float b);
template <>
__device__ __forceinline__ uint32_t pack_p<__nv_bfloat16>(float a, float b) {
    return __byte_perm(__float_as_uint(a) + 0x8000u, __float_as_uint(b) + 0x8000u, 0x7632);
}
template <>
__device__ __forceinline__ uint32_t pack_p<__half>(float a, float b) {
    return pack16<__half>(a, b);
}

// Bounded wait for an mbarrier phase with no abort flag (teardown drains).
__device__ __forceinline__ void drain_wait(uint64_t* bar, uint32_t parity, int* err) {
    const unsigned long long t0 = globaltimer();
    while (!mbar_try_wait(bar, parity))
        if (globaltimer() - t0 > WAIT_LIMIT_NS) {
            atomicOr(err, ERR_WAIT_TIMEOUT);
            return;
        }
}

template <typename T>
__global__ void __launch_bounds__(TC_THREADS, 1)
    attention_tc_kernel(const __grid_constant__ CUtensorMap qkv_map, T* __restrict__ out,
                        const int* __restrict__ cu_seqlens, int M, int max_len, int min_len, int* err) {
    extern __shared__ uint8_t tc_smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(tc_smem_raw) + 1023) & ~uintptr_t(1023));
    Bars* bar = reinterpret_cast<Bars*>(smem + SMEM_BAR);
    volatile int* abort_flag = &bar->abort;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    const int seq = blockIdx.z, h = blockIdx.y;
    const int start = cu_seqlens[seq];  // batch offsets: written before the forward starts
    const int L = cu_seqlens[seq + 1] - start;
    if (start < 0 || L < 0 || L > max_len || start > M - L) {
        if (blockIdx.x == 0 && threadIdx.x == 0) atomicOr(err, ERR_BAD_INDEX);
        griddep_exit();
        return;
    }
    const int q0 = blockIdx.x * (NQT * TQ);
    if (L < min_len || q0 >= L) {  // shorter sequences are the mma.sync kernel's
        griddep_exit();
        return;
    }
    const int nq = min(NQT, (L - q0 + TQ - 1) / TQ);  // query tiles with rows in the sequence
    const int nkt = (L + TK - 1) / TK;

    if (threadIdx.x == 0) {
        mbar_init(&bar->q_full, 1);
        for (int s = 0; s < KV_STAGES; s++) {
            mbar_init(&bar->kv_full[s], 1);
            mbar_init(&bar->kv_empty[s], 1);
        }
        for (int q = 0; q < NQT; q++) {
            mbar_init(&bar->s_full[q], 1);
            mbar_init(&bar->s_free[q], TQ);
            mbar_init(&bar->p_full[q], TQ);
            mbar_init(&bar->o_full[q], 1);
        }
        mbar_init(&bar->drain, 1);
        bar->abort = 0;
        fence_barrier_init();
        fence_proxy_async();
    }
    if (warp == 8 && lane == 0) prefetch_tmap(&qkv_map);
    if (warp == 9) {
        tmem_alloc(&bar->tmem, TMEM_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = bar->tmem;
    griddep_launch();
    griddep_wait();  // qkv comes from the preceding projection

    if (warp == 8) {
        // ---------------------------------------------------------- TMA producer
        if (lane == 0) {
            int issued_phase[KV_STAGES];
            for (int s = 0; s < KV_STAGES; s++) issued_phase[s] = -1;
            mbar_arrive_expect_tx(&bar->q_full, nq * TILE_BYTES);
            for (int q = 0; q < nq; q++)
                tma_load_2d(smem + SMEM_Q + q * TILE_BYTES, &qkv_map, &bar->q_full, h * HD, start + q0 + q * TQ);
            for (int j = 0; j < nkt && !*abort_flag; j++) {
                const int s = j % KV_STAGES;
                const uint32_t ph = (j / KV_STAGES) & 1;
                if (!mbar_wait(&bar->kv_empty[s], ph ^ 1, err, abort_flag)) break;
                mbar_arrive_expect_tx(&bar->kv_full[s], 2 * TILE_BYTES);
                tma_load_2d(smem + SMEM_K + s * TILE_BYTES, &qkv_map, &bar->kv_full[s], D + h * HD, start + j * TK);
                tma_load_2d(smem + SMEM_V + s * TILE_BYTES, &qkv_map, &bar->kv_full[s], 2 * D + h * HD,
                            start + j * TK);
                issued_phase[s] = (int)ph;
            }
            // every load issued lands before shared memory goes away
            drain_wait(&bar->q_full, 0, err);
            for (int s = 0; s < KV_STAGES; s++)
                if (issued_phase[s] >= 0) drain_wait(&bar->kv_full[s], (uint32_t)issued_phase[s], err);
        }
        __syncwarp();
    } else if (warp == 9) {
        // ---------------------------------------------------------- MMA issuer
        if (lane == 0) {
            constexpr bool BF = std::is_same<T, __nv_bfloat16>::value;
            const uint32_t idesc_s = BF ? IDESC_S_BF16 : IDESC_S_F16;
            const uint32_t idesc_o = BF ? IDESC_O_BF16 : IDESC_O_F16;
            const uint32_t sq = smem_u32(smem + SMEM_Q), sk = smem_u32(smem + SMEM_K), sv = smem_u32(smem + SMEM_V);
            auto issue_s = [&](int q, int j) {
                const int s = j % KV_STAGES;
#pragma unroll
                for (int ks = 0; ks < HD / 16; ks++)
                    tc_mma_f16(tmem + q * TK, sw128_desc(sq + q * TILE_BYTES) + 2 * ks,
                               sw128_desc(sk + s * TILE_BYTES) + 2 * ks, idesc_s, ks != 0);
                tc_commit(&bar->s_full[q]);
            };
            // P: two 64-key K-major atoms of 16 KB, 32 bytes per 16-key step;
            // V: MN-major, 16 keys (2 KB) per step, 8-key groups 1 KB apart
            // P_q from TMEM (16-bit pairs, 8 columns per 16 keys), V MN-major
            // from shared memory, 16 keys (2 KB) per step
            auto issue_o = [&](int q, int j) {
                const int s = j % KV_STAGES;
#pragma unroll
                for (int ks = 0; ks < TK / 16; ks++)
                    tc_mma_f16_ts(tmem + 2 * TK + q * HD, tmem + P_COL + q * (TK / 2) + ks * 8,
                                  sw128_desc(sv + s * TILE_BYTES + ks * 2048), idesc_o, (j | ks) != 0);
                tc_commit(&bar->o_full[q]);
            };
            bool ok = mbar_wait(&bar->q_full, 0, err, abort_flag);
            if (ok) ok = mbar_wait(&bar->kv_full[0], 0, err, abort_flag);
            if (ok) {
                tc_fence_after();
                for (int q = 0; q < nq; q++) issue_s(q, 0);
            }
            for (int j = 0; j < nkt && ok; j++) {
                // S_q(j+1) as soon as the softmax has copied S_q(j) out of
                // TMEM, then P_q V_j once it has written P_q(j)
                if (j + 1 < nkt) {
                    ok = mbar_wait(&bar->kv_full[(j + 1) % KV_STAGES], ((j + 1) / KV_STAGES) & 1, err, abort_flag);
                    for (int q = 0; q < nq && ok; q++) {
                        ok = mbar_wait(&bar->s_free[q], j & 1, err, abort_flag);
                        if (ok) {
                            tc_fence_after();
                            issue_s(q, j + 1);
                        }
                    }
                }
                for (int q = 0; q < nq && ok; q++) {
                    ok = mbar_wait(&bar->p_full[q], j & 1, err, abort_flag);
                    if (ok) {
                        tc_fence_after();
                        issue_o(q, j);
                    }
                }
                if (ok) tc_commit(&bar->kv_empty[j % KV_STAGES]);
            }
            // every MMA issued completes before TMEM and shared memory go away
            tc_commit(&bar->drain);
            drain_wait(&bar->drain, 0, err);
        }
        __syncwarp();
    } else {
        // ---------------------------------------------------------- softmax
        const int q = warp >> 2;                 // query tile of this warpgroup
        const int quarter = warp & 3;            // TMEM lanes this warp may read
        const int row = quarter * 32 + lane;     // query row in the tile
        const int qi = q0 + q * TQ + row;        // query row in the sequence
        const uint32_t t_s = tmem + ((uint32_t)(quarter * 32) << 16) + q * TK;
        const uint32_t t_o = tmem + ((uint32_t)(quarter * 32) << 16) + 2 * TK + q * HD;
        const float sl2 = 0.125f * 1.4426950408889634f;  // 1/sqrt(64) * log2(e)
        constexpr float RESCALE = 8.0f;                  // exponent growth that moves the reference point
        float m = -INFINITY, l = 0.f;
        bool ok = q < nq;
        // Both warpgroups run every tile's token_wait / token_pass, also
        // after a failed wait (ok false) or without a query tile (q >= nq),
        // so neither is ever left waiting for the other.
        for (int j = 0; j < nkt; j++) {
            float sv[TK];
            float u = 0.f, alpha = 1.0f;
            bool rescale = false;
            if (ok) ok = __all_sync(0xffffffffu, mbar_wait(&bar->s_full[q], j & 1, err, abort_flag));
            if (ok) {
                tc_fence_after();
#pragma unroll
                for (int c = 0; c < TK; c += 32) tmem_ld32(t_s + c, *reinterpret_cast<uint32_t(*)[32]>(&sv[c]));
                tc_wait_ld();
                tc_fence_before();
                mbar_arrive(&bar->s_free[q]);  // S_q may be overwritten by the next tile's MMA
                const int kend = L - j * TK;   // keys of this tile inside the sequence (>= 1)
                if (kend < TK) {               // only the sequence's last tile is masked
#pragma unroll
                    for (int i = 0; i < TK; i++)
                        if (i >= kend) sv[i] = -INFINITY;
                }
                float t[8];
#pragma unroll
                for (int i = 0; i < 8; i++) t[i] = fmaxf(sv[i], sv[i + 8]);
#pragma unroll
                for (int i = 16; i < TK; i += 8)
#pragma unroll
                    for (int k = 0; k < 8; k++) t[k] = fmaxf(t[k], sv[i + k]);
                const float mx =
                    fmaxf(fmaxf(fmaxf(t[0], t[1]), fmaxf(t[2], t[3])), fmaxf(fmaxf(t[4], t[5]), fmaxf(t[6], t[7])));
                // move the reference point when the maximum grew by more than
                // RESCALE in the exponent (always on the first tile); the warp
                // rescales its rows of O together (TMEM access is per warp),
                // after P is written
                const bool need = (mx - m) * sl2 > RESCALE;
                if (j == 0) {
                    m = mx;
                } else if (need) {
                    alpha = ex2f((m - mx) * sl2);
                    m = mx;
                    l *= alpha;
                }
                rescale = j > 0 && __any_sync(0xffffffffu, need);
                u = m * sl2;
            }
            if (q == 1 || j > 0) token_wait(q);  // group 0 starts with the token
            if (ok && j > 0) {
                // P_q and O_q are free once P_q(j-1) V has completed (this is
                // also what keeps p_full from running two phases ahead)
                ok = __all_sync(0xffffffffu, mbar_wait(&bar->o_full[q], (j - 1) & 1, err, abort_flag));
                if (ok) tc_fence_after();
            }
            if (ok) {
                // p, rounded to 16 bits in pairs, into P_q's 64 TMEM columns
                // (column c: keys 2c and 2c + 1), with the row sum in f32
                const uint32_t t_p = tmem + ((uint32_t)(quarter * 32) << 16) + P_COL + q * (TK / 2);
                float ps[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
                for (int c4 = 0; c4 < 4; c4++) {
                    uint32_t pk[16];
#pragma unroll
                    for (int i = 0; i < 16; i++) {
                        const float a = ex2f(fmaf(sv[32 * c4 + 2 * i], sl2, -u));
                        const float b = ex2f(fmaf(sv[32 * c4 + 2 * i + 1], sl2, -u));
                        ps[(2 * i) & 7] += a;
                        ps[(2 * i + 1) & 7] += b;
                        pk[i] = pack_p<T>(a, b);
                    }
                    tmem_st16(t_p + 16 * c4, pk);
                }
                l += ((ps[0] + ps[1]) + (ps[2] + ps[3])) + ((ps[4] + ps[5]) + (ps[6] + ps[7]));
                if (rescale) {
#pragma unroll
                    for (int c = 0; c < HD; c += 32) {
                        uint32_t r[32];
                        tmem_ld32(t_o + c, r);
                        tc_wait_ld();
#pragma unroll
                        for (int i = 0; i < 32; i++) r[i] = __float_as_uint(__uint_as_float(r[i]) * alpha);
                        tmem_st32(t_o + c, r);
                    }
                }
                tc_wait_st();
                tc_fence_before();
                mbar_arrive(&bar->p_full[q]);
            }
            token_pass(q);
        }
        if (q == 0) token_wait(0);  // takes group 1's last token_pass
        if (ok) {
            // O_q is complete once the last P V has
            ok = __all_sync(0xffffffffu, mbar_wait(&bar->o_full[q], (nkt - 1) & 1, err, abort_flag));
            if (ok) {
                tc_fence_after();
                float o[HD];
#pragma unroll
                for (int c = 0; c < HD; c += 32) tmem_ld32(t_o + c, *reinterpret_cast<uint32_t(*)[32]>(&o[c]));
                tc_wait_ld();
                if (qi < L) {
                    const float inv = 1.0f / l;
                    uint4* dst = reinterpret_cast<uint4*>(out + (size_t)(start + qi) * D + h * HD);
#pragma unroll
                    for (int c = 0; c < HD / 8; c++) {
                        uint4 v;
                        v.x = pack16<T>(o[8 * c + 0] * inv, o[8 * c + 1] * inv);
                        v.y = pack16<T>(o[8 * c + 2] * inv, o[8 * c + 3] * inv);
                        v.z = pack16<T>(o[8 * c + 4] * inv, o[8 * c + 5] * inv);
                        v.w = pack16<T>(o[8 * c + 6] * inv, o[8 * c + 7] * inv);
                        dst[c] = v;
                    }
                }
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 9) tmem_dealloc(tmem, TMEM_COLS);
}

}  // namespace

cudaError_t launch_attention_tc(bool bf16, const CUtensorMap& qkv_map, void* out, const int* cu_seqlens, int n_seqs,
                                int M, int max_len, int min_len, int* err, cudaStream_t stream) {
    if (n_seqs <= 0 || max_len < min_len) return cudaSuccess;
    dim3 grid((max_len + NQT * TQ - 1) / (NQT * TQ), H, n_seqs);
    if (bf16)
        return launch_k(attention_tc_kernel<__nv_bfloat16>, grid, TC_THREADS, SMEM_TC, stream, qkv_map,
                        static_cast<__nv_bfloat16*>(out), cu_seqlens, M, max_len, min_len, err);
    return launch_k(attention_tc_kernel<__half>, grid, TC_THREADS, SMEM_TC, stream, qkv_map,
                    static_cast<__half*>(out), cu_seqlens, M, max_len, min_len, err);
}

cudaError_t attention_tc_prepare() {
    cudaError_t e = cudaFuncSetAttribute(attention_tc_kernel<__nv_bfloat16>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_TC);
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(attention_tc_kernel<__half>, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_TC);
    return e;
}

}  // namespace laya
