// gemm.cu -- persistent tcgen05 GEMM for the projection layers.
//
// One CTA per SM, 320 threads, warp-specialised:
//   warp 0      TMA producer: A tile [128 x 128] and B tile [BN x 128] per
//               k-block, each as two 64-column boxes (128B swizzle), into a
//               STAGES-deep shared-memory ring.
//   warp 1      allocates TMEM; one thread issues tcgen05.mma (M=128, N=BN,
//               K=16) into a double-buffered f32 accumulator in TMEM and
//               commits to mbarriers (ring slot free / accumulator full).
//   warps 2..9  epilogue, two warps per TMEM lane quarter (each warp may only
//               read the 32 lanes = tile rows its warp id selects), one per
//               half of the tile's columns: tcgen05.ld of the accumulator,
//               the fused elementwise op, a swizzled 32 x 128-byte tile in
//               shared memory, and a TMA store of it (the residual stream: a
//               TMA reduce-add, so the f32 stream is never read by the SM).
// The accumulator is double-buffered, so the epilogue of tile i overlaps the
// MMAs of tile i+1. Every wait is bounded (common.cuh); a CTA that gives up
// records the error, drains its own TMA loads and MMAs, frees TMEM and exits.
//
// Numerics: inputs are 16-bit, products are exact in f32 and accumulate in
// f32, as the reference's f32 FMA chains over f16-widened weights do
// (src/main.zig:934-974); only the rounding of the activations to 16 bits
// and the summation order differ.
#include <cstdio>

#include "gemm.cuh"

namespace laya {

namespace {

constexpr int BM = 128;
constexpr int BK = 128;    // K per pipeline stage
constexpr int KSUB = 64;   // K per 128-byte-swizzled sub-tile (one TMA box wide)
constexpr int EPI_WARPS = 8;
constexpr int NUM_THREADS = 64 + 32 * EPI_WARPS;
constexpr int STAGING_BYTES = 32 * 128;  // one 32-row x 128-byte output tile
// Staging tiles per epilogue warp. One: with 64 KB operand stages (K = 128
// per stage) a second tile per warp would leave room for only two stages,
// and three stages with one tile measured faster (GLU 35.3 vs 37.2 us).
template <int EPI>
constexpr int staging_bufs() {
    return 1;
}
constexpr int SMEM_LIMIT = 227 * 1024;

template <int BN, int EPI, bool PAIR = false>
struct Cfg {
    static constexpr int STAGING_BUFS = staging_bufs<EPI>();
    static constexpr int B_ROWS = PAIR ? BN / 2 : BN;  // B rows this CTA loads per tile
    static constexpr int A_BYTES = BM * BK * 2;
    static constexpr int B_BYTES = B_ROWS * BK * 2;
    static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
    static constexpr int FIXED = EPI_WARPS * STAGING_BUFS * STAGING_BYTES + 1024 /*align*/ + 256 /*barriers*/;
    static constexpr int FIT = (SMEM_LIMIT - FIXED) / STAGE_BYTES;
    static constexpr int STAGES = FIT < 6 ? FIT : 6;
    static constexpr int RING = STAGES * STAGE_BYTES;
    static constexpr int TMEM_COLS = 2 * BN;  // two accumulators of BN f32 columns
    static constexpr int SMEM = RING + FIXED;
    static_assert(STAGES >= 3, "operand ring too shallow");
};

template <typename T>
struct Pack;
template <>
struct Pack<__nv_bfloat16> {
    static __device__ __forceinline__ uint32_t two(float a, float b) {
        __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
        return *reinterpret_cast<uint32_t*>(&h);
    }
};
template <>
struct Pack<__half> {
    static __device__ __forceinline__ uint32_t two(float a, float b) {
        __half2 h = __floats2half2_rn(a, b);
        return *reinterpret_cast<uint32_t*>(&h);
    }
};

// 32 consecutive f32 columns of this thread's row.
__device__ __forceinline__ void load_cols(uint32_t taddr, float (&v)[32]) {
    uint32_t r[32];
    tmem_ld32(taddr, r);
    tc_wait_ld();
#pragma unroll
    for (int i = 0; i < 32; i++) v[i] = __uint_as_float(r[i]);
}

// Two 16-column groups of this thread's row, one wait for both.
__device__ __forceinline__ void load_cols16x2(uint32_t taddr0, uint32_t taddr1, float (&v0)[16], float (&v1)[16]) {
    uint32_t r0[16], r1[16];
    tmem_ld16(taddr0, r0);
    tmem_ld16(taddr1, r1);
    tc_wait_ld();
#pragma unroll
    for (int i = 0; i < 16; i++) {
        v0[i] = __uint_as_float(r0[i]);
        v1[i] = __uint_as_float(r1[i]);
    }
}

template <int NV>
__device__ __forceinline__ void add_bias(float (&v)[NV], const float* bias, int col) {
    if (bias) {
        const float4* b = reinterpret_cast<const float4*>(bias + col);
#pragma unroll
        for (int q = 0; q < NV / 4; q++) {
            const float4 t = __ldg(b + q);
            v[4 * q] += t.x;
            v[4 * q + 1] += t.y;
            v[4 * q + 2] += t.z;
            v[4 * q + 3] += t.w;
        }
    }
}

// Row `lane` of a 32 x 128-byte staging tile, 16-byte chunk `j`, in the
// 128-byte swizzle the output tensor map expects (chunk j of row r lands at
// chunk j ^ (r % 8)); the tile base is 1024-byte aligned.
__device__ __forceinline__ uint4* stage_chunk(uint8_t* tile, int lane, int j) {
    return reinterpret_cast<uint4*>(tile + lane * 128 + ((j ^ (lane & 7)) << 4));
}

// NV values -> 2*NV bytes of 16-bit elements at chunks [c0, c0 + NV/8).
template <typename T, int NV>
__device__ __forceinline__ void stage16(uint8_t* tile, int lane, int c0, const float (&v)[NV]) {
#pragma unroll
    for (int q = 0; q < NV / 8; q++) {
        uint4 u;
        u.x = Pack<T>::two(v[8 * q + 0], v[8 * q + 1]);
        u.y = Pack<T>::two(v[8 * q + 2], v[8 * q + 3]);
        u.z = Pack<T>::two(v[8 * q + 4], v[8 * q + 5]);
        u.w = Pack<T>::two(v[8 * q + 6], v[8 * q + 7]);
        *stage_chunk(tile, lane, c0 + q) = u;
    }
}

// 32 f32 values -> the whole 128-byte row.
__device__ __forceinline__ void stage32(uint8_t* tile, int lane, const float (&v)[32]) {
#pragma unroll
    for (int q = 0; q < 8; q++)
        *stage_chunk(tile, lane, q) =
            make_uint4(__float_as_uint(v[4 * q]), __float_as_uint(v[4 * q + 1]), __float_as_uint(v[4 * q + 2]),
                       __float_as_uint(v[4 * q + 3]));
}

// Hand the staged tile to the TMA unit: make the generic-proxy writes
// visible to the async proxy, then one lane issues the store.
template <bool REDUCE>
__device__ __forceinline__ void flush_stage(const CUtensorMap* map, uint8_t* tile, int lane, int col, int row) {
    fence_proxy_async();
    __syncwarp();
    if (lane == 0) {
        if (REDUCE) tma_reduce_add_2d(map, tile, col, row);
        else tma_store_2d(map, tile, col, row);
        bulk_commit();
    }
}

// An epilogue warp's NBUF staging tiles, used in turn: the next one to fill
// is free once the store issued NBUF tiles ago has read it (lane 0 issues
// and commits every store, so its bulk groups are the warp's).
template <int NBUF>
struct Staging {
    uint8_t* base;
    int n;  // tiles handed out so far
    __device__ __forceinline__ uint8_t* next(int lane) {
        if (lane == 0) bulk_wait_read<NBUF - 1>();
        __syncwarp();
        return base + (n++ % NBUF) * STAGING_BYTES;
    }
};

// EPI_QKV: (cos, sin) of row m0q + lane's position for the 32 frequencies,
// from the frequency-major per-token rows: for each i the warp's 32
// consecutive rows are 512 contiguous bytes. Rows past M are computed but
// their stores are clipped; they read row 0.
__device__ __forceinline__ void rope_load(const GemmArgs& a, int m0q, int lane, float4 (&cs)[16]) {
    const int r = m0q + lane;
    const float4* src = a.rope_tok + (r < a.M ? r : 0);
#pragma unroll
    for (int i = 0; i < 16; i++) cs[i] = __ldg(src + (size_t)i * a.rope_ld);
}

// cs: EPI_QKV's rope_load of this warp's rows (unused otherwise).
template <int BN, int EPI, typename T>
__device__ __forceinline__ void epilogue_tile(const GemmArgs& a, const CUtensorMap* out_map,
                                              Staging<staging_bufs<EPI>()>& st,
                                              uint32_t tacc, int half, int lane, int m0q, int n_blk,
                                              const float4 (&cs)[16]) {
    constexpr int HALF = BN / 2;  // accumulator columns this warp owns
    if constexpr (EPI == EPI_GLU) {
        // tile columns [0, BN/2) are gate rows, [BN/2, BN) the matching up rows;
        // this warp produces output columns [half*BN/4, (half+1)*BN/4) of the tile
        constexpr int OUT = BN / 4;
        static_assert(OUT == 64 || OUT == 32, "GLU tile");
        uint8_t* tile = nullptr;
#pragma unroll 1
        for (int c = 0; c < OUT; c += 32) {
            float g[32], u[32];
            load_cols(tacc + half * OUT + c, g);
            load_cols(tacc + HALF + half * OUT + c, u);
#pragma unroll
            for (int i = 0; i < 32; i++) g[i] = gelu_as(g[i]) * u[i];
            if (c == 0) tile = st.next(lane);
            stage16<T>(tile, lane, (c / 32) * 4, g);
        }
        flush_stage<false>(out_map, tile, lane, n_blk * HALF + half * OUT, m0q);
    } else if constexpr (EPI == EPI_QKV) {
        const int col0 = n_blk * BN + half * HALF;
        const bool rope = col0 < a.rope_cols;
#pragma unroll 1
        for (int c = 0; c < HALF; c += 64) {
            // one head (64 columns): rotate_half pairs column d with d + 32
            // (src/main.zig:2512-2519); done in two passes of 16 frequencies
            // so that only 32 accumulator values are live beside the pairs
            const int col = col0 + c;
            uint8_t* tile = st.next(lane);
#pragma unroll
            for (int hq = 0; hq < 2; hq++) {
                float x0[16], x1[16];
                load_cols16x2(tacc + half * HALF + c + 16 * hq, tacc + half * HALF + c + 32 + 16 * hq, x0, x1);
                add_bias(x0, a.bias, col + 16 * hq);
                add_bias(x1, a.bias, col + 32 + 16 * hq);
                if (rope) {
#pragma unroll
                    for (int d = 0; d < 16; d += 2) {
                        const float4 t = cs[8 * hq + d / 2];  // (cos, sin) of frequencies 16hq+d, 16hq+d+1
                        const float a0 = x0[d], b0 = x1[d], a1 = x0[d + 1], b1 = x1[d + 1];
                        x0[d] = a0 * t.x - b0 * t.y;
                        x1[d] = b0 * t.x + a0 * t.y;
                        x0[d + 1] = a1 * t.z - b1 * t.w;
                        x1[d + 1] = b1 * t.z + a1 * t.w;
                    }
                }
                stage16<T>(tile, lane, 2 * hq, x0);
                stage16<T>(tile, lane, 4 + 2 * hq, x1);
            }
            flush_stage<false>(out_map, tile, lane, col, m0q);
        }
    } else if constexpr (EPI == EPI_F32 || EPI == EPI_RESID) {
#pragma unroll 1
        for (int c = 0; c < HALF; c += 32) {
            float v[32];
            load_cols(tacc + half * HALF + c, v);
            const int col = n_blk * BN + half * HALF + c;
            add_bias(v, a.bias, col);
            uint8_t* tile = st.next(lane);
            stage32(tile, lane, v);
            flush_stage<EPI == EPI_RESID>(out_map, tile, lane, col, m0q);
        }
    } else {  // EPI_ACT16, EPI_RELU
#pragma unroll 1
        for (int c = 0; c < HALF; c += 64) {
            float x0[32], x1[32];
            load_cols(tacc + half * HALF + c, x0);
            load_cols(tacc + half * HALF + c + 32, x1);
            const int col = n_blk * BN + half * HALF + c;
            add_bias(x0, a.bias, col);
            add_bias(x1, a.bias, col + 32);
            if constexpr (EPI == EPI_RELU) {
#pragma unroll
                for (int i = 0; i < 32; i++) {
                    x0[i] = fmaxf(x0[i], 0.0f);
                    x1[i] = fmaxf(x1[i], 0.0f);
                }
            }
            uint8_t* tile = st.next(lane);
            stage16<T>(tile, lane, 0, x0);
            stage16<T>(tile, lane, 4, x1);
            flush_stage<false>(out_map, tile, lane, col, m0q);
        }
    }
}

// PAIR: a cluster of two CTAs computes a 256 x BN tile with cta_group::2
// MMAs issued by rank 0; each CTA loads its own 128 A rows and BN/2 B rows,
// holds its 128 accumulator rows in its own TMEM and runs its own epilogue.
template <int BN, int EPI, typename T, bool PAIR>
__device__ __forceinline__ void gemm_body(const CUtensorMap& a_map, const CUtensorMap& b_map,
                                          const CUtensorMap& out_map, const GemmArgs& args) {
    using C = Cfg<BN, EPI, PAIR>;
    constexpr int TILE_M = PAIR ? 2 * BM : BM;
    constexpr uint32_t IDESC = idesc_f16(TILE_M, BN, std::is_same<T, __nv_bfloat16>::value);
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* staging = smem + C::RING;
    uint64_t* full = reinterpret_cast<uint64_t*>(staging + EPI_WARPS * C::STAGING_BUFS * STAGING_BYTES);
    uint64_t* empty = full + C::STAGES;
    uint64_t* tfull = empty + C::STAGES;
    uint64_t* tempty = tfull + 2;
    uint64_t* drain = tempty + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const uint32_t rank = PAIR ? cluster_rank() : 0;
    const bool leader = rank == 0;
    const int unit = PAIR ? (blockIdx.x >> 1) : blockIdx.x;       // this CTA's (pair's) index
    const int units = PAIR ? (gridDim.x >> 1) : gridDim.x;
    const int tiles_m = (args.M + TILE_M - 1) / TILE_M;
    const int tiles_n = args.N / BN;
    const int total = tiles_m * tiles_n;
    const int nk = args.K / BK;

    if (threadIdx.x == 0) {
        for (int s = 0; s < C::STAGES; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < 2; b++) {
            mbar_init(&tfull[b], 1);
            mbar_init(&tempty[b], PAIR ? 2 * EPI_WARPS : EPI_WARPS);
        }
        mbar_init(drain, 1);
        *abort_flag = 0;
        fence_barrier_init();
        fence_proxy_async();
    }
    if (warp == 0 && lane == 0) {
        prefetch_tmap(&a_map);
        prefetch_tmap(&b_map);
        prefetch_tmap(&out_map);
    }
    if (warp == 1) {
        if constexpr (PAIR) {
            tmem_alloc_pair(tmem_slot, C::TMEM_COLS);
            tmem_relinquish_pair();
        } else {
            tmem_alloc(tmem_slot, C::TMEM_COLS);
            tmem_relinquish();
        }
    }
    tc_fence_before();
    if constexpr (PAIR) cluster_sync();  // the peer's barriers exist before anyone signals them
    else __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    // When every CTA (pair) has at most one tile (small M: a few SMs stream
    // each projection's weights), the producer asks for its tile's B boxes
    // in L2 now, so their HBM latency overlaps the previous kernel's tail
    // (single decisions 2.6-3% faster). This is only a hint: L2 is
    // coherent, so a B that the previous kernel still writes is read
    // correctly after the wait. With more tiles than CTAs the
    // prefetched boxes only displace live activations from L2 (0.8% slower
    // on a 64 x 180 batch), so there is none.
    if (warp == 0 && lane == 0 && unit < total && total <= units) {
        const int n0 = (unit % tiles_n) * BN + (int)rank * C::B_ROWS;
        for (int kb = 0; kb < nk; kb++)
            for (int j = 0; j < BK / KSUB; j++) tma_prefetch_l2_2d(&b_map, kb * BK + j * KSUB, n0);
    }
    // The first ring stages' weight boxes are requested now as well when
    // no kernel writes B (the context's weights; a caller's matrix may
    // come from the kernel just before): their HBM latency overlaps the
    // previous kernel's tail, and after the dependency wait only the
    // activations (A) of those stages remain to load. The stages are
    // fresh, so no empty-barrier wait is needed; each stage's full barrier
    // is armed for its A and B bytes together.
    const int pre =
        (warp == 0 && lane == 0 && unit < total && args.b_const) ? (nk < C::STAGES ? nk : C::STAGES) : 0;
    if (pre) {
        const int n0 = (unit % tiles_n) * BN + (int)rank * C::B_ROWS;
        for (int kb = 0; kb < pre; kb++) {
            uint8_t* sa = smem + kb * C::STAGE_BYTES;
            if constexpr (PAIR) {
                const uint32_t bar = mapa_shared(smem_u32(&full[kb]), 0);
                if (leader) mbar_arrive_expect_tx(&full[kb], 2 * C::STAGE_BYTES);
                for (int j = 0; j < BK / KSUB; j++)
                    tma_load_2d_pair(sa + C::A_BYTES + j * C::B_ROWS * KSUB * 2, &b_map, bar, kb * BK + j * KSUB, n0);
            } else {
                mbar_arrive_expect_tx(&full[kb], C::STAGE_BYTES);
                for (int j = 0; j < BK / KSUB; j++)
                    tma_load_2d(sa + C::A_BYTES + j * C::B_ROWS * KSUB * 2, &b_map, &full[kb], kb * BK + j * KSUB, n0);
            }
        }
    }
    // Set-up above overlaps the previous kernel's tail; activations and
    // outputs are touched only after it has completed.
    griddep_launch();
    griddep_wait();

    if (warp == 0) {
        if (lane == 0) {
            int stage = 0;
            uint32_t phase = 0;
            int issued_phase[C::STAGES];
            for (int s = 0; s < C::STAGES; s++) issued_phase[s] = -1;
            // the A boxes of the stages whose B boxes were requested above,
            // unconditionally, so every armed stage completes
            if (pre) {
                const int m0 = (unit / tiles_n) * TILE_M + (int)rank * BM;
                for (int kb = 0; kb < pre; kb++) {
                    uint8_t* sa = smem + kb * C::STAGE_BYTES;
                    if constexpr (PAIR) {
                        const uint32_t bar = mapa_shared(smem_u32(&full[kb]), 0);
                        for (int j = 0; j < BK / KSUB; j++)
                            tma_load_2d_pair(sa + j * BM * KSUB * 2, &a_map, bar, kb * BK + j * KSUB, m0);
                    } else {
                        for (int j = 0; j < BK / KSUB; j++)
                            tma_load_2d(sa + j * BM * KSUB * 2, &a_map, &full[kb], kb * BK + j * KSUB, m0);
                    }
                    issued_phase[kb] = 0;
                }
                stage = pre % C::STAGES;
                phase = pre == C::STAGES ? 1u : 0u;
            }
            for (int t = unit; t < total && !*abort_flag; t += units) {
                const int m0 = (t / tiles_n) * TILE_M + (int)rank * BM;
                const int n0 = (t % tiles_n) * BN + (int)rank * C::B_ROWS;
                for (int kb = t == unit ? pre : 0; kb < nk; kb++) {
                    if (!mbar_wait(&empty[stage], phase ^ 1, args.err, abort_flag)) goto producer_done;
                    uint8_t* sa = smem + stage * C::STAGE_BYTES;
                    if constexpr (PAIR) {
                        // both CTAs' bytes complete on rank 0's barrier; only rank 0 arms it
                        const uint32_t bar = mapa_shared(smem_u32(&full[stage]), 0);
                        if (leader) mbar_arrive_expect_tx(&full[stage], 2 * C::STAGE_BYTES);
                        for (int j = 0; j < BK / KSUB; j++) {
                            tma_load_2d_pair(sa + j * BM * KSUB * 2, &a_map, bar, kb * BK + j * KSUB, m0);
                            tma_load_2d_pair(sa + C::A_BYTES + j * C::B_ROWS * KSUB * 2, &b_map, bar,
                                             kb * BK + j * KSUB, n0);
                        }
                    } else {
                        mbar_arrive_expect_tx(&full[stage], C::STAGE_BYTES);
                        for (int j = 0; j < BK / KSUB; j++) {
                            tma_load_2d(sa + j * BM * KSUB * 2, &a_map, &full[stage], kb * BK + j * KSUB, m0);
                            tma_load_2d(sa + C::A_BYTES + j * C::B_ROWS * KSUB * 2, &b_map, &full[stage],
                                        kb * BK + j * KSUB, n0);
                        }
                    }
                    issued_phase[stage] = (int)phase;
                    if (++stage == C::STAGES) {
                        stage = 0;
                        phase ^= 1;
                    }
                }
            }
        producer_done:
            // Let every load this thread issued land before shared memory goes
            // away. In a pair the completions are counted on rank 0's barrier;
            // this CTA's empty barrier flips only after rank 0 consumed them.
            for (int s = 0; s < C::STAGES; s++) {
                if (issued_phase[s] < 0) continue;
                uint64_t* bar = PAIR ? &empty[s] : &full[s];
                const unsigned long long t0 = globaltimer();
                while (!mbar_try_wait(bar, (uint32_t)issued_phase[s])) {
                    if (globaltimer() - t0 > WAIT_LIMIT_NS) {
                        atomicOr(args.err, ERR_WAIT_TIMEOUT);
                        break;
                    }
                }
            }
        }
        __syncwarp();
    } else if (warp == 1) {
        if (lane == 0 && leader) {
            int stage = 0;
            uint32_t phase = 0;
            int it = 0;
            for (int t = unit; t < total; t += units, it++) {
                const int buf = it & 1;
                const uint32_t tph = (it >> 1) & 1;
                if (!mbar_wait(&tempty[buf], tph ^ 1, args.err, abort_flag)) break;
                tc_fence_after();
                const uint32_t d = tmem_base + buf * BN;
                bool ok = true;
                for (int kb = 0; kb < nk; kb++) {
                    if (!mbar_wait(&full[stage], phase, args.err, abort_flag)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t sa = smem_u32(smem + stage * C::STAGE_BYTES);
#pragma unroll
                    for (int k = 0; k < BK / 16; k++) {
                        // sub-tile k / 4 of the stage, 16-column step k % 4 inside it (32 B = 2 in the descriptor)
                        const int j = k / (KSUB / 16), ks = k % (KSUB / 16);
                        const uint64_t adesc = sw128_desc(sa + j * BM * KSUB * 2) + 2 * ks;
                        const uint64_t bdesc = sw128_desc(sa + C::A_BYTES + j * C::B_ROWS * KSUB * 2) + 2 * ks;
                        if constexpr (PAIR) tc_mma_f16_pair(d, adesc, bdesc, IDESC, (kb | k) != 0);
                        else tc_mma_f16(d, adesc, bdesc, IDESC, (kb | k) != 0);
                    }
                    if constexpr (PAIR) tc_commit_pair(&empty[stage], 0x3);
                    else tc_commit(&empty[stage]);
                    if (++stage == C::STAGES) {
                        stage = 0;
                        phase ^= 1;
                    }
                }
                if (!ok) break;
                if constexpr (PAIR) tc_commit_pair(&tfull[buf], 0x3);
                else tc_commit(&tfull[buf]);
            }
            // All MMAs this thread issued are complete once `drain` flips.
            if constexpr (PAIR) tc_commit_pair(drain, 0x1);
            else tc_commit(drain);
            const unsigned long long t0 = globaltimer();
            while (!mbar_try_wait(drain, 0)) {
                if (globaltimer() - t0 > WAIT_LIMIT_NS) {
                    atomicOr(args.err, ERR_WAIT_TIMEOUT);
                    break;
                }
            }
        }
        __syncwarp();
    } else {
        const int e = warp - 2;
        const int q = warp & 3;          // TMEM lane quarter this warp may access
        const int half = e >> 2;         // which half of the tile's columns
        Staging<C::STAGING_BUFS> st{staging + e * C::STAGING_BUFS * STAGING_BYTES, 0};
        const uint32_t tempty_leader = PAIR ? mapa_shared(smem_u32(tempty), 0) : 0;
        int it = 0;
        for (int t = unit; t < total; t += units, it++) {
            const int buf = it & 1;
            const uint32_t tph = (it >> 1) & 1;
            const int m0q = (t / tiles_n) * TILE_M + (int)rank * BM + q * 32;
            // the RoPE pairs are requested before the accumulator wait, so
            // their latency overlaps the tile's MMAs
            float4 cs[16];
            if constexpr (EPI == EPI_QKV) {
                if ((t % tiles_n) * BN + half * (BN / 2) < args.rope_cols) rope_load(args, m0q, lane, cs);
            }
            int ok = 1;
            if (lane == 0) ok = mbar_wait(&tfull[buf], tph, args.err, abort_flag);
            ok = __shfl_sync(0xffffffffu, ok, 0);
            if (!ok) break;
            tc_fence_after();
            const uint32_t tacc = tmem_base + ((uint32_t)(q * 32) << 16) + buf * BN;
            epilogue_tile<BN, EPI, T>(args, &out_map, st, tacc, half, lane, m0q, t % tiles_n, cs);
            tc_fence_before();
            __syncwarp();
            if (lane == 0) {
                if constexpr (PAIR) mbar_arrive_cluster(tempty_leader + buf * 8);
                else mbar_arrive(&tempty[buf]);
            }
        }
        // Shared memory must outlive the stores' reads of it, nothing more:
        // the global writes (stores, L2 reduce-adds) are performed and
        // visible to the next kernel once this grid completes, so teardown
        // overlaps their draining (0.3-0.5 us per launch).
        if (lane == 0) bulk_wait_read_all();
        __syncwarp();
    }

    tc_fence_before();
    if constexpr (PAIR) cluster_sync();  // neither CTA frees TMEM while the pair may still use it
    else __syncthreads();
    tc_fence_after();
    if (warp == 1) {
        if constexpr (PAIR) tmem_dealloc_pair(tmem_base, C::TMEM_COLS);
        else tmem_dealloc(tmem_base, C::TMEM_COLS);
    }
}

template <int BN, int EPI, typename T>
__global__ void __launch_bounds__(NUM_THREADS, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap a_map, const __grid_constant__ CUtensorMap b_map,
                const __grid_constant__ CUtensorMap out_map, GemmArgs args) {
    gemm_body<BN, EPI, T, false>(a_map, b_map, out_map, args);
}

template <int EPI, typename T>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(NUM_THREADS, 1)
    gemm_pair_kernel(const __grid_constant__ CUtensorMap a_map, const __grid_constant__ CUtensorMap b_map,
                     const __grid_constant__ CUtensorMap out_map, GemmArgs args) {
    gemm_body<256, EPI, T, true>(a_map, b_map, out_map, args);
}

template <int BN, int EPI, typename T>
cudaError_t prepare_one() {
    if constexpr (BN == 256)
        return cudaFuncSetAttribute(gemm_pair_kernel<EPI, T>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    Cfg<256, EPI, true>::SMEM);
    else
        return cudaFuncSetAttribute(gemm_kernel<BN, EPI, T>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    Cfg<BN, EPI>::SMEM);
}

template <int BN, typename T>
cudaError_t prepare_bn() {
    cudaError_t e = cudaSuccess;
    if (e == cudaSuccess) e = prepare_one<BN, EPI_F32, T>();
    if (e == cudaSuccess) e = prepare_one<BN, EPI_ACT16, T>();
    if (e == cudaSuccess) e = prepare_one<BN, EPI_QKV, T>();
    if (e == cudaSuccess) e = prepare_one<BN, EPI_RESID, T>();
    if (e == cudaSuccess) e = prepare_one<BN, EPI_GLU, T>();
    if (e == cudaSuccess) e = prepare_one<BN, EPI_RELU, T>();
    return e;
}

// BN = 256: CTA pairs (cluster of 2, 256 x 256 tiles); BN = 128: single CTAs.
template <int BN, int EPI, typename T>
cudaError_t launch_one(const CUtensorMap& a_map, const CUtensorMap& b_map, const CUtensorMap& out_map,
                       const GemmArgs& args, int num_sms, cudaStream_t stream) {
    if constexpr (BN == 256) {
        using C = Cfg<256, EPI, true>;
        const int tiles = ((args.M + 2 * BM - 1) / (2 * BM)) * (args.N / BN);
        const int pairs = tiles < num_sms / 2 ? tiles : num_sms / 2;
        if (pairs <= 0) return cudaSuccess;
        return launch_k(gemm_pair_kernel<EPI, T>, 2 * pairs, NUM_THREADS, C::SMEM, stream, a_map, b_map, out_map,
                        args);
    } else {
        using C = Cfg<BN, EPI>;
        const int tiles = ((args.M + BM - 1) / BM) * (args.N / BN);
        const int grid = tiles < num_sms ? tiles : num_sms;
        if (grid <= 0) return cudaSuccess;
        return launch_k(gemm_kernel<BN, EPI, T>, grid, NUM_THREADS, C::SMEM, stream, a_map, b_map, out_map, args);
    }
}

template <int BN, typename T>
cudaError_t dispatch_epi(int epi, const CUtensorMap& a, const CUtensorMap& b, const CUtensorMap& o,
                         const GemmArgs& args, int sms, cudaStream_t s) {
    switch (epi) {
        case EPI_F32: return launch_one<BN, EPI_F32, T>(a, b, o, args, sms, s);
        case EPI_ACT16: return launch_one<BN, EPI_ACT16, T>(a, b, o, args, sms, s);
        case EPI_QKV: return launch_one<BN, EPI_QKV, T>(a, b, o, args, sms, s);
        case EPI_RESID: return launch_one<BN, EPI_RESID, T>(a, b, o, args, sms, s);
        case EPI_GLU: return launch_one<BN, EPI_GLU, T>(a, b, o, args, sms, s);
        case EPI_RELU: return launch_one<BN, EPI_RELU, T>(a, b, o, args, sms, s);
    }
    return cudaErrorInvalidValue;
}

using EncodeFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                              const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                              CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeFn encoder() {
    static EncodeFn encode = nullptr;
    if (!encode) {
        void* fn = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess || !fn)
            return nullptr;
        encode = reinterpret_cast<EncodeFn>(fn);
    }
    return encode;
}

}  // namespace

CUresult make_tmap_2d(CUtensorMap* map, const void* base, uint64_t inner, uint64_t rows, uint32_t box_rows,
                      bool bf16) {
    EncodeFn encode = encoder();
    if (!encode) return CUDA_ERROR_NOT_FOUND;
    const cuuint64_t dims[2] = {inner, rows};
    const cuuint64_t strides[1] = {inner * 2};
    const cuuint32_t box[2] = {64, box_rows};
    const cuuint32_t estr[2] = {1, 1};
    return encode(map, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2,
                  const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
}

CUresult make_out_map(CUtensorMap* map, void* base, uint64_t inner, uint64_t rows, int elem_bytes, bool bf16) {
    EncodeFn encode = encoder();
    if (!encode) return CUDA_ERROR_NOT_FOUND;
    const cuuint64_t dims[2] = {inner, rows};
    const cuuint64_t strides[1] = {inner * (uint64_t)elem_bytes};
    const cuuint32_t box[2] = {(cuuint32_t)(128 / elem_bytes), 32};
    const cuuint32_t estr[2] = {1, 1};
    const CUtensorMapDataType dt = elem_bytes == 4 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                                   : bf16          ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                   : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    return encode(map, dt, 2, base, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
}

cudaError_t gemm_prepare() {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    static unsigned long long done = 0;  // one bit per device
    if (dev < 64 && (done >> dev) & 1ull) return cudaSuccess;
    if (e == cudaSuccess) e = prepare_bn<256, __nv_bfloat16>();
    if (e == cudaSuccess) e = prepare_bn<256, __half>();
    if (e == cudaSuccess) e = prepare_bn<128, __nv_bfloat16>();
    if (e == cudaSuccess) e = prepare_bn<128, __half>();
    if (e == cudaSuccess && dev < 64) done |= 1ull << dev;
    return e;
}

cudaError_t launch_gemm(int epi, int bn, bool bf16, const CUtensorMap& a_map, const CUtensorMap& b_map,
                        const CUtensorMap& out_map, const GemmArgs& args, int num_sms, cudaStream_t stream) {
    if (args.K % BK || args.N % bn || args.M < 0) return cudaErrorInvalidValue;
    if ((epi == EPI_GLU || epi == EPI_QKV) && bn != 256) return cudaErrorInvalidValue;
    if (bn == 256)
        return bf16 ? dispatch_epi<256, __nv_bfloat16>(epi, a_map, b_map, out_map, args, num_sms, stream)
                    : dispatch_epi<256, __half>(epi, a_map, b_map, out_map, args, num_sms, stream);
    if (bn == 128)
        return bf16 ? dispatch_epi<128, __nv_bfloat16>(epi, a_map, b_map, out_map, args, num_sms, stream)
                    : dispatch_epi<128, __half>(epi, a_map, b_map, out_map, args, num_sms, stream);
    return cudaErrorInvalidValue;
}

}  // namespace laya
