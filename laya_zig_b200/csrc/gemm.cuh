// gemm.cuh -- tcgen05 projection GEMM with fused epilogues (declarations).
//
// out = A[M,K] * B[N,K]^T, A and B 16-bit (bf16 or f16) K-major, f32
// accumulation in TMEM. Replaces the reference's linear16/packed kernel
// (src/main.zig:844-1099) and fuses the elementwise job that follows each
// projection in `forward` (src/main.zig:2641-2754).
#pragma once
#include "common.cuh"

namespace laya {

enum Epilogue : int {
    EPI_F32 = 0,    // out_f32 = acc (+ bias)                          plain GEMM
    EPI_ACT16 = 1,  // out16 = acc (+ bias)                           plain GEMM
    EPI_QKV = 2,    // out16 = rope(acc (+ bias)) on q,k columns        splitJob+ropeJob (2626-2634, 2496-2521)
    EPI_RESID = 3,  // out_f32 += acc (+ bias)                          addResJob (2571-2578), biasJob (1073-1079)
    EPI_GLU = 4,    // out16[j] = gelu(acc[gate j]) * acc[up j]         mlpJob (2557-2569)
    EPI_RELU = 5,   // out16 = relu(acc + bias)                         reluJob (2580-2586)
};

struct GemmArgs {
    int M, N, K;
    const float* bias;      // [N] or null
    const float4* rope_tok; // EPI_QKV: [16][rope_ld], (cos, sin) of frequencies 2i, 2i+1 for row r at [i][r]
    int rope_ld;
    int rope_cols;          // EPI_QKV: RoPE applies to columns [0, rope_cols)
    int* err;               // device error word
    int b_const;            // 1: no kernel writes B (the context's weights), so its first
                            // ring stages are loaded before the dependency wait
};

// 2-D tensor map over a row-major [rows][inner] 16-bit matrix, box
// [box_rows][64] with 128-byte swizzle: the operand layout of the GEMM
// (UMMA K-major, SWIZZLE_128B).
CUresult make_tmap_2d(CUtensorMap* map, const void* base, uint64_t inner, uint64_t rows, uint32_t box_rows,
                      bool bf16);

// Output tensor map of an epilogue: [rows][inner] row-major, elements of
// `elem_bytes` (2: 16-bit of the GEMM's type, 4: f32), box of 32 rows x
// 128 bytes with 128-byte swizzle. The epilogue writes it with TMA stores
// (EPI_RESID: TMA reduce-add). Rows at or past `rows` are never written.
CUresult make_out_map(CUtensorMap* map, void* base, uint64_t inner, uint64_t rows, int elem_bytes, bool bf16);

// Raise the dynamic shared-memory limit of every GEMM instantiation on the
// current device (once per device; must not run during stream capture).
cudaError_t gemm_prepare();

// Launch one GEMM. BN (128 or 256) must divide N, 64 must divide K.
// BN = 256 runs CTA pairs (256 x 256 tiles, cta_group::2), BN = 128 single
// CTAs (128 x 128). A's and B's maps both have 128-row boxes. Returns a CUDA
// error code.
cudaError_t launch_gemm(int epi, int bn, bool bf16, const CUtensorMap& a_map, const CUtensorMap& b_map,
                        const CUtensorMap& out_map, const GemmArgs& args, int num_sms, cudaStream_t stream);

}  // namespace laya
