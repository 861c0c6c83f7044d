// kernels.cuh -- launchers for the row-wise kernels (norm.cu, tail.cu, convert.cu).
#pragma once
#include "common.cuh"

namespace laya {

// norm.cu ------------------------------------------------------------------
// rope: the [MAX_POS][32] (cos, sin) table; rope_tok: [16][rope_ld] float4,
// row i of token t = (cos, sin) of frequencies 2i and 2i+1 at t's position.
cudaError_t launch_embed(bool bf16, const uint32_t* ids, const int* cu, int n_seqs, int M, const void* emb,
                         const float* w, float* x, void* xn, const float2* rope, float4* rope_tok, int rope_ld,
                         int* seq_of, int* err, cudaStream_t s);
cudaError_t launch_ln(bool bf16, const float* x, void* xn, const float* w, const float* b, int M, int num_sms,
                      cudaStream_t s);
// pre_temb (nullable): [M][768] f32, receives LN_final(x) before the type
// embedding is added (the reference's "final" --dumpstats point).
cudaError_t launch_final(bool bf16, float* x, void* xn, const float* wf, const float* type_emb,
                         const uint32_t* qtypes, const int* seq_of, const float* w1, const float* b1, int M,
                         float* pre_temb, int* err, cudaStream_t s);

// out5 = {x[0], x[1], x[2], sum, absolute sum} of n f32 values, in f64
// (the reference's --dumpstats fingerprint, src/main.zig:113-121).
cudaError_t launch_dump_stats(const float* x, size_t n, double* out5, cudaStream_t s);

// tail.cu ------------------------------------------------------------------
struct TailWeights {
    const float *s0w, *s0b, *s1w, *s1b, *s3w, *s3b;  // scorer: LN, 768x768 + b, 1x768 + b
    const float *a0t, *a0b, *a2w, *a2b;              // act head: 772x256 (act_head.0.weight transposed) + b, 2x256 + b
};
constexpr int SCORER_GROUPS = D / 64;  // partial sums per marker, one per 64 scorer outputs
constexpr int MAX_MARKERS_PER_SEQ = 1024;

// mv: [G][768] scratch, partial: [G][SCORER_GROUPS] scratch. x has M rows;
// M < 0 takes cu_seqlens[n_seqs] as the row count. The offset tables are
// checked on the device: a marker outside its sequence, a sequence's marker
// run outside [0, G) or longer than MAX_MARKERS_PER_SEQ, or a [CLS] row
// outside [0, M) sets ERR_BAD_INDEX and is skipped (its outputs zeroed or
// left unwritten), so nothing outside the buffers is read or written.
cudaError_t launch_tail(const float* x, const int* cu_seqlens, const uint32_t* markers, const int* cu_markers,
                        int n_seqs, int G, int M, const TailWeights& w, float* mv, float* partial, float* logits,
                        float* act, float* pooled, int* err, cudaStream_t s);

// convert.cu ---------------------------------------------------------------
// dst[r][c] (16-bit, bf16 or f16) <- src (F32 / F16 / BF16 tag) row perm(r);
// glu_perm interleaves a [2*half][cols] gate|up matrix into tiles of
// `tile` rows: tile/2 gate rows followed by the matching tile/2 up rows.
cudaError_t launch_convert16(void* dst, bool dst_bf16, const void* src, int src_dtype, size_t rows, size_t cols,
                             int glu_tile, cudaStream_t s);
cudaError_t launch_convert_f32(float* dst, const void* src, int src_dtype, size_t n, cudaStream_t s);
// dst[cols][rows] = src[rows][cols]^T, f32.
cudaError_t launch_transpose_f32(float* dst, const float* src, int rows, int cols, cudaStream_t s);

}  // namespace laya
