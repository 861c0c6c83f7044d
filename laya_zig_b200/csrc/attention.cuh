// attention.cuh -- packed-sequence attention (declarations).
#pragma once
#include "common.cuh"

namespace laya {

// qkv_map: make_tmap_2d over qkv [M][3*768] 16-bit (q | k | v, head-major)
// with 64-row boxes; out: [M][768]. cu_seqlens: [n_seqs + 1] token offsets.
// window < 0: full attention, otherwise keys with |i - j| <= window only
// (src/main.zig:2440-2444). A sequence whose offsets leave [0, M) or whose
// length exceeds max_len sets ERR_BAD_INDEX in *err and is skipped.
// long_len: sequences of at least this many tokens are skipped (the tcgen05
// kernel takes them); INT_MAX skips none.
cudaError_t launch_attention(bool bf16, const CUtensorMap& qkv_map, void* out, const int* cu_seqlens, int n_seqs,
                             int M, int max_len, int window, int* err, cudaStream_t stream,
                             int long_len = 0x7fffffff);

// Raise the attention kernels' dynamic shared-memory limit on the current
// device (before any capture).
cudaError_t attention_prepare();

// attention_tc.cu: the tcgen05 kernel for global layers, on sequences of at
// least `min_len` tokens (shorter ones are left to launch_attention's
// mma.sync kernel, which skips the long ones when told their threshold).
// qkv_map: make_tmap_2d over qkv [M][2304] with 128-row boxes.
cudaError_t launch_attention_tc(bool bf16, const CUtensorMap& qkv_map, void* out, const int* cu_seqlens, int n_seqs,
                                int M, int max_len, int min_len, int* err, cudaStream_t stream);
cudaError_t attention_tc_prepare();

// Sequences this long or longer take the tcgen05 kernel on global layers
// (LAYA_ATTN_TC_MIN_LEN in the environment overrides; 0 disables it).
int attention_tc_min_len();

}  // namespace laya
