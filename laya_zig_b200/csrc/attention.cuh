// attention.cuh -- packed-sequence attention (declarations).
#pragma once
#include "common.cuh"

namespace laya {

// qkv: [M][3*768] 16-bit (q | k | v, head-major), out: [M][768].
// cu_seqlens: [n_seqs + 1] token offsets. window < 0: full attention,
// otherwise keys with |i - j| <= window only (src/main.zig:2440-2444).
// A sequence whose offsets leave [0, M) or whose length exceeds max_len
// sets ERR_BAD_INDEX in *err and is skipped.
cudaError_t launch_attention(bool bf16, const void* qkv, void* out, const int* cu_seqlens, int n_seqs, int M,
                             int max_len, int window, int* err, cudaStream_t stream);

// Raise the attention kernels' dynamic shared-memory limit on the current
// device (before any capture).
cudaError_t attention_prepare();

}  // namespace laya
