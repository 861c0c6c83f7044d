// attention.cuh -- packed-sequence attention (declarations).
#pragma once
#include "common.cuh"

namespace laya {

// qkv: [tokens][3*768] 16-bit (q | k | v, head-major), out: [tokens][768].
// cu_seqlens: [n_seqs + 1] token offsets. window < 0: full attention,
// otherwise keys with |i - j| <= window only (src/main.zig:2440-2444).
cudaError_t launch_attention(bool bf16, const void* qkv, void* out, const int* cu_seqlens, int n_seqs, int max_len,
                             int window, cudaStream_t stream);

// Raise the attention kernels' dynamic shared-memory limit on the current
// device (before any capture).
cudaError_t attention_prepare();

}  // namespace laya
