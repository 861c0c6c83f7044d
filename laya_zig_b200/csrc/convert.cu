// convert.cu -- weight upload conversions (run once per context).
//
// The reference keeps matrices as F16 views of the mapped file and widens
// small tensors to f32 copies (src/main.zig:1312-1355). Here every matrix is
// converted on the device into the GEMM element type (bf16 by default, f16
// optionally) and every small tensor into f32; the GLU input projection is
// also re-ordered so that a 256-row GEMM tile holds 128 gate rows and the
// 128 up rows they multiply (the fused GLU epilogue needs both).
#include "kernels.cuh"

namespace laya {
namespace {

__device__ __forceinline__ float load_any(const void* src, int dtype, size_t i) {
    if (dtype == 0) return static_cast<const float*>(src)[i];
    const uint16_t u = static_cast<const uint16_t*>(src)[i];
    if (dtype == 1) return __half2float(__ushort_as_half(u));
    return __uint_as_float((uint32_t)u << 16);
}

template <typename T>
__device__ __forceinline__ T from_f(float v);
template <>
__device__ __forceinline__ __nv_bfloat16 from_f<__nv_bfloat16>(float v) { return __float2bfloat16_rn(v); }
template <>
__device__ __forceinline__ __half from_f<__half>(float v) { return __float2half_rn(v); }

template <typename T>
__global__ void convert16_kernel(T* dst, const void* src, int dtype, size_t rows, size_t cols, int glu_tile) {
    const size_t n = rows * cols;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        const size_t r = i / cols, c = i % cols;
        size_t sr = r;
        if (glu_tile > 0) {
            const size_t half = rows / 2, ht = glu_tile / 2;
            const size_t t = r / glu_tile, j = r % glu_tile;
            sr = j < ht ? t * ht + j : half + t * ht + (j - ht);
        }
        dst[i] = from_f<T>(load_any(src, dtype, sr * cols + c));
    }
}

__global__ void convert_f32_kernel(float* dst, const void* src, int dtype, size_t n) {
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        dst[i] = load_any(src, dtype, i);
}

__global__ void transpose_f32_kernel(float* dst, const float* src, int rows, int cols) {
    const size_t n = (size_t)rows * cols;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        const size_t r = i / cols, c = i % cols;
        dst[c * rows + r] = src[i];
    }
}

}  // namespace

cudaError_t launch_transpose_f32(float* dst, const float* src, int rows, int cols, cudaStream_t s) {
    transpose_f32_kernel<<<148 * 4, 256, 0, s>>>(dst, src, rows, cols);
    return cudaGetLastError();
}

cudaError_t launch_convert16(void* dst, bool dst_bf16, const void* src, int src_dtype, size_t rows, size_t cols,
                             int glu_tile, cudaStream_t s) {
    const int grid = 148 * 8;
    if (dst_bf16)
        convert16_kernel<__nv_bfloat16><<<grid, 256, 0, s>>>(static_cast<__nv_bfloat16*>(dst), src, src_dtype, rows,
                                                             cols, glu_tile);
    else
        convert16_kernel<__half><<<grid, 256, 0, s>>>(static_cast<__half*>(dst), src, src_dtype, rows, cols, glu_tile);
    return cudaGetLastError();
}

cudaError_t launch_convert_f32(float* dst, const void* src, int src_dtype, size_t n, cudaStream_t s) {
    convert_f32_kernel<<<148 * 4, 256, 0, s>>>(dst, src, src_dtype, n);
    return cudaGetLastError();
}

}  // namespace laya
