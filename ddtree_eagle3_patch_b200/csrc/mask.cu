// Dense-mask helpers around the packed ancestor bitmask.
//
// tree_mask_fill writes the additive-mask rows that the reference's
// compile_ddtree_tree produces for an HF verify forward (ddtree.py:230-251);
// mask_to_bits goes the other way for callers that pass a dense mask to the
// verify attention (eagle3.py:28-43 builds one from a [T, T] tree mask).

#include "common.cuh"

namespace ddt {
namespace mask {

template <typename T>
__device__ __forceinline__ T from_double(double v);
template <>
__device__ __forceinline__ float from_double<float>(double v) { return (float)v; }
template <>
__device__ __forceinline__ __nv_bfloat16 from_double<__nv_bfloat16>(double v) { return __double2bfloat16(v); }
template <>
__device__ __forceinline__ __half from_double<__half>(double v) { return __double2half(v); }

template <typename T>
__global__ void tree_mask_fill_kernel(T* mask, int64_t row_stride, int64_t rows, int64_t col0, int64_t cols,
                                      int64_t past, int64_t n, const uint32_t* vis, int64_t W, int64_t prev_start,
                                      int64_t prev_len, double min_value) {
    const int64_t total = rows * cols;
    const T zero = from_double<T>(0.0), mn = from_double<T>(min_value);
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t r = i / cols, c = col0 + i % cols;
        const bool in_new = r < n && c >= past && c < past + n;
        const bool in_old = r < prev_len && c >= prev_start && c < prev_start + prev_len;
        if (in_new) {
            const int64_t u = c - past;
            const bool v = (vis[r * W + (u >> 5)] >> (u & 31)) & 1u;
            mask[r * row_stride + c] = v ? zero : mn;
        } else if (in_old) {
            mask[r * row_stride + c] = zero;
        }
    }
}

template <typename T>
__device__ __forceinline__ bool visible(T v, double min_value);
template <>
__device__ __forceinline__ bool visible<float>(float v, double mn) { return (double)v > mn * 0.5; }
template <>
__device__ __forceinline__ bool visible<__nv_bfloat16>(__nv_bfloat16 v, double mn) {
    return (double)__bfloat162float(v) > mn * 0.5;
}
template <>
__device__ __forceinline__ bool visible<__half>(__half v, double mn) { return (double)__half2float(v) > mn * 0.5; }
template <>
__device__ __forceinline__ bool visible<uint8_t>(uint8_t v, double) { return v != 0; }

template <typename T>
__global__ void mask_to_bits_kernel(const T* mask, int64_t row_stride, int64_t col_offset, int64_t n, uint32_t* vis,
                                    int64_t W, double min_value) {
    const int64_t total = n * W;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t r = i / W, w = i % W;
        uint32_t bits = 0;
        for (int b = 0; b < 32; ++b) {
            const int64_t u = w * 32 + b;
            if (u < n && visible<T>(mask[r * row_stride + col_offset + u], min_value)) bits |= 1u << b;
        }
        vis[r * W + w] = bits;
    }
}

}  // namespace mask
}  // namespace ddt

using namespace ddt;
using namespace ddt::mask;

extern "C" int ddt_tree_mask_fill(void* m, int dtype, int64_t row_stride, int64_t rows_cap, int64_t past_length,
                                  int64_t n_rows, const uint32_t* visibility, int64_t vis_words, int64_t prev_start,
                                  int64_t prev_len, double min_value, ddt_stream_t stream) {
    if (!m) return set_error(DDT_EINVAL, "mask is null");
    if (n_rows > 0 && !visibility) return set_error(DDT_EINVAL, "visibility is null");
    if (n_rows < 0 || prev_len < 0 || past_length < 0 || prev_start < 0) return set_error(DDT_EINVAL, "negative size");
    if (n_rows > rows_cap || prev_len > rows_cap) return set_error(DDT_EINVAL, "rows exceed the mask buffer");
    if (past_length + n_rows > row_stride || prev_start + prev_len > row_stride)
        return set_error(DDT_EINVAL, "columns exceed the mask row");
    if (n_rows > 0 && vis_words < ceil_div(n_rows, 32)) return set_error(DDT_EINVAL, "vis_words too small");
    int64_t rows = n_rows > prev_len ? n_rows : prev_len;
    int64_t c0 = past_length, c1 = past_length + n_rows;
    if (prev_len > 0) {
        c0 = c0 < prev_start ? c0 : prev_start;
        c1 = c1 > prev_start + prev_len ? c1 : prev_start + prev_len;
    }
    const int64_t cols = c1 - c0;
    if (rows <= 0 || cols <= 0) return DDT_OK;
    const int64_t total = rows * cols;
    const unsigned blocks = (unsigned)(ceil_div(total, 256) < 1024 ? ceil_div(total, 256) : 1024);
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    if (dtype == DDT_F32)
        tree_mask_fill_kernel<float><<<blocks, 256, 0, st>>>(static_cast<float*>(m), row_stride, rows, c0, cols,
                                                             past_length, n_rows, visibility, vis_words, prev_start,
                                                             prev_len, min_value);
    else if (dtype == DDT_BF16)
        tree_mask_fill_kernel<__nv_bfloat16><<<blocks, 256, 0, st>>>(static_cast<__nv_bfloat16*>(m), row_stride, rows,
                                                                     c0, cols, past_length, n_rows, visibility,
                                                                     vis_words, prev_start, prev_len, min_value);
    else if (dtype == DDT_F16)
        tree_mask_fill_kernel<__half><<<blocks, 256, 0, st>>>(static_cast<__half*>(m), row_stride, rows, c0, cols,
                                                              past_length, n_rows, visibility, vis_words, prev_start,
                                                              prev_len, min_value);
    else
        return set_error(DDT_EINVAL, "mask dtype %d", dtype);
    return check_launch("tree_mask_fill_kernel");
}

extern "C" int ddt_mask_to_bits(const void* m, int dtype, int64_t row_stride, int64_t col_offset, int64_t n_rows,
                                uint32_t* visibility, int64_t vis_words, ddt_stream_t stream) {
    if (!m || !visibility) return set_error(DDT_EINVAL, "null pointer");
    if (n_rows <= 0) return DDT_OK;
    if (vis_words < ceil_div(n_rows, 32)) return set_error(DDT_EINVAL, "vis_words too small");
    if (col_offset < 0 || col_offset + n_rows > row_stride) return set_error(DDT_EINVAL, "columns exceed the row");
    const int64_t total = n_rows * vis_words;
    const unsigned blocks = (unsigned)(ceil_div(total, 256) < 1024 ? ceil_div(total, 256) : 1024);
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    // the dtype's most negative finite value: anything above half of it counts as visible
    if (dtype == DDT_F32)
        mask_to_bits_kernel<float><<<blocks, 256, 0, st>>>(static_cast<const float*>(m), row_stride, col_offset,
                                                           n_rows, visibility, vis_words, -3.4028234663852886e38);
    else if (dtype == DDT_BF16)
        mask_to_bits_kernel<__nv_bfloat16><<<blocks, 256, 0, st>>>(static_cast<const __nv_bfloat16*>(m), row_stride,
                                                                   col_offset, n_rows, visibility, vis_words,
                                                                   -3.3895313892515355e38);
    else if (dtype == DDT_F16)
        mask_to_bits_kernel<__half><<<blocks, 256, 0, st>>>(static_cast<const __half*>(m), row_stride, col_offset,
                                                            n_rows, visibility, vis_words, -65504.0);
    else if (dtype == DDT_BOOL)
        mask_to_bits_kernel<uint8_t><<<blocks, 256, 0, st>>>(static_cast<const uint8_t*>(m), row_stride, col_offset,
                                                             n_rows, visibility, vis_words, 0.0);
    else
        return set_error(DDT_EINVAL, "mask dtype %d", dtype);
    return check_launch("mask_to_bits_kernel");
}
