// In-place append of new K/V rows into a preallocated cache at a row offset
// read from device memory.
//
// The reference's verify forward grows every layer's cache with
// DynamicCache.update, a torch.cat of the whole cache per layer per round
// (transformers cache_utils.py, DynamicLayer.update, reached from
// ddtree.py:523-531).  A preallocated cache only copies the new rows; taking
// the destination row from device memory lets one captured launch serve
// every round of a decode loop, whose prefix length changes each round.
//
// One CTA per (head, K or V): the CTA copies the rows of that head with
// 16-byte loads and stores.  Rows whose destination falls outside
// [0, dst_rows) are skipped, so a bad offset never writes out of bounds.
#include "common.cuh"

namespace ddt {
namespace cache {

constexpr int kThreads = 256;

__global__ void __launch_bounds__(kThreads)
kv_append_kernel(const unsigned char* __restrict__ k_src, const unsigned char* __restrict__ v_src,
                 int64_t s_head, int64_t s_row, unsigned char* k_dst, unsigned char* v_dst, int64_t d_head,
                 int64_t d_row, int64_t dst_rows, int rows, int row_bytes, const int32_t* offset_dev,
                 const int32_t* rows_dev) {
    griddep_launch_dependents();
    griddep_wait();
    const int h = blockIdx.x >> 1;
    const bool is_v = blockIdx.x & 1;
    const int off = __ldg(offset_dev);
    int n = rows;
    if (rows_dev) {
        const int r = __ldg(rows_dev);
        n = r < 0 ? 0 : (r < rows ? r : rows);
    }
    const unsigned char* src = (is_v ? v_src : k_src) + (int64_t)h * s_head;
    unsigned char* dst = (is_v ? v_dst : k_dst) + (int64_t)h * d_head;
    const int vec = row_bytes >> 4;
    for (int i = threadIdx.x; i < n * vec; i += kThreads) {
        const int r = i / vec, c = i % vec;
        const int64_t row = (int64_t)off + r;
        if (row < 0 || row >= dst_rows) continue;
        const uint4 x = *reinterpret_cast<const uint4*>(src + (int64_t)r * s_row + c * 16);
        *reinterpret_cast<uint4*>(dst + row * d_row + c * 16) = x;
    }
}

}  // namespace cache
}  // namespace ddt

using namespace ddt;

extern "C" int ddt_kv_append(const void* k_src, const void* v_src, int64_t src_head_stride_bytes,
                             int64_t src_row_stride_bytes, void* k_dst, void* v_dst, int64_t dst_head_stride_bytes,
                             int64_t dst_row_stride_bytes, int64_t dst_rows, int64_t heads, int64_t rows,
                             int64_t row_bytes, const int32_t* offset_dev, const int32_t* rows_dev,
                             ddt_stream_t stream) {
    if (!k_src || !v_src || !k_dst || !v_dst || !offset_dev) return set_error(DDT_EINVAL, "null argument");
    if (heads <= 0 || rows < 0 || row_bytes <= 0 || dst_rows < 0) return set_error(DDT_EINVAL, "bad sizes");
    if (rows == 0) return DDT_OK;
    if (heads > 32768 || rows > (1 << 24) || row_bytes > (1 << 20)) return set_error(DDT_EUNSUPPORTED, "sizes too large");
    auto mis = [](const void* p) { return reinterpret_cast<uintptr_t>(p) % 16 != 0; };
    if (mis(k_src) || mis(v_src) || mis(k_dst) || mis(v_dst) || row_bytes % 16 || src_head_stride_bytes % 16 ||
        src_row_stride_bytes % 16 || dst_head_stride_bytes % 16 || dst_row_stride_bytes % 16)
        return set_error(DDT_EINVAL, "pointers, strides and row bytes must be multiples of 16 bytes");
    if (src_row_stride_bytes < row_bytes || dst_row_stride_bytes < row_bytes)
        return set_error(DDT_EINVAL, "row strides smaller than a row");
    if (reinterpret_cast<uintptr_t>(offset_dev) % 4 || (rows_dev && reinterpret_cast<uintptr_t>(rows_dev) % 4))
        return set_error(DDT_EINVAL, "offset_dev / rows_dev must be 4-byte aligned");
    launch_k(cache::kv_append_kernel, dim3((unsigned)(2 * heads)), dim3(cache::kThreads), 0,
             reinterpret_cast<cudaStream_t>(stream), static_cast<const unsigned char*>(k_src),
             static_cast<const unsigned char*>(v_src), src_head_stride_bytes, src_row_stride_bytes,
             static_cast<unsigned char*>(k_dst), static_cast<unsigned char*>(v_dst), dst_head_stride_bytes,
             dst_row_stride_bytes, dst_rows, (int)rows, (int)row_bytes, offset_dev, rows_dev);
    return check_launch("kv_append_kernel");
}
