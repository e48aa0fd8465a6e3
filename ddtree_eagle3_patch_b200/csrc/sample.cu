// Temperature sampling of verify rows on sm_100a.
//
// Replaces sample(logits, temperature) for temperature > 0
// (model/utils.py:31-35): softmax(logits / T) followed by
// torch.multinomial(probs, 1), one draw per row.  The draw is made with the
// Gumbel-max rule: argmax_j (logits_j / T + G_j), G_j = -log(-log U_j), with
// U_j uniform in (0, 1), is distributed exactly as softmax(logits / T).  The
// uniforms come from Philox4x32-10 (Salmon, Moraes, Dror, Shaw: "Parallel
// random numbers: as easy as 1, 2, 3", SC 2011), keyed by the caller's seed
// and counted by (element / 4, row, offset), so a (seed, offset) pair gives
// the same draws on every run and a new offset gives fresh ones.  The draws
// follow the same distribution as torch's, not torch's generator stream.
//
// Bound: compute (a quarter of a Philox block and two logarithms per
// element), over one read of the logits (n_rows x vocab).  Two launches:
// (rows x chunks) CTAs each reduce a chunk to its best 64-bit key (ordered
// value, then the complement of the index, so ties go to the lower index)
// into the workspace; one warp per row then reduces its chunks.
#include "common.cuh"

namespace ddt {
namespace sample {

constexpr int kThreads = 256;
constexpr int kChunks = 16;

// Philox4x32-10: ten rounds of the published round function.
__device__ __forceinline__ uint4 philox4x32_10(uint4 ctr, uint2 key) {
    constexpr uint32_t kM0 = 0xD2511F53u, kM1 = 0xCD9E8D57u;
    constexpr uint32_t kW0 = 0x9E3779B9u, kW1 = 0xBB67AE85u;
#pragma unroll
    for (int r = 0; r < 10; ++r) {
        const uint32_t hi0 = __umulhi(kM0, ctr.x), lo0 = kM0 * ctr.x;
        const uint32_t hi1 = __umulhi(kM1, ctr.z), lo1 = kM1 * ctr.z;
        ctr = make_uint4(hi1 ^ ctr.y ^ key.x, lo1, hi0 ^ ctr.w ^ key.y, lo0);
        key.x += kW0;
        key.y += kW1;
    }
    return ctr;
}

// Uniform in (0, 1): (x + 0.5) / 2^32, never 0 or 1 in float.
__device__ __forceinline__ float unit_open(uint32_t x) {
    return fminf(((float)x + 0.5f) * 2.3283064365386963e-10f, 0.99999994f);
}

// E = -log(u) >= 1.1e-10.  Within 2^-6 of u = 1 it is the series
// w + w^2/2 + w^3/3 + w^4/4 in w = 1 - u, which the draw gives exactly
// ((~x + 0.5) 2^-32; truncation below 1.3e-8 relative), so E never reaches
// 0.  Elsewhere |log2 u| > 0.022 and the hardware base-2 logarithm's
// absolute error (~2^-22) stays below 1e-5 of it.
__device__ __forceinline__ float neg_log_unit(uint32_t x) {
    if (x >= 0xFC000000u) {
        const float w = ((float)(~x) + 0.5f) * 2.3283064365386963e-10f;
        return w * (1.f + w * (0.5f + w * (0.33333334f + w * 0.25f)));
    }
    return -__log2f(unit_open(x)) * 0.6931471805599453f;
}

__device__ __forceinline__ float gumbel(uint32_t x) {
    return -__log2f(neg_log_unit(x)) * 0.6931471805599453f;
}

template <typename T>
__device__ __forceinline__ float to_f32(T v);
template <>
__device__ __forceinline__ float to_f32<float>(float v) { return v; }
template <>
__device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }
template <>
__device__ __forceinline__ float to_f32<__half>(__half v) { return __half2float(v); }

// Best key of a candidate: ordered perturbed value, then ~index.  A NaN
// logit never wins (its key is 0).
__device__ __forceinline__ unsigned long long cand_key(float v, float inv_t, uint32_t x, int64_t j) {
    const float s = fmaf(v, inv_t, gumbel(x));
    if (s != s) return 0ull;
    return ((unsigned long long)ord_f32(s) << 32) | (0xffffffffu - (uint32_t)j);
}

__device__ __forceinline__ unsigned long long warp_max_u64(unsigned long long v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const unsigned long long w = __shfl_xor_sync(DDT_FULL_MASK, v, o);
        v = w > v ? w : v;
    }
    return v;
}

// CTA (chunk c, row r): the best key of elements [c0, c1) of row r.  Each
// thread takes groups of four consecutive elements, one Philox block each.
template <typename T>
__global__ void __launch_bounds__(kThreads)
chunk_kernel(const T* __restrict__ logits, int64_t vocab, int64_t row_stride, int64_t chunk, float inv_t,
             uint2 key, uint2 offset, unsigned long long* __restrict__ best) {
    const int c = blockIdx.x;
    const int64_t r = blockIdx.y;
    const int64_t c0 = (int64_t)c * chunk, c1 = min(c0 + chunk, vocab);
    const T* row = logits + r * row_stride;
    unsigned long long b = 0ull;
    for (int64_t q = c0 / 4 + threadIdx.x; 4 * q < c1; q += kThreads) {
        const uint4 x = philox4x32_10(make_uint4((uint32_t)q, (uint32_t)r, offset.x, offset.y), key);
        const uint32_t xs[4] = {x.x, x.y, x.z, x.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const int64_t j = 4 * q + e;
            if (j < c1) {
                const unsigned long long k = cand_key(to_f32(row[j]), inv_t, xs[e], j);
                b = k > b ? k : b;
            }
        }
    }
    b = warp_max_u64(b);
    __shared__ unsigned long long wb[kThreads / 32];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (lane == 0) wb[warp] = b;
    __syncthreads();
    if (warp == 0) {
        b = lane < kThreads / 32 ? wb[lane] : 0ull;
        b = warp_max_u64(b);
        if (lane == 0) best[r * kChunks + c] = b;
    }
}

// One warp per row: the best of its chunks, decoded to the token index.
__global__ void __launch_bounds__(128)
finish_kernel(const unsigned long long* __restrict__ best, int64_t n_rows, int64_t* __restrict__ out) {
    const int64_t r = (int64_t)blockIdx.x * 4 + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (r >= n_rows) return;
    unsigned long long b = lane < kChunks ? best[r * kChunks + lane] : 0ull;
    b = warp_max_u64(b);
    if (lane == 0) out[r] = b ? (int64_t)(0xffffffffu - (uint32_t)b) : 0;
}

}  // namespace sample
}  // namespace ddt

using namespace ddt;

extern "C" size_t ddt_sample_rows_workspace_size(int64_t n_rows, int64_t vocab) {
    (void)vocab;
    return n_rows > 0 ? sizeof(unsigned long long) * (size_t)n_rows * sample::kChunks : 256;
}

extern "C" int ddt_sample_rows(const void* logits, int dtype, int64_t n_rows, int64_t vocab, int64_t row_stride,
                               float temperature, uint64_t seed, uint64_t offset, int64_t* out, void* workspace,
                               size_t workspace_bytes, ddt_stream_t stream) {
    if (n_rows < 0 || vocab <= 0 || vocab >= ((int64_t)1 << 31) || row_stride < vocab)
        return set_error(DDT_EINVAL, "bad sizes (n_rows %lld, vocab %lld, row_stride %lld)", (long long)n_rows,
                         (long long)vocab, (long long)row_stride);
    if (!(temperature > 0.f) || !(temperature < INFINITY))
        return set_error(DDT_EINVAL, "temperature must be positive and finite (greedy rows use ddt_argmax_rows)");
    if (n_rows == 0) return DDT_OK;
    if (!logits || !out) return set_error(DDT_EINVAL, "null pointer");
    if (!workspace || workspace_bytes < ddt_sample_rows_workspace_size(n_rows, vocab) ||
        reinterpret_cast<uintptr_t>(workspace) % 256)
        return set_error(DDT_EWORKSPACE, "sample workspace needs %zu bytes (256-aligned)",
                         ddt_sample_rows_workspace_size(n_rows, vocab));
    if (n_rows > 65535) return set_error(DDT_EUNSUPPORTED, "n_rows %lld > 65535", (long long)n_rows);
    // chunks of a multiple of four elements, so each Philox block stays in one chunk
    const int64_t chunk = ceil_div(ceil_div(vocab, sample::kChunks), 4) * 4;
    const float inv_t = 1.f / temperature;
    const uint2 key = make_uint2((uint32_t)seed, (uint32_t)(seed >> 32));
    const uint2 off = make_uint2((uint32_t)offset, (uint32_t)(offset >> 32));
    auto* best = static_cast<unsigned long long*>(workspace);
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    const dim3 grid(sample::kChunks, (unsigned)n_rows);
    switch (dtype) {
        case DDT_F32:
            sample::chunk_kernel<float><<<grid, sample::kThreads, 0, st>>>(
                static_cast<const float*>(logits), vocab, row_stride, chunk, inv_t, key, off, best);
            break;
        case DDT_BF16:
            sample::chunk_kernel<__nv_bfloat16><<<grid, sample::kThreads, 0, st>>>(
                static_cast<const __nv_bfloat16*>(logits), vocab, row_stride, chunk, inv_t, key, off, best);
            break;
        case DDT_F16:
            sample::chunk_kernel<__half><<<grid, sample::kThreads, 0, st>>>(
                static_cast<const __half*>(logits), vocab, row_stride, chunk, inv_t, key, off, best);
            break;
        default:
            return set_error(DDT_EINVAL, "dtype %d is not a float type", dtype);
    }
    int rc = check_launch("sample_chunk_kernel");
    if (rc) return rc;
    sample::finish_kernel<<<(unsigned)ceil_div(n_rows, 4), 128, 0, st>>>(best, n_rows, out);
    return check_launch("sample_finish_kernel");
}
