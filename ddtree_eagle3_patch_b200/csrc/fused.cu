// Fused elementwise steps of a Qwen3-style decoder layer, for the verify and
// draft forwards of a decode round.
//
// At batch 1 with ~33 verify rows a decoder layer's GEMMs stream the weights
// once (HBM-bound, tens of microseconds), but the eager layer around them
// issues ~45 small elementwise kernels (RMSNorm alone is 7: cast, square,
// mean, add, rsqrt, multiply, weight), each a few microseconds of launch and
// tail even inside a CUDA graph.  These kernels do those steps in one pass
// each, in the arithmetic order of the stock modules so that a float32 model
// gives the same values to rounding and a bf16 model rounds where they do:
//
//   rms_norm            Qwen3RMSNorm: w * to_dtype(x * rsqrt(mean(x^2) + eps)),
//                       the mean and rsqrt in fp32
//   qk_norm_rope_append q_norm / k_norm (the same RMSNorm over head_dim), the
//                       rotary embedding (x * cos) + (rotate_half(x) * sin)
//                       with each product rounded to the dtype as torch does,
//                       the rotated queries written out and the new K/V rows
//                       written straight into the cache at rows read from
//                       device memory (so the launch can be captured once)
//   silu_mul            act_fn(gate) * up with SiLU, silu rounded first
//
// All are HBM/latency-bound elementwise passes over a few hundred KB.
#include "common.cuh"

namespace ddt {
namespace fused {

// ---------------------------------------------------------------------------
// RMSNorm of rows whose 16-byte vectors fit VPT per thread: the row is read
// once into registers, reduced, and written from registers.
template <typename T, int THREADS, int VPT>
__global__ void __launch_bounds__(THREADS)
rms_norm_vec_kernel(const T* __restrict__ x, int64_t x_stride, const T* __restrict__ w, T* __restrict__ y,
                    int64_t y_stride, int cols, float eps) {
    griddep_launch_dependents();
    griddep_wait();
    constexpr int E = 16 / sizeof(T);
    const int nv = cols / E;
    const uint4* xr = reinterpret_cast<const uint4*>(x + (int64_t)blockIdx.x * x_stride);
    const uint4* wr = reinterpret_cast<const uint4*>(w);
    uint4* yr = reinterpret_cast<uint4*>(y + (int64_t)blockIdx.x * y_stride);
    uint4 v[VPT];
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
        const int c = threadIdx.x + i * THREADS;
        v[i] = c < nv ? xr[c] : make_uint4(0u, 0u, 0u, 0u);
        const T* e = reinterpret_cast<const T*>(&v[i]);
#pragma unroll
        for (int j = 0; j < E; ++j) {
            const float f = to_f32<T>(e[j]);
            ss = fmaf(f, f, ss);
        }
    }
    __shared__ float red[THREADS / 32];
#pragma unroll
    for (int o = 16; o; o >>= 1) ss += __shfl_xor_sync(DDT_FULL_MASK, ss, o);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < THREADS / 32; ++i) s += red[i];
    const float r = rsqrtf(s / (float)cols + eps);
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
        const int c = threadIdx.x + i * THREADS;
        if (c >= nv) break;
        const uint4 wv = wr[c];
        const T* e = reinterpret_cast<const T*>(&v[i]);
        const T* we = reinterpret_cast<const T*>(&wv);
        uint4 o;
        T* oe = reinterpret_cast<T*>(&o);
#pragma unroll
        for (int j = 0; j < E; ++j) oe[j] = from_f32<T>(to_f32<T>(we[j]) * rnd<T>(to_f32<T>(e[j]) * r));
        yr[c] = o;
    }
}

// ---------------------------------------------------------------------------
// RMSNorm of rows: one CTA per row (any width or alignment).
template <typename T, int THREADS>
__global__ void __launch_bounds__(THREADS)
rms_norm_kernel(const T* __restrict__ x, int64_t x_stride, const T* __restrict__ w, T* __restrict__ y,
                int64_t y_stride, int cols, float eps) {
    griddep_launch_dependents();
    griddep_wait();
    const T* xr = x + (int64_t)blockIdx.x * x_stride;
    T* yr = y + (int64_t)blockIdx.x * y_stride;
    float ss = 0.f;
    for (int c = threadIdx.x; c < cols; c += THREADS) {
        const float v = to_f32<T>(xr[c]);
        ss = fmaf(v, v, ss);
    }
    __shared__ float red[THREADS / 32];
#pragma unroll
    for (int o = 16; o; o >>= 1) ss += __shfl_xor_sync(DDT_FULL_MASK, ss, o);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    if (threadIdx.x < 32) {
        float s = threadIdx.x < THREADS / 32 ? red[threadIdx.x] : 0.f;
#pragma unroll
        for (int o = 16; o; o >>= 1) s += __shfl_xor_sync(DDT_FULL_MASK, s, o);
        if (threadIdx.x == 0) red[0] = s;
    }
    __syncthreads();
    const float r = rsqrtf(red[0] / (float)cols + eps);
    for (int c = threadIdx.x; c < cols; c += THREADS) {
        const float v = rnd<T>(to_f32<T>(xr[c]) * r);
        yr[c] = from_f32<T>(to_f32<T>(w[c]) * v);
    }
}

// ---------------------------------------------------------------------------
// q/k RMSNorm + rotary embedding + cache append.  One CTA per K/V row; a
// warp handles one head (128 dims, 4 per lane); the rotate_half partner of
// dims 4l..4l+3 sits in lane l ^ 16.
struct RopeParams {
    const void* q_raw;
    int64_t q_stride;
    const void* a_k;
    const void* a_v;
    int64_t a_stride;
    int a_rows;
    const void* b_k;
    const void* b_v;
    int64_t b_stride;
    int b_rows;
    const void* qw;
    const void* kw;
    float eps_q, eps_k;
    const void* cos;
    const void* sin;
    int64_t cs_stride;
    int hq, hkv;
    void* q_out;
    int64_t q_out_stride;
    void* cache_k;
    void* cache_v;
    int64_t cache_head_stride, cache_row_stride, cache_rows;
    const int32_t* rs;   // [start, ctx_offset, ctx_count]
};

template <typename T>
__device__ __forceinline__ void norm_rope_head(const T* src, const T* w, float eps, const T* cosr, const T* sinr,
                                               int lane, float out[4]) {
    float x[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) x[i] = to_f32<T>(src[4 * lane + i]);
    float ss = x[0] * x[0] + x[1] * x[1] + x[2] * x[2] + x[3] * x[3];
#pragma unroll
    for (int o = 16; o; o >>= 1) ss += __shfl_xor_sync(DDT_FULL_MASK, ss, o);
    const float r = rsqrtf(ss / 128.f + eps);
    float n[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) n[i] = rnd<T>(to_f32<T>(w[4 * lane + i]) * rnd<T>(x[i] * r));
    float p[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) p[i] = __shfl_xor_sync(DDT_FULL_MASK, n[i], 16);
    const bool lo_half = lane < 16;   // dims 0..63: rotate_half gives -x[d + 64]
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const float rot = lo_half ? -p[i] : p[i];
        const float c = to_f32<T>(cosr[4 * lane + i]), s = to_f32<T>(sinr[4 * lane + i]);
        out[i] = rnd<T>(rnd<T>(n[i] * c) + rnd<T>(rot * s));
    }
}

template <typename T>
__global__ void __launch_bounds__(256)
qk_norm_rope_append_kernel(RopeParams p) {
    griddep_launch_dependents();
    griddep_wait();
    const int t = blockIdx.x;                       // K/V row: [0, a_rows) ctx, then b rows
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const bool is_b = t >= p.a_rows;
    const int tb = t - p.a_rows;
    const T* krow = is_b ? static_cast<const T*>(p.b_k) + (int64_t)tb * p.b_stride
                         : static_cast<const T*>(p.a_k) + (int64_t)t * p.a_stride;
    const T* vrow = is_b ? static_cast<const T*>(p.b_v) + (int64_t)tb * p.b_stride
                         : static_cast<const T*>(p.a_v) + (int64_t)t * p.a_stride;
    const T* cosr = static_cast<const T*>(p.cos) + (int64_t)t * p.cs_stride;
    const T* sinr = static_cast<const T*>(p.sin) + (int64_t)t * p.cs_stride;
    int64_t dest;
    if (is_b) {
        dest = (int64_t)__ldg(p.rs) + tb;
    } else {
        const int cnt = __ldg(p.rs + 2);
        dest = t < cnt ? (int64_t)__ldg(p.rs + 1) + t : -1;
    }
    const bool store_kv = dest >= 0 && dest < p.cache_rows;
    const int n_tasks = 2 * p.hkv + (is_b ? p.hq : 0);
    for (int task = blockIdx.y * 8 + warp; task < n_tasks; task += 8 * gridDim.y) {
        if (task < p.hkv) {                         // K head: norm + rope -> cache
            const int h = task;
            float o[4];
            norm_rope_head<T>(krow + h * 128, static_cast<const T*>(p.kw), p.eps_k, cosr, sinr, lane, o);
            if (store_kv) {
                T* dst = static_cast<T*>(p.cache_k) + h * p.cache_head_stride + dest * p.cache_row_stride;
#pragma unroll
                for (int i = 0; i < 4; ++i) dst[4 * lane + i] = from_f32<T>(o[i]);
            }
        } else if (task < 2 * p.hkv) {              // V head: copy -> cache
            const int h = task - p.hkv;
            if (store_kv) {
                const T* src = vrow + h * 128;
                T* dst = static_cast<T*>(p.cache_v) + h * p.cache_head_stride + dest * p.cache_row_stride;
#pragma unroll
                for (int i = 0; i < 4; ++i) dst[4 * lane + i] = src[4 * lane + i];
            }
        } else {                                     // Q head of a block row: norm + rope -> q_out
            const int h = task - 2 * p.hkv;
            const T* qrow = static_cast<const T*>(p.q_raw) + (int64_t)tb * p.q_stride + h * 128;
            float o[4];
            norm_rope_head<T>(qrow, static_cast<const T*>(p.qw), p.eps_q, cosr, sinr, lane, o);
            T* dst = static_cast<T*>(p.q_out) + (int64_t)tb * p.q_out_stride + h * 128;
#pragma unroll
            for (int i = 0; i < 4; ++i) dst[4 * lane + i] = from_f32<T>(o[i]);
        }
    }
}

// ---------------------------------------------------------------------------
// SiLU(gate) * up, elementwise (silu_times in common.cuh).

// grid (column blocks, rows): each thread one 16-byte vector of a row when
// the row strides allow it, else one element
template <typename T, bool VEC>
__global__ void __launch_bounds__(256)
silu_mul_kernel(const T* __restrict__ g, const T* __restrict__ u, int64_t in_stride, T* __restrict__ out,
                int64_t out_stride, int64_t rows, int64_t cols) {
    griddep_launch_dependents();
    griddep_wait();
    const int64_t r = blockIdx.y;
    const T* gr = g + r * in_stride;
    const T* ur = u + r * in_stride;
    T* orow = out + r * out_stride;
    if (VEC) {
        constexpr int E = 16 / sizeof(T);
        for (int64_t c = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) * E; c < cols;
             c += (int64_t)gridDim.x * blockDim.x * E) {
            const uint4 gv = *reinterpret_cast<const uint4*>(gr + c);
            const uint4 uv = *reinterpret_cast<const uint4*>(ur + c);
            uint4 ov;
            const T* ge = reinterpret_cast<const T*>(&gv);
            const T* ue = reinterpret_cast<const T*>(&uv);
            T* oe = reinterpret_cast<T*>(&ov);
#pragma unroll
            for (int j = 0; j < E; ++j) oe[j] = silu_times<T>(ge[j], ue[j]);
            *reinterpret_cast<uint4*>(orow + c) = ov;
        }
    } else {
        for (int64_t c = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; c < cols; c += (int64_t)gridDim.x * blockDim.x)
            orow[c] = silu_times<T>(gr[c], ur[c]);
    }
}

}  // namespace fused
}  // namespace ddt

using namespace ddt;

extern "C" int ddt_rms_norm(const void* x, int dtype, int64_t x_row_stride, const void* weight, void* y,
                            int64_t y_row_stride, int64_t rows, int64_t cols, float eps, ddt_stream_t stream) {
    if (!x || !weight || !y) return set_error(DDT_EINVAL, "null argument");
    if (rows < 0 || cols <= 0 || x_row_stride < cols || y_row_stride < cols) return set_error(DDT_EINVAL, "bad sizes");
    if (rows == 0) return DDT_OK;
    if (rows > 0x7fffffff || cols > (1 << 24)) return set_error(DDT_EUNSUPPORTED, "sizes too large");
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    const int esz = dtype == DDT_F32 ? 4 : 2;
    const int per_vec = 16 / esz;
    const bool vec = reinterpret_cast<uintptr_t>(x) % 16 == 0 && reinterpret_cast<uintptr_t>(y) % 16 == 0 &&
                     reinterpret_cast<uintptr_t>(weight) % 16 == 0 && cols % per_vec == 0 &&
                     x_row_stride % per_vec == 0 && y_row_stride % per_vec == 0;
    const int64_t nvec = cols / per_vec;
#define DDT_RMS_VEC(T, VPT)                                                                                         \
    launch_k(fused::rms_norm_vec_kernel<T, 256, VPT>, dim3((unsigned)rows), dim3(256), 0, st,                        \
             static_cast<const T*>(x), x_row_stride, static_cast<const T*>(weight), static_cast<T*>(y),              \
             y_row_stride, (int)cols, eps)
    if (vec && nvec <= 256 * 4 && (dtype == DDT_BF16 || dtype == DDT_F32 || dtype == DDT_F16)) {
        if (dtype == DDT_BF16) {
            if (nvec <= 512) DDT_RMS_VEC(__nv_bfloat16, 2); else DDT_RMS_VEC(__nv_bfloat16, 4);
        } else if (dtype == DDT_F16) {
            if (nvec <= 512) DDT_RMS_VEC(__half, 2); else DDT_RMS_VEC(__half, 4);
        } else {
            if (nvec <= 512) DDT_RMS_VEC(float, 2); else DDT_RMS_VEC(float, 4);
        }
#undef DDT_RMS_VEC
        return check_launch("rms_norm_vec_kernel");
    }
    const dim3 grid((unsigned)rows);
    if (dtype == DDT_BF16)
        launch_k(fused::rms_norm_kernel<__nv_bfloat16, 256>, grid, dim3(256), 0, st,
                 static_cast<const __nv_bfloat16*>(x), x_row_stride, static_cast<const __nv_bfloat16*>(weight),
                 static_cast<__nv_bfloat16*>(y), y_row_stride, (int)cols, eps);
    else if (dtype == DDT_F32)
        launch_k(fused::rms_norm_kernel<float, 256>, grid, dim3(256), 0, st, static_cast<const float*>(x),
                 x_row_stride, static_cast<const float*>(weight), static_cast<float*>(y), y_row_stride, (int)cols,
                 eps);
    else if (dtype == DDT_F16)
        launch_k(fused::rms_norm_kernel<__half, 256>, grid, dim3(256), 0, st, static_cast<const __half*>(x),
                 x_row_stride, static_cast<const __half*>(weight), static_cast<__half*>(y), y_row_stride, (int)cols,
                 eps);
    else
        return set_error(DDT_EINVAL, "dtype %d", dtype);
    return check_launch("rms_norm_kernel");
}

extern "C" int ddt_qk_norm_rope_append(int dtype, const void* q_raw, int64_t q_row_stride, const void* ctx_k,
                                       const void* ctx_v, int64_t ctx_row_stride, int64_t ctx_rows,
                                       const void* new_k, const void* new_v, int64_t new_row_stride,
                                       int64_t new_rows, const void* q_norm_weight, const void* k_norm_weight,
                                       float eps_q, float eps_k, const void* cos, const void* sin,
                                       int64_t cs_row_stride, int64_t hq, int64_t hkv, int64_t head_dim,
                                       void* q_out, int64_t q_out_row_stride, void* cache_k, void* cache_v,
                                       int64_t cache_head_stride, int64_t cache_row_stride, int64_t cache_rows,
                                       const int32_t* rs, ddt_stream_t stream) {
    if (head_dim != 128) return set_error(DDT_EUNSUPPORTED, "head_dim %lld (only 128)", (long long)head_dim);
    if (!q_raw || !new_k || !new_v || !q_norm_weight || !k_norm_weight || !cos || !sin || !q_out || !cache_k ||
        !cache_v || !rs)
        return set_error(DDT_EINVAL, "null argument");
    if (ctx_rows < 0 || new_rows <= 0 || hq <= 0 || hkv <= 0 || cache_rows < 0) return set_error(DDT_EINVAL, "bad sizes");
    if (ctx_rows > 0 && (!ctx_k || !ctx_v)) return set_error(DDT_EINVAL, "context rows without context tensors");
    if (q_row_stride < hq * 128 || new_row_stride < hkv * 128 || (ctx_rows && ctx_row_stride < hkv * 128) ||
        q_out_row_stride < hq * 128 || cs_row_stride < 128 || cache_row_stride < 128)
        return set_error(DDT_EINVAL, "row strides too small");
    if (ctx_rows + new_rows > 0x7fffffff || hq + 2 * hkv > 4096) return set_error(DDT_EUNSUPPORTED, "sizes too large");
    if (reinterpret_cast<uintptr_t>(rs) % 4) return set_error(DDT_EINVAL, "rs must be 4-byte aligned");
    fused::RopeParams p;
    p.q_raw = q_raw;
    p.q_stride = q_row_stride;
    p.a_k = ctx_k;
    p.a_v = ctx_v;
    p.a_stride = ctx_row_stride;
    p.a_rows = (int)ctx_rows;
    p.b_k = new_k;
    p.b_v = new_v;
    p.b_stride = new_row_stride;
    p.b_rows = (int)new_rows;
    p.qw = q_norm_weight;
    p.kw = k_norm_weight;
    p.eps_q = eps_q;
    p.eps_k = eps_k;
    p.cos = cos;
    p.sin = sin;
    p.cs_stride = cs_row_stride;
    p.hq = (int)hq;
    p.hkv = (int)hkv;
    p.q_out = q_out;
    p.q_out_stride = q_out_row_stride;
    p.cache_k = cache_k;
    p.cache_v = cache_v;
    p.cache_head_stride = cache_head_stride;
    p.cache_row_stride = cache_row_stride;
    p.cache_rows = cache_rows;
    p.rs = rs;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    // one warp per head task: (K heads, V heads, Q heads) of a row over grid.y CTAs of 8 warps
    const dim3 grid((unsigned)(ctx_rows + new_rows), (unsigned)ceil_div(2 * hkv + hq, 8));
    if (dtype == DDT_BF16)
        launch_k(fused::qk_norm_rope_append_kernel<__nv_bfloat16>, grid, dim3(256), 0, st, p);
    else if (dtype == DDT_F32)
        launch_k(fused::qk_norm_rope_append_kernel<float>, grid, dim3(256), 0, st, p);
    else if (dtype == DDT_F16)
        launch_k(fused::qk_norm_rope_append_kernel<__half>, grid, dim3(256), 0, st, p);
    else
        return set_error(DDT_EINVAL, "dtype %d", dtype);
    return check_launch("qk_norm_rope_append_kernel");
}

extern "C" int ddt_silu_mul_rows(const void* gate, const void* up, int64_t in_row_stride, void* out,
                                 int64_t out_row_stride, int64_t rows, int64_t cols, int dtype, ddt_stream_t stream) {
    if (!gate || !up || !out) return set_error(DDT_EINVAL, "null argument");
    if (rows < 0 || cols < 0 || (rows > 1 && (in_row_stride < cols || out_row_stride < cols)))
        return set_error(DDT_EINVAL, "bad sizes");
    if (rows == 0 || cols == 0) return DDT_OK;
    if (rows > 65535) return set_error(DDT_EUNSUPPORTED, "rows %lld > 65535", (long long)rows);
    const int esz = dtype == DDT_F32 ? 4 : 2;
    const int per_vec = 16 / esz;
    const bool vec = reinterpret_cast<uintptr_t>(gate) % 16 == 0 && reinterpret_cast<uintptr_t>(up) % 16 == 0 &&
                     reinterpret_cast<uintptr_t>(out) % 16 == 0 && cols % per_vec == 0 &&
                     (rows == 1 || (in_row_stride % per_vec == 0 && out_row_stride % per_vec == 0));
    const int64_t per_row = vec ? cols / per_vec : cols;
    const int64_t cap = 65535;
    const int64_t bx = ceil_div(per_row, 256);
    const dim3 grid((unsigned)(bx < cap ? bx : cap), (unsigned)rows);
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
#define DDT_SILU(T)                                                                                                \
    do {                                                                                                           \
        if (vec)                                                                                                   \
            launch_k(fused::silu_mul_kernel<T, true>, grid, dim3(256), 0, st, static_cast<const T*>(gate),         \
                     static_cast<const T*>(up), in_row_stride, static_cast<T*>(out), out_row_stride, rows, cols);   \
        else                                                                                                       \
            launch_k(fused::silu_mul_kernel<T, false>, grid, dim3(256), 0, st, static_cast<const T*>(gate),        \
                     static_cast<const T*>(up), in_row_stride, static_cast<T*>(out), out_row_stride, rows, cols);   \
    } while (0)
    if (dtype == DDT_BF16)
        DDT_SILU(__nv_bfloat16);
    else if (dtype == DDT_F32)
        DDT_SILU(float);
    else if (dtype == DDT_F16)
        DDT_SILU(__half);
    else
        return set_error(DDT_EINVAL, "dtype %d", dtype);
#undef DDT_SILU
    return check_launch("silu_mul_kernel");
}

extern "C" int ddt_silu_mul(const void* gate, const void* up, void* out, int dtype, int64_t n, ddt_stream_t stream) {
    if (n < 0) return set_error(DDT_EINVAL, "bad size");
    return ddt_silu_mul_rows(gate, up, n, out, n, 1, n, dtype, stream);
}
