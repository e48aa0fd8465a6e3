// Shared helpers for the sm_100a kernels of the DDTree hot path.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include "../../include/ddtree_b200.h"

#define DDT_FULL_MASK 0xffffffffu

namespace ddt {

// Record an error message for ddt_last_error() and return the status.
int set_error(int status, const char* fmt, ...);
int check_launch(const char* what);
// Fill *a with the programmatic-stream-serialization launch attribute and
// return 1 while ddt_set_pdl(1) is in force; else return 0.
unsigned pdl_attr(cudaLaunchAttribute* a);
bool pdl_enabled();

// Launch `kernel` on `st`, as a programmatic dependent launch while
// ddt_set_pdl(1) is in force.
template <typename... KArgs, typename... Args>
cudaError_t launch_k(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                     Args&&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    cfg.numAttrs = pdl_attr(attr);
    cfg.attrs = attr;
    return cudaLaunchKernelEx(&cfg, kernel, static_cast<Args&&>(args)...);
}

// Programmatic dependent launch: wait until the preceding grid in the
// stream has completed and its memory is visible (returns at once when the
// kernel was not launched as a dependent) ...
__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
// ... and let the next grid in the stream be scheduled once every CTA of this
// grid has executed this (or exited).
__device__ __forceinline__ void griddep_launch_dependents() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// Order-preserving map of an fp32 bit pattern onto uint32 (larger float ->
// larger integer; NaN with the sign bit clear maps above +inf).
__device__ __forceinline__ uint32_t ord_f32(float f) {
    uint32_t u = __float_as_uint(f);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float unord_f32(uint32_t o) {
    uint32_t u = (o & 0x80000000u) ? (o & 0x7fffffffu) : ~o;
    return __uint_as_float(u);
}
// Top-k key of a logit: the ordered value, then the complement of the token
// id, so that larger keys are larger values and, among equal values, lower
// ids (torch.topk's order is undefined on ties; this library's is this one).
__device__ __forceinline__ unsigned long long topk_key(float v, int64_t idx) {
    return ((unsigned long long)ord_f32(v) << 32) | (unsigned long long)(0xffffffffu - (uint32_t)idx);
}

// Per-block statistics that the draft head's GEMM (ddt_wgemm_head) leaves
// for the tree build (ddt_tree_build_head): for every token row t and every
// block b of 128 vocabulary rows, the max m[t][b] of the block's bf16
// logits (NaN if the block holds one), s[t][b] = sum of exp(x - m[t][b])
// over them (summed in float64, stored as float32), and the block's largest
// topk_key() key[t][b].
constexpr int kHeadBlock = 128;
struct HeadStatsLayout {
    size_t m, s, keys, total;
};
__host__ __device__ inline HeadStatsLayout head_stats_layout(int64_t rows, int64_t nblk) {
    HeadStatsLayout h;
    const size_t n = (size_t)rows * (size_t)nblk;
    h.m = 0;
    h.s = (sizeof(float) * n + 255) & ~size_t(255);
    h.keys = h.s + ((sizeof(float) * n + 255) & ~size_t(255));
    h.total = h.keys + sizeof(unsigned long long) * n;
    return h;
}

// Same for float64.
__device__ __forceinline__ uint64_t ord_f64(double d) {
    uint64_t u = (uint64_t)__double_as_longlong(d);
    return (u & 0x8000000000000000ull) ? ~u : (u | 0x8000000000000000ull);
}

__device__ __forceinline__ float bf16_bits_to_f32(uint16_t b) {
    return __uint_as_float(((uint32_t)b) << 16);
}

template <typename T>
__device__ __forceinline__ float to_f32(T v);
template <>
__device__ __forceinline__ float to_f32<float>(float v) { return v; }
template <>
__device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }
template <>
__device__ __forceinline__ float to_f32<__half>(__half v) { return __half2float(v); }

template <typename T>
__device__ __forceinline__ T from_f32(float v);
template <>
__device__ __forceinline__ float from_f32<float>(float v) { return v; }
template <>
__device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float v) { return __float2bfloat16_rn(v); }
template <>
__device__ __forceinline__ __half from_f32<__half>(float v) { return __float2half_rn(v); }

// value rounded to T and back (identity for float)
template <typename T>
__device__ __forceinline__ float rnd(float v) { return to_f32<T>(from_f32<T>(v)); }

// SiLU(g) * u for g, u already in T: silu rounded to T first, then the
// product rounded, as torch's act_fn(gate) * up does in T.
template <typename T>
__device__ __forceinline__ T silu_times(T g, T u) {
    const float gv = to_f32<T>(g);
    const float s = rnd<T>(gv / (1.f + expf(-gv)));
    return from_f32<T>(s * to_f32<T>(u));
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__host__ __device__ __forceinline__ int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }

}  // namespace ddt
