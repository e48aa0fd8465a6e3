// Tree-masked verify attention for float32 models, on the CUDA cores.
//
// Same operation as ddt_tree_attention (softmax(Q K^T * scale + tree mask) V
// with GQA, the mask given as packed ancestor bits), for targets that run in
// float32.  The tensor cores have no float32 input form that keeps 1e-5
// relative accuracy (kind::tf32 rounds operands to 10 mantissa bits), so this
// kernel does the dot products with fp32 FMAs and the exponentials with the
// accurate expf.  It is the numerics path for float32 checks and small
// models, not the throughput path: the bf16 models of every benchmark
// configuration use the tcgen05 kernel.
//
// Layout: one CTA per (block of 16 query rows, KV head).  A row is one
// (token, query head of the group) pair, token-major.  The CTA stages 32
// keys of K and V at a time in shared memory; each warp owns 4 rows.  For a
// row, lane j scores key j of the chunk against the row's query (K rows
// padded to 129 floats so the 32 lanes hit 32 banks), the warp keeps the
// online-softmax max and sum, and each lane accumulates 4 of the 128 output
// dimensions.
//
// The prefix length may come from device memory (`past_dev`), so a captured
// launch serves every round of a decode loop: keys [past, past + n_tokens)
// are the tree rows, keys past them are never read.
#include "common.cuh"

namespace ddt {
namespace attn32 {

constexpr int HD = 128;
constexpr int KC = 32;          // keys per shared-memory chunk
constexpr int ROWS = 16;        // query rows per CTA
constexpr int WARPS = 4;
constexpr int RPW = ROWS / WARPS;
constexpr int KPAD = HD + 1;

struct Params {
    const float* q;
    int64_t q_stride_tok, q_stride_head;
    const float* k;
    const float* v;
    int64_t kv_stride_head, kv_stride_row;
    float* out;
    int64_t o_stride_tok, o_stride_head;
    int n_tokens, hq, hkv, group;
    int past;                   // the prefix length, or its upper bound when past_dev is given
    const int32_t* past_dev;    // nullable: device-side prefix length, clamped to [0, past]
    const uint32_t* vis;
    int vis_words;
    const int64_t* key_lo;      // nullable: sliding-window lower bound per token
    float scale;
};

__global__ void __launch_bounds__(WARPS * 32)
tree_attn_f32_kernel(Params p) {
    __shared__ float ks[KC][KPAD];
    __shared__ float4 vs[KC][HD / 4];
    __shared__ float qs[ROWS][HD];

    const int h = blockIdx.y;                  // KV head
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int rows_total = p.n_tokens * p.group;
    const int row0 = blockIdx.x * ROWS;
    const int past = p.past_dev ? min(max(__ldg(p.past_dev), 0), p.past) : p.past;
    const int kv_len = past + p.n_tokens;

    // stage the CTA's query rows (zeros for rows past the end)
    for (int i = threadIdx.x; i < ROWS * (HD / 4); i += blockDim.x) {
        const int r = i / (HD / 4), c4 = i % (HD / 4);
        const int R = row0 + r;
        float4 val = make_float4(0.f, 0.f, 0.f, 0.f);
        if (R < rows_total) {
            const int t = R / p.group, g = R % p.group;
            const float* src = p.q + (int64_t)t * p.q_stride_tok + (int64_t)(h * p.group + g) * p.q_stride_head;
            val = *reinterpret_cast<const float4*>(src + 4 * c4);
        }
        *reinterpret_cast<float4*>(&qs[r][4 * c4]) = val;
    }

    int tok[RPW], lo[RPW];
    bool valid[RPW];
    float m[RPW], l[RPW], o[RPW][4];
#pragma unroll
    for (int i = 0; i < RPW; ++i) {
        const int R = row0 + warp * RPW + i;
        valid[i] = R < rows_total;
        tok[i] = valid[i] ? R / p.group : 0;
        lo[i] = 0;
        if (valid[i] && p.key_lo) {
            const int64_t x = __ldg(p.key_lo + tok[i]);
            lo[i] = x <= 0 ? 0 : (x >= past ? past : (int)x);
        }
        m[i] = -INFINITY;
        l[i] = 0.f;
        o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
    }

    const float* kh = p.k + (int64_t)h * p.kv_stride_head;
    const float* vh = p.v + (int64_t)h * p.kv_stride_head;
    for (int k0 = 0; k0 < kv_len; k0 += KC) {
        __syncthreads();   // the previous chunk is no longer read
        for (int i = threadIdx.x; i < KC * (HD / 4); i += blockDim.x) {
            const int j = i / (HD / 4), c4 = i % (HD / 4);
            float4 kv4 = make_float4(0.f, 0.f, 0.f, 0.f), vv4 = kv4;
            if (k0 + j < kv_len) {
                kv4 = *reinterpret_cast<const float4*>(kh + (int64_t)(k0 + j) * p.kv_stride_row + 4 * c4);
                vv4 = *reinterpret_cast<const float4*>(vh + (int64_t)(k0 + j) * p.kv_stride_row + 4 * c4);
            }
            ks[j][4 * c4 + 0] = kv4.x;
            ks[j][4 * c4 + 1] = kv4.y;
            ks[j][4 * c4 + 2] = kv4.z;
            ks[j][4 * c4 + 3] = kv4.w;
            vs[j][c4] = vv4;
        }
        __syncthreads();
        const int key = k0 + lane;
#pragma unroll
        for (int i = 0; i < RPW; ++i) {
            if (!valid[i]) continue;                    // warp-uniform
            const float* qr = qs[warp * RPW + i];
            float s = 0.f;
#pragma unroll 8
            for (int d = 0; d < HD; ++d) s = fmaf(qr[d], ks[lane][d], s);
            bool vis = key < kv_len;
            if (vis) {
                if (key < past) {
                    vis = key >= lo[i];
                } else {
                    const int u = key - past;
                    vis = (__ldg(p.vis + (int64_t)tok[i] * p.vis_words + (u >> 5)) >> (u & 31)) & 1u;
                }
            }
            s = vis ? s * p.scale : -INFINITY;
            float cm = s;
#pragma unroll
            for (int off = 16; off; off >>= 1) cm = fmaxf(cm, __shfl_xor_sync(DDT_FULL_MASK, cm, off));
            const float mn = fmaxf(m[i], cm);
            if (mn == -INFINITY) continue;             // nothing visible yet (warp-uniform)
            const float alpha = expf(m[i] - mn);       // m = -inf gives 0
            const float pj = vis ? expf(s - mn) : 0.f;
            float ps = pj;
#pragma unroll
            for (int off = 16; off; off >>= 1) ps += __shfl_xor_sync(DDT_FULL_MASK, ps, off);
            l[i] = l[i] * alpha + ps;
            m[i] = mn;
            float a0 = o[i][0] * alpha, a1 = o[i][1] * alpha, a2 = o[i][2] * alpha, a3 = o[i][3] * alpha;
#pragma unroll 8
            for (int j = 0; j < KC; ++j) {
                const float w = __shfl_sync(DDT_FULL_MASK, pj, j);
                const float4 vv = vs[j][lane];
                a0 = fmaf(w, vv.x, a0);
                a1 = fmaf(w, vv.y, a1);
                a2 = fmaf(w, vv.z, a2);
                a3 = fmaf(w, vv.w, a3);
            }
            o[i][0] = a0; o[i][1] = a1; o[i][2] = a2; o[i][3] = a3;
        }
    }
#pragma unroll
    for (int i = 0; i < RPW; ++i) {
        if (!valid[i]) continue;
        const int R = row0 + warp * RPW + i;
        const int g = R % p.group;
        const float inv = l[i] > 0.f ? 1.f / l[i] : 0.f;
        float* dst = p.out + (int64_t)tok[i] * p.o_stride_tok + (int64_t)(h * p.group + g) * p.o_stride_head;
        *reinterpret_cast<float4*>(dst + 4 * lane) = make_float4(o[i][0] * inv, o[i][1] * inv, o[i][2] * inv,
                                                                 o[i][3] * inv);
    }
}

}  // namespace attn32
}  // namespace ddt

using namespace ddt;

extern "C" int ddt_tree_attention_f32(const ddt_attention_args* a, const int64_t* key_lo, const int32_t* past_dev,
                                      ddt_stream_t stream) {
    using namespace ddt::attn32;
    if (!a) return set_error(DDT_EINVAL, "args is null");
    if (!a->q || !a->k || !a->v || !a->out || !a->visibility) return set_error(DDT_EINVAL, "null tensor pointer");
    if (a->head_dim != HD) return set_error(DDT_EUNSUPPORTED, "head_dim %lld (only 128)", (long long)a->head_dim);
    if (a->n_tokens <= 0 || a->hq <= 0 || a->hkv <= 0 || a->hq % a->hkv)
        return set_error(DDT_EINVAL, "bad head counts / tokens");
    if (a->past_length < 0 || a->kv_rows < a->past_length + a->n_tokens)
        return set_error(DDT_EINVAL, "kv_rows %lld < past %lld + n_tokens %lld", (long long)a->kv_rows,
                         (long long)a->past_length, (long long)a->n_tokens);
    if (a->past_length + a->n_tokens >= ((int64_t)1 << 31) || a->n_tokens * a->hq >= ((int64_t)1 << 31))
        return set_error(DDT_EINVAL, "sequence too long");
    if (a->vis_words < ceil_div(a->n_tokens, 32)) return set_error(DDT_EINVAL, "vis_words too small");
    if (!(a->scale == a->scale) || a->scale <= 0.f) return set_error(DDT_EINVAL, "scale must be positive");
    auto mis = [](const void* ptr, int b) { return reinterpret_cast<uintptr_t>(ptr) % b != 0; };
    if (mis(a->q, 16) || mis(a->k, 16) || mis(a->v, 16) || mis(a->out, 16))
        return set_error(DDT_EINVAL, "q/k/v/out must be 16-byte aligned");
    if (a->q_stride_tok % 4 || a->q_stride_head % 4 || a->kv_stride_head % 4 || a->kv_stride_row % 4 ||
        a->o_stride_tok % 4 || a->o_stride_head % 4)
        return set_error(DDT_EINVAL, "strides must be multiples of 4 elements");
    if (key_lo && mis(key_lo, 8)) return set_error(DDT_EINVAL, "key_lo must be 8-byte aligned");
    if (past_dev && mis(past_dev, 4)) return set_error(DDT_EINVAL, "past_dev must be 4-byte aligned");
    Params p;
    p.q = static_cast<const float*>(a->q);
    p.q_stride_tok = a->q_stride_tok;
    p.q_stride_head = a->q_stride_head;
    p.k = static_cast<const float*>(a->k);
    p.v = static_cast<const float*>(a->v);
    p.kv_stride_head = a->kv_stride_head;
    p.kv_stride_row = a->kv_stride_row;
    p.out = static_cast<float*>(a->out);
    p.o_stride_tok = a->o_stride_tok;
    p.o_stride_head = a->o_stride_head;
    p.n_tokens = (int)a->n_tokens;
    p.hq = (int)a->hq;
    p.hkv = (int)a->hkv;
    p.group = (int)(a->hq / a->hkv);
    p.past = (int)a->past_length;
    p.past_dev = past_dev;
    p.vis = a->visibility;
    p.vis_words = (int)a->vis_words;
    p.key_lo = key_lo;
    p.scale = a->scale;
    const int64_t rows = a->n_tokens * p.group;
    dim3 grid((unsigned)ceil_div(rows, ROWS), (unsigned)a->hkv);
    tree_attn_f32_kernel<<<grid, WARPS * 32, 0, reinterpret_cast<cudaStream_t>(stream)>>>(p);
    return check_launch("tree_attn_f32_kernel");
}
