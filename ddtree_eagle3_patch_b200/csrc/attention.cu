// Kernel (2): tree-masked verify attention on sm_100a tensor cores.
//
// One layer of softmax(Q K^T * scale + tree_mask) V for the verify forward
// (ddtree.py:523-531; the mask built at ddtree.py:247-253), GQA without
// repeating K/V.
//
// Rows of one KV head: the G = hq/hkv query heads of every tree token,
// packed token-major (row = token * G + head_in_group), 128 rows per M tile.
// CTA = (key split, M tile, KV head).  Warp roles:
//   warp 0     TMA producer: Q tile once, then K/V tiles of 128 keys into a
//              two-stage ring (128-byte swizzle, plain local loads).
//   warp 1     TMEM owner and the single tcgen05.mma issuer:
//              S[b] = Q K^T (SS MMA, 128x128x128) into TMEM columns b*128,
//              O   += P V   (TS MMA, A = P read from TMEM) into columns 256+.
//   warps 2-5  one thread per row: S from TMEM, scale, tree mask from the
//              packed ancestor bitmask, online softmax with lazy rescaling,
//              P written back over S as bf16, then the epilogue.
// With more than one split the CTA writes its normalised partial and
// log-sum-exp and attn_combine_kernel merges the splits.

#include <cudaTypedefs.h>

#include <mutex>

#include "common.cuh"
#include "sm100.cuh"

namespace ddt {
namespace attn {

using namespace ddt::sm100;

constexpr int kThreads = 192;
constexpr int BM = 128;
constexpr int BN = 128;
constexpr int HD = 128;
constexpr uint32_t kHalf = 128 * 64 * 2;  // one 64-column half of a 128-row bf16 tile (16 KB)
constexpr uint32_t kTile = 2 * kHalf;     // 32 KB
constexpr uint32_t kSmemQ = 0;
constexpr uint32_t kSmemK0 = kTile;           // K stage s at kSmemK0 + s * 2 * kTile
constexpr uint32_t kSmemV0 = 2 * kTile;       // V stage s at kSmemV0 + s * 2 * kTile
constexpr uint32_t kSmemBar = 5 * kTile;      // 160 KB
constexpr uint32_t kSmemBytes = kSmemBar + 256 + 1024;  // + barriers + alignment slack
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kIdescQK = idesc_bf16_f32(BM, BN, false, false);
constexpr uint32_t kIdescPV = idesc_bf16_f32(BM, HD, false, true);

struct Params {
    int n_tokens, hq, hkv, group, tokens_per_tile, past, n_kt, splits;
    const uint32_t* vis;
    int vis_words;
    float scale_log2;
    __nv_bfloat16* out;
    int64_t o_stride_tok, o_stride_head;
    float* part_o;
    float* part_lse;
    int* status;
};

// Visibility of keys u0 .. u0+31 relative to the tree start for one row:
// u < 0 is prefix (visible), u >= n is beyond the tree (hidden).
__device__ __forceinline__ uint32_t vis_bits(const uint32_t* row, int W, int u0, int n, bool row_valid) {
    uint32_t prefix = 0u;
    if (u0 < 0) prefix = (u0 <= -32) ? 0xffffffffu : ((1u << (-u0)) - 1u);
    if (!row_valid) return prefix;
    if (u0 + 32 <= 0) return prefix;
    uint32_t tree;
    if (u0 >= 0) {
        const int w0 = u0 >> 5, sh = u0 & 31;
        const uint32_t lo = w0 < W ? __ldg(row + w0) : 0u;
        const uint32_t hi = (w0 + 1) < W ? __ldg(row + w0 + 1) : 0u;
        tree = sh ? ((lo >> sh) | (hi << (32 - sh))) : lo;
        const int left = n - u0;
        if (left < 32) tree &= left > 0 ? ((1u << left) - 1u) : 0u;
    } else {
        const int sh = -u0;  // 1..31 columns of prefix first
        tree = __ldg(row) << sh;
        const int left = n + sh;  // column index where the tree ends
        if (left < 32) tree &= (1u << left) - 1u;
    }
    return prefix | tree;
}

__device__ __forceinline__ void flag_error(int* status, int code) {
    if (status) atomicCAS(status, 0, code);
}

__global__ void __launch_bounds__(kThreads, 1)
tree_attn_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
                 const __grid_constant__ CUtensorMap tv, const Params p) {
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    unsigned char* smem = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kSmemBar);
    uint64_t* q_full = bars + 0;
    uint64_t* kv_full = bars + 1;   // [2]
    uint64_t* s_full = bars + 3;    // [2]
    uint64_t* p_full = bars + 5;    // [2]
    uint64_t* pv_done = bars + 7;   // [2]
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 9);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int split = blockIdx.x, mt = blockIdx.y, g = blockIdx.z;
    const int kt0 = (int)((int64_t)split * p.n_kt / p.splits);
    const int kt1 = (int)((int64_t)(split + 1) * p.n_kt / p.splits);
    const int nj = kt1 - kt0;

    if (threadIdx.x == 0) {
        mbar_init(q_full, 1);
        for (int b = 0; b < 2; ++b) {
            mbar_init(&kv_full[b], 1);
            mbar_init(&s_full[b], 1);
            mbar_init(&p_full[b], 128);
            mbar_init(&pv_done[b], 1);
        }
        fence_mbar_init();
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, kTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const uint32_t s_addr = smem_u32(smem);

    if (warp == 0) {
        // ------------------------------------------------------------ producer
        if (lane == 0 && nj > 0) {
            prefetch_tmap(&tq);
            prefetch_tmap(&tk);
            prefetch_tmap(&tv);
            mbar_arrive_expect_tx(q_full, kTile);
            tma_load_3d(smem + kSmemQ, &tq, 0, g * p.group, mt * p.tokens_per_tile, q_full);
            tma_load_3d(smem + kSmemQ + kHalf, &tq, 64, g * p.group, mt * p.tokens_per_tile, q_full);
            int issued = 0;
            bool ok = true;
            for (int jj = 0; jj < nj; ++jj) {
                const int b = jj & 1;
                if (jj >= 2 && !mbar_wait(&pv_done[b], ((jj >> 1) - 1) & 1)) {
                    flag_error(p.status, 1);
                    ok = false;
                    break;
                }
                const int key0 = (kt0 + jj) * BN;
                unsigned char* ks = smem + kSmemK0 + b * 2 * kTile;
                unsigned char* vs = smem + kSmemV0 + b * 2 * kTile;
                mbar_arrive_expect_tx(&kv_full[b], 2 * kTile);
                tma_load_3d(ks, &tk, 0, key0, g, &kv_full[b]);
                tma_load_3d(ks + kHalf, &tk, 64, key0, g, &kv_full[b]);
                tma_load_3d(vs, &tv, 0, key0, g, &kv_full[b]);
                tma_load_3d(vs + kHalf, &tv, 64, key0, g, &kv_full[b]);
                issued = jj + 1;
            }
            if (!ok) {
                // let the copies already in flight land before the CTA exits
                for (int jj = issued - 2 < 0 ? 0 : issued - 2; jj < issued; ++jj)
                    mbar_wait(&kv_full[jj & 1], (jj >> 1) & 1);
                mbar_wait(q_full, 0);
            }
        }
    } else if (warp == 1) {
        // ------------------------------------------------------------ MMA issuer
        if (lane == 0 && nj > 0) {
            bool ok = mbar_wait(q_full, 0);
            tc_fence_after();
            const uint32_t q_s = s_addr + kSmemQ;
            auto issue_pv = [&](int i) -> bool {
                const int b1 = i & 1;
                if (!mbar_wait(&p_full[b1], (i >> 1) & 1)) return false;
                tc_fence_after();
                const uint32_t v_s = s_addr + kSmemV0 + b1 * 2 * kTile;
#pragma unroll
                for (int kk = 0; kk < 8; ++kk) {
                    const uint64_t bdesc = smem_desc_sw128(v_s + kk * 2048, kHalf, 1024);
                    mma_ts(tmem + 256, tmem + b1 * 128 + kk * 8, bdesc, kIdescPV, (i > 0 || kk > 0) ? 1u : 0u);
                }
                mma_commit(&pv_done[b1]);
                return true;
            };
            for (int jj = 0; jj < nj && ok; ++jj) {
                const int b = jj & 1;
                ok = mbar_wait(&kv_full[b], (jj >> 1) & 1);
                if (ok && jj >= 2) ok = mbar_wait(&pv_done[b], ((jj >> 1) - 1) & 1);
                if (!ok) break;
                tc_fence_after();
                const uint32_t k_s = s_addr + kSmemK0 + b * 2 * kTile;
#pragma unroll
                for (int kk = 0; kk < 8; ++kk) {
                    const uint32_t off = (kk >> 2) * kHalf + (kk & 3) * 32;
                    const uint64_t adesc = smem_desc_sw128(q_s + off, 16, 1024);
                    const uint64_t bdesc = smem_desc_sw128(k_s + off, 16, 1024);
                    mma_ss(tmem + b * 128, adesc, bdesc, kIdescQK, kk > 0 ? 1u : 0u);
                }
                mma_commit(&s_full[b]);
                if (jj >= 1) ok = issue_pv(jj - 1);
            }
            if (ok) ok = issue_pv(nj - 1);
            if (!ok) flag_error(p.status, 2);
            // drain: the last commit covers every MMA issued before it
            if (ok) mbar_wait(&pv_done[(nj - 1) & 1], ((nj - 1) >> 1) & 1);
        }
    } else {
        // ------------------------------------------------------------ softmax + epilogue
        const int qw = warp & 3;
        const int row = qw * 32 + lane;
        const uint32_t lane_addr = (uint32_t)(qw * 32) << 16;
        const int t_local = row / p.group;
        const int hl = row - t_local * p.group;
        const int token = mt * p.tokens_per_tile + t_local;
        const int head = g * p.group + hl;
        const bool valid = token < p.n_tokens;
        const uint32_t* vrow = valid ? p.vis + (int64_t)token * p.vis_words : p.vis;
        float m_ref = -INFINITY, l = 0.f;
        bool ok = true;
        for (int jj = 0; jj < nj && ok; ++jj) {
            const int b = jj & 1;
            if (!mbar_wait(&s_full[b], (jj >> 1) & 1)) {
                ok = false;
                break;
            }
            tc_fence_after();
            uint32_t sr[4][32];
#pragma unroll
            for (int q = 0; q < 4; ++q) tmem_ld32(tmem + lane_addr + b * 128 + q * 32, sr[q]);
            tmem_wait_ld();
            const int u_base = (kt0 + jj) * BN - p.past;
            float mx = -INFINITY;
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const uint32_t vb = vis_bits(vrow, p.vis_words, u_base + q * 32, p.n_tokens, valid);
#pragma unroll
                for (int c = 0; c < 32; ++c) {
                    float s = __uint_as_float(sr[q][c]) * p.scale_log2;
                    s = (vb >> c) & 1u ? s : -INFINITY;
                    sr[q][c] = __float_as_uint(s);
                    mx = fmaxf(mx, s);
                }
            }
            const float m_new = fmaxf(m_ref, mx);
            if (jj == 0) {
                m_ref = m_new;
            } else if (m_new > m_ref + 8.0f) {
                const float alpha = exp2f(m_ref - m_new);
                if (!mbar_wait(&pv_done[(jj - 1) & 1], ((jj - 1) >> 1) & 1)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    uint32_t o[32];
                    tmem_ld32(tmem + lane_addr + 256 + q * 32, o);
                    tmem_wait_ld();
#pragma unroll
                    for (int c = 0; c < 32; ++c) o[c] = __float_as_uint(__uint_as_float(o[c]) * alpha);
                    tmem_st32(tmem + lane_addr + 256 + q * 32, o);
                }
                tmem_wait_st();
                l *= alpha;
                m_ref = m_new;
            }
            const float m_use = m_ref == -INFINITY ? 0.f : m_ref;
            uint32_t pk[2][32];
            float lsum = 0.f;
#pragma unroll
            for (int q = 0; q < 4; ++q) {
#pragma unroll
                for (int c = 0; c < 32; c += 2) {
                    const float p0 = exp2f(__uint_as_float(sr[q][c]) - m_use);
                    const float p1 = exp2f(__uint_as_float(sr[q][c + 1]) - m_use);
                    lsum += p0 + p1;
                    __nv_bfloat162 h = __floats2bfloat162_rn(p0, p1);
                    pk[q >> 1][(q & 1) * 16 + (c >> 1)] = *reinterpret_cast<uint32_t*>(&h);
                }
            }
            l += lsum;
            tmem_st32(tmem + lane_addr + b * 128, pk[0]);
            tmem_st32(tmem + lane_addr + b * 128 + 32, pk[1]);
            tmem_wait_st();
            tc_fence_before();
            mbar_arrive(&p_full[b]);
        }
        if (ok && nj > 0) ok = mbar_wait(&pv_done[(nj - 1) & 1], ((nj - 1) >> 1) & 1);
        if (!ok) {
            flag_error(p.status, 3);
        } else if (nj > 0) {
            tc_fence_after();
            float o[HD];
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                uint32_t r[32];
                tmem_ld32(tmem + lane_addr + 256 + q * 32, r);
                tmem_wait_ld();
#pragma unroll
                for (int c = 0; c < 32; ++c) o[q * 32 + c] = __uint_as_float(r[c]);
            }
            if (valid) {
                const float inv = l > 0.f ? 1.f / l : 0.f;
                if (p.splits == 1) {
                    __nv_bfloat16* dst = p.out + (int64_t)token * p.o_stride_tok + (int64_t)head * p.o_stride_head;
#pragma unroll
                    for (int v = 0; v < HD / 8; ++v) {
                        uint4 pkt;
                        uint32_t* w = reinterpret_cast<uint32_t*>(&pkt);
#pragma unroll
                        for (int e = 0; e < 4; ++e) {
                            __nv_bfloat162 h = __floats2bfloat162_rn(o[v * 8 + 2 * e] * inv, o[v * 8 + 2 * e + 1] * inv);
                            w[e] = *reinterpret_cast<uint32_t*>(&h);
                        }
                        *reinterpret_cast<uint4*>(dst + v * 8) = pkt;
                    }
                } else {
                    const int64_t prow = ((int64_t)split * p.n_tokens + token) * p.hq + head;
                    float4* dst = reinterpret_cast<float4*>(p.part_o + prow * HD);
#pragma unroll
                    for (int v = 0; v < HD / 4; ++v)
                        dst[v] = make_float4(o[4 * v] * inv, o[4 * v + 1] * inv, o[4 * v + 2] * inv, o[4 * v + 3] * inv);
                    p.part_lse[prow] = l > 0.f ? m_ref + log2f(l) : -INFINITY;
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, kTmemCols);
    }
}

// Merge of the split partials: out = sum_s 2^(lse_s - M) o_s / sum_s 2^(lse_s - M).
__global__ void __launch_bounds__(256)
attn_combine_kernel(const float* __restrict__ part_o, const float* __restrict__ part_lse, int splits, int n_tokens,
                    int hq, __nv_bfloat16* out, int64_t o_stride_tok, int64_t o_stride_head) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t row = (int64_t)blockIdx.x * 8 + warp;
    if (row >= (int64_t)n_tokens * hq) return;
    const int token = (int)(row / hq), head = (int)(row % hq);
    float M = -INFINITY;
    for (int s = 0; s < splits; ++s) M = fmaxf(M, part_lse[(int64_t)s * n_tokens * hq + row]);
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    float wsum = 0.f;
    if (M != -INFINITY) {
        for (int s = 0; s < splits; ++s) {
            const int64_t prow = (int64_t)s * n_tokens * hq + row;
            const float w = exp2f(part_lse[prow] - M);
            const float4 v = reinterpret_cast<const float4*>(part_o + prow * HD)[lane];
            acc.x += w * v.x;
            acc.y += w * v.y;
            acc.z += w * v.z;
            acc.w += w * v.w;
            wsum += w;
        }
    }
    const float inv = wsum > 0.f ? 1.f / wsum : 0.f;
    __nv_bfloat16* dst = out + (int64_t)token * o_stride_tok + (int64_t)head * o_stride_head + lane * 4;
    __nv_bfloat162 a = __floats2bfloat162_rn(acc.x * inv, acc.y * inv);
    __nv_bfloat162 b = __floats2bfloat162_rn(acc.z * inv, acc.w * inv);
    uint2 pkt;
    pkt.x = *reinterpret_cast<uint32_t*>(&a);
    pkt.y = *reinterpret_cast<uint32_t*>(&b);
    *reinterpret_cast<uint2*>(dst) = pkt;
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* f = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
        else
            cudaGetLastError();
    });
    return fn;
}

static int make_map(CUtensorMap* m, const void* base, uint64_t d0, uint64_t d1, uint64_t d2, uint64_t s1_bytes,
                    uint64_t s2_bytes, uint32_t b0, uint32_t b1, uint32_t b2) {
    auto fn = encode_fn();
    if (!fn) return set_error(DDT_ECUDA, "cuTensorMapEncodeTiled is unavailable");
    cuuint64_t dims[3] = {d0, d1, d2};
    cuuint64_t strides[2] = {s1_bytes, s2_bytes};
    cuuint32_t box[3] = {b0, b1, b2};
    cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return set_error(DDT_EINVAL, "cuTensorMapEncodeTiled failed (%d)", (int)r);
    return DDT_OK;
}

struct Plan {
    int group, tpt, n_kt, mtiles, splits;
    size_t ws_bytes;
};

static Plan plan_for(int64_t n_tokens, int64_t hq, int64_t hkv, int64_t past, int sms) {
    Plan pl;
    pl.group = (int)(hq / hkv);
    pl.tpt = BM / pl.group;
    pl.n_kt = (int)ceil_div(past + n_tokens, BN);
    pl.mtiles = (int)ceil_div(n_tokens, pl.tpt);
    int64_t s = (int64_t)sms / (hkv * pl.mtiles);
    if (s < 1) s = 1;
    if (s > pl.n_kt) s = pl.n_kt;
    pl.splits = (int)s;
    size_t o = 256;  // status word
    if (pl.splits > 1) {
        o += sizeof(float) * (size_t)pl.splits * n_tokens * hq * HD;
        o = (o + 255) & ~size_t(255);
        o += sizeof(float) * (size_t)pl.splits * n_tokens * hq;
        o = (o + 255) & ~size_t(255);
    }
    pl.ws_bytes = o;
    return pl;
}

}  // namespace attn
}  // namespace ddt

using namespace ddt;
using namespace ddt::attn;

extern "C" size_t ddt_tree_attention_workspace_size(int64_t n_tokens, int64_t hq, int64_t hkv, int64_t past_length,
                                                    int device) {
    if (n_tokens <= 0 || hq <= 0 || hkv <= 0 || hq % hkv || past_length < 0) return 256;
    const int sms = ddt_sm_count(device);
    return plan_for(n_tokens, hq, hkv, past_length, sms > 0 ? sms : 148).ws_bytes;
}

extern "C" int ddt_tree_attention(const ddt_attention_args* a, void* workspace, size_t workspace_bytes,
                                  ddt_stream_t stream) {
    if (!a) return set_error(DDT_EINVAL, "args is null");
    if (!a->q || !a->k || !a->v || !a->out || !a->visibility) return set_error(DDT_EINVAL, "null tensor pointer");
    if (a->head_dim != HD) return set_error(DDT_EUNSUPPORTED, "head_dim %lld (only 128)", (long long)a->head_dim);
    if (a->n_tokens <= 0 || a->hq <= 0 || a->hkv <= 0 || a->hq % a->hkv)
        return set_error(DDT_EINVAL, "bad head counts / tokens");
    const int64_t group = a->hq / a->hkv;
    if (group > BM || BM % group) return set_error(DDT_EUNSUPPORTED, "GQA group %lld must divide 128", (long long)group);
    if (a->past_length < 0 || a->kv_rows < a->past_length + a->n_tokens)
        return set_error(DDT_EINVAL, "kv_rows %lld < past %lld + n_tokens %lld", (long long)a->kv_rows,
                         (long long)a->past_length, (long long)a->n_tokens);
    if (a->past_length + a->n_tokens >= ((int64_t)1 << 31)) return set_error(DDT_EINVAL, "sequence too long");
    if (a->vis_words < ceil_div(a->n_tokens, 32)) return set_error(DDT_EINVAL, "vis_words too small");
    if (!(a->scale == a->scale) || a->scale <= 0.f) return set_error(DDT_EINVAL, "scale must be positive");
    auto mis = [](const void* ptr) { return reinterpret_cast<uintptr_t>(ptr) % 16 != 0; };
    if (mis(a->q) || mis(a->k) || mis(a->v) || mis(a->out))
        return set_error(DDT_EINVAL, "q/k/v/out must be 16-byte aligned");
    if ((a->q_stride_tok * 2) % 16 || (a->q_stride_head * 2) % 16 || (a->kv_stride_head * 2) % 16 ||
        (a->kv_stride_row * 2) % 16 || (a->o_stride_tok * 2) % 16 || (a->o_stride_head * 2) % 16)
        return set_error(DDT_EINVAL, "strides must be multiples of 8 elements");
    int dev = 0;
    cudaGetDevice(&dev);
    const Plan pl = plan_for(a->n_tokens, a->hq, a->hkv, a->past_length, ddt_sm_count(dev));
    if (!workspace || workspace_bytes < pl.ws_bytes || reinterpret_cast<uintptr_t>(workspace) % 256)
        return set_error(DDT_EWORKSPACE, "attention workspace needs %zu bytes (256-aligned), got %zu", pl.ws_bytes,
                         workspace_bytes);
    CUtensorMap tq, tk, tv;
    int rc = make_map(&tq, a->q, HD, a->hq, a->n_tokens, a->q_stride_head * 2, a->q_stride_tok * 2, 64,
                      (uint32_t)group, (uint32_t)pl.tpt);
    if (rc) return rc;
    rc = make_map(&tk, a->k, HD, a->kv_rows, a->hkv, a->kv_stride_row * 2, a->kv_stride_head * 2, 64, BN, 1);
    if (rc) return rc;
    rc = make_map(&tv, a->v, HD, a->kv_rows, a->hkv, a->kv_stride_row * 2, a->kv_stride_head * 2, 64, BN, 1);
    if (rc) return rc;
    static std::once_flag attr_once;
    static cudaError_t attr_err = cudaSuccess;
    std::call_once(attr_once, [] {
        attr_err = cudaFuncSetAttribute(tree_attn_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemBytes);
    });
    if (attr_err != cudaSuccess) return set_error(DDT_ECUDA, "cudaFuncSetAttribute: %s", cudaGetErrorString(attr_err));
    unsigned char* ws = static_cast<unsigned char*>(workspace);
    Params p;
    p.n_tokens = (int)a->n_tokens;
    p.hq = (int)a->hq;
    p.hkv = (int)a->hkv;
    p.group = pl.group;
    p.tokens_per_tile = pl.tpt;
    p.past = (int)a->past_length;
    p.n_kt = pl.n_kt;
    p.splits = pl.splits;
    p.vis = a->visibility;
    p.vis_words = (int)a->vis_words;
    p.scale_log2 = a->scale * 1.4426950408889634f;
    p.out = static_cast<__nv_bfloat16*>(a->out);
    p.o_stride_tok = a->o_stride_tok;
    p.o_stride_head = a->o_stride_head;
    p.status = reinterpret_cast<int*>(ws);
    p.part_o = nullptr;
    p.part_lse = nullptr;
    if (pl.splits > 1) {
        size_t o = 256;
        p.part_o = reinterpret_cast<float*>(ws + o);
        o += sizeof(float) * (size_t)pl.splits * a->n_tokens * a->hq * HD;
        o = (o + 255) & ~size_t(255);
        p.part_lse = reinterpret_cast<float*>(ws + o);
    }
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    dim3 grid((unsigned)pl.splits, (unsigned)pl.mtiles, (unsigned)a->hkv);
    tree_attn_kernel<<<grid, kThreads, kSmemBytes, st>>>(tq, tk, tv, p);
    rc = check_launch("tree_attn_kernel");
    if (rc) return rc;
    if (pl.splits > 1) {
        const int64_t rows = a->n_tokens * a->hq;
        attn_combine_kernel<<<(unsigned)ceil_div(rows, 8), 256, 0, st>>>(p.part_o, p.part_lse, pl.splits,
                                                                         (int)a->n_tokens, (int)a->hq, p.out,
                                                                         a->o_stride_tok, a->o_stride_head);
        rc = check_launch("attn_combine_kernel");
    }
    return rc;
}
