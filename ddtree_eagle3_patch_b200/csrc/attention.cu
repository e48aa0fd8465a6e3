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
    const int64_t* key_lo;   // sliding window: first visible prefix key per token, or null
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

// First visible prefix key of a row under a sliding window, clamped to
// [0, past]: prefix keys before it are hidden (the reference's
// sliding_attention mask, ddtree.py:276-283).  Without a window, 0.
__device__ __forceinline__ int row_key_lo(const int64_t* key_lo, int token, bool row_valid, int past) {
    if (!key_lo || !row_valid) return 0;
    const int64_t lo = __ldg(key_lo + token);
    return lo <= 0 ? 0 : (lo >= past ? past : (int)lo);
}

// Window mask of keys k0 .. k0+31: bit c is clear for a prefix key
// (k0 + c < past) before `lo`; every other key keeps its bit.
__device__ __forceinline__ uint32_t window_bits(int k0, int lo, int past) {
    const int d = lo - k0;
    uint32_t w = d <= 0 ? 0xffffffffu : (d >= 32 ? 0u : (0xffffffffu << d));
    const int t = past - k0;
    if (t <= 0) return 0xffffffffu;
    if (t < 32) w |= 0xffffffffu << t;
    return w;
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
        const int lo = row_key_lo(p.key_lo, token, valid, p.past);
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
                uint32_t vb = vis_bits(vrow, p.vis_words, u_base + q * 32, p.n_tokens, valid);
                if (lo > 0) vb &= window_bits(p.past + u_base + q * 32, lo, p.past);
#pragma unroll
                for (int c = 0; c < 32; ++c) {
                    float s = __uint_as_float(sr[q][c]) * p.scale_log2;
                    s = (vb >> c) & 1u ? s : -INFINITY;
                    sr[q][c] = __float_as_uint(s);
                    mx = fmaxf(mx, s);
                }
            }
            const float m_new = fmaxf(m_ref, mx);
            // the O rescale reads and writes TMEM with warp-collective
            // tcgen05.ld / st, so the warp takes it together when any of its
            // rows needs it; the other rows scale by exactly 1
            const bool grow = jj > 0 && m_new > m_ref + 8.0f;
            if (jj == 0) {
                m_ref = m_new;
            } else if (__any_sync(__activemask(), grow)) {
                const float alpha = grow ? exp2f(m_ref - m_new) : 1.f;
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
                if (grow) {
                    l *= alpha;
                    m_ref = m_new;
                }
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
// Split-key kernel: one CTA per (key split, M-tile pair, KV head), holding at
// most two key tiles of 128 keys and up to two M tiles of its KV head.
//
// The rows of a KV head are cut into 128-row M tiles, taken two at a time
// (tiles A and B, one softmax warpgroup each), plus a tail of <= 4 rows (one
// token of a group of <= 4 heads) with its own warpgroup.  The tail's two
// products run transposed on the tensor core with N = 16 rows (S_t^T = K Q_t^T,
// O_t^T = V^T P_t^T), so each of its threads owns one key, then one dim;
// its softmax is column-wise on CUDA cores.  Every load is
// issued when the CTA starts; the MMA warp then issues the products in the
// order their operands become ready, and every barrier completes exactly
// once, so each wait is on parity 0.
//
//   warps 0-3    softmax + epilogue of M tile A (TMEM lane = row)
//   warps 4-7    softmax + epilogue of M tile B
//   warps 8-11   the tail rows
//   warp 12      TMEM owner; runs the load and MMA schedule in step, one
//                elected lane issuing each TMA copy and tcgen05.mma
//                (warps 13-15 only complete the warpgroup so registers can
//                move to the softmax warpgroups)
//
// Shared memory: Q_A, Q_B, K_0, K_1, V_0, V_1 (32 KB each), the tail's Q and
// P tiles and its reductions.  P of a main tile goes to shared memory (the
// P.V product reads it as an SS operand) into a slot whose last reader is
// done: P(A,0) -> Q_A, P(B,0) -> Q_B, P(A,1) -> K_0, P(B,1) -> K_1.  Since P
// does not stay in TMEM, an S buffer is free as soon as its softmax has
// loaded it.
// TMEM columns: S(A,0) then O_A at 0, S(B,0) then O_B at 128, S(A,1) at 256,
// S(B,1) at 384.  S_t^T of the tail's key tiles takes columns 128 + 16 j
// between B's load of S(B,0) and P.V(B,0), issued after the four main S
// products; O_t^T takes 256 + 16 j once S(A,1) is loaded.  The two key tiles of a main row merge
// online (lazy rescaling of O); the tail's tiles merge at the end.
// ---------------------------------------------------------------------------
namespace split {

constexpr int kThreads = 512;
constexpr uint32_t kSlot = 2 * kHalf;                 // 32 KB
constexpr uint32_t kQA = 0, kQB = kSlot, kK0 = 2 * kSlot, kK1 = 3 * kSlot, kV0 = 4 * kSlot, kV1 = 5 * kSlot;
constexpr uint32_t kQT = 6 * kSlot;                   // tail Q tile, 16 rows x 128 dims: two 2 KB halves
constexpr uint32_t kPT = kQT + 4096;                  // tail P(j): 16 rows x 128 keys bf16 (K-major, 128-byte swizzle), 4 KB each
constexpr uint32_t kRed = kPT + 8192;                 // tail reductions and per-tile statistics
constexpr uint32_t kBar = kRed + 4096;
constexpr uint32_t kSmemBytes = kBar + 512 + 1024;
constexpr uint32_t kTHalf = 16 * 128;
constexpr uint32_t kColA = 0, kColB = 128, kCol1 = 256, kColT = 384;
constexpr uint32_t kIdescPVs = idesc_bf16_f32(BM, HD, false, true);   // P K-major from shared memory
constexpr uint32_t kIdescQKt = idesc_bf16_f32(128, 16, false, false); // tail: S_t^T = K Q_t^T
constexpr uint32_t kIdescPVt = idesc_bf16_f32(128, 16, true, false);  // tail: O_t^T = V^T P_t^T (V^T MN-major)
constexpr float kFix = 16777216.f;                    // 2^24: fixed-point scale of tail probabilities

struct Params {
    int n_tokens, hq, hkv, group, tpt, past, n_kt, tpc, splits;
    int n_mt, n_groups, tail_rows, tail_token0;
    const uint32_t* vis;
    int vis_words;
    float scale_log2;
    __nv_bfloat16* out;
    int64_t o_stride_tok, o_stride_head;
    __nv_bfloat16* part_o;
    float* part_lse;
    int* status;
    const int64_t* key_lo;   // sliding window: first visible prefix key per token, or null
    // Run-time prefix length, or null.  When set, `past` and `n_kt` above
    // describe the largest prefix the launch covers (the grid is planned for
    // it) and the kernel reads the actual prefix here, clamped to [0, past]:
    // CTAs whose key tiles lie past the actual keys exit at once.
    const int32_t* past_dev;
    // Keys [0, stable) are written by no kernel still running on the stream:
    // K tiles wholly below it load before griddepcontrol.wait.  Read from
    // stable_dev at run time when set (clamped to [0, past]), else `stable`.
    const int32_t* stable_dev;
    int stable;
};

// Prefix length and key-tile count of this launch (see Params::past_dev).
__device__ __forceinline__ void runtime_keys(const Params& p, int& past, int& n_kt) {
    past = p.past;
    n_kt = p.n_kt;
    if (p.past_dev) {
        const int v = __ldg(p.past_dev);
        past = v < 0 ? 0 : (v > p.past ? p.past : v);
        n_kt = (past + p.n_tokens + BN - 1) / BN;
    }
}

// Barriers; each completes exactly once per CTA.
enum : int {
    bQ = 0,
    bK0 = 1,       // + j
    bV0 = 3,       // + j
    bS0 = 5,       // + 2 * slot + j      (S ready)
    bFreeQA = 9,   // every reader of Q_A done (MMA commit)
    bFreeK0 = 10,  // every reader of K_0 done (MMA commit)
    bFreeQB = 11,
    bFreeK1 = 12,
    bP0 = 13,      // + 2 * slot + j      (P in shared memory)
    bPV0 = 17,     // + 2 * slot + j      (P.V complete)
    bDrain = 21,
    bX1 = 22,      // S(A,1) loaded: its TMEM block may take the tail's P.V
    bPt0 = 23,     // + j                 (tail P in shared memory)
    bPVt = 25,     // the tail's P.V products complete
    bSt = 26,      // the tail's S products complete
    bStLd = 27,    // the tail has loaded S_t: P.V(B,0) may take its TMEM block
    bX0B = 28,     // S(B,0) loaded: its TMEM block may take the tail's S products
    kNumBars = 29
};

// P(slot, j) goes to the slot freed earliest for it: tile 0's P to the
// M tile's own Q slot (free once both its S products completed), tile 1's
// P to a K slot (free once every S product reading it completed).
__device__ __forceinline__ uint32_t p_slot(int slot, int j) {
    return j == 0 ? (slot ? kQB : kQA) : (slot ? kK1 : kK0);
}
__device__ __forceinline__ int free_bar(int slot, int j) {
    return j == 0 ? (slot ? bFreeQB : bFreeQA) : (slot ? bFreeK1 : bFreeK0);
}
__device__ __forceinline__ float warp_max(float v) {
    float m;
    asm volatile("redux.sync.max.f32 %0, %1, 0xffffffff;" : "=f"(m) : "f"(v));
    return m;
}
__device__ __forceinline__ uint32_t warp_sum_u32(uint32_t v) {
    uint32_t s;
    asm volatile("redux.sync.add.u32 %0, %1, 0xffffffff;" : "=r"(s) : "r"(v));
    return s;
}

// Merge of one row's split partials: bf16 partials normalised by their own
// sum, weights 2^(lse_s - max).  One warp: lane s loads split s's
// log-sum-exp while every lane loads its 4 dims of up to CHUNK splits, all
// in one batch of independent loads (neither depends on the max), so a row
// costs one memory round trip per CHUNK splits.  Loads bypass L1: the partials
// were written by other SMs during this launch.
template <int CHUNK>
__device__ __forceinline__ void merge_row(const __nv_bfloat16* part_o, const float* part_lse, int splits,
                                          int64_t split_stride, int64_t base, int lane, __nv_bfloat16* dst) {
    float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f, wsum = 0.f, M = -INFINITY;
    for (int s0 = 0; s0 < splits; s0 += CHUNK) {
        const int ns = min(CHUNK, splits - s0);
        const float l = lane < ns ? __ldcg(part_lse + (s0 + lane) * split_stride + base) : -INFINITY;
        uint2 raw[CHUNK];
#pragma unroll
        for (int i = 0; i < CHUNK; ++i)
            raw[i] = i < ns ? __ldcg(reinterpret_cast<const uint2*>(part_o + ((s0 + i) * split_stride + base) * HD) + lane)
                            : make_uint2(0u, 0u);
        float m;
        asm volatile("redux.sync.max.f32 %0, %1, 0xffffffff;" : "=f"(m) : "f"(l));
        const float m_new = fmaxf(M, m);
        if (m_new == -INFINITY) continue;
        // rescale what earlier passes accumulated (only with more than CHUNK splits)
        const float c = M == -INFINITY ? 0.f : exp2f(M - m_new);
        a0 *= c;
        a1 *= c;
        a2 *= c;
        a3 *= c;
        wsum *= c;
        M = m_new;
        const float w_lane = l == -INFINITY ? 0.f : exp2f(l - M);
#pragma unroll
        for (int i = 0; i < CHUNK; ++i) {
            if (i < ns) {
                const float w = __shfl_sync(DDT_FULL_MASK, w_lane, i);
                const __nv_bfloat162 x = *reinterpret_cast<const __nv_bfloat162*>(&raw[i].x);
                const __nv_bfloat162 y = *reinterpret_cast<const __nv_bfloat162*>(&raw[i].y);
                a0 = fmaf(w, __low2float(x), a0);
                a1 = fmaf(w, __high2float(x), a1);
                a2 = fmaf(w, __low2float(y), a2);
                a3 = fmaf(w, __high2float(y), a3);
                wsum += w;
            }
        }
    }
    const float inv = wsum > 0.f ? 1.f / wsum : 0.f;
    __nv_bfloat162 a = __floats2bfloat162_rn(a0 * inv, a1 * inv);
    __nv_bfloat162 b2 = __floats2bfloat162_rn(a2 * inv, a3 * inv);
    uint2 pkt;
    pkt.x = *reinterpret_cast<uint32_t*>(&a);
    pkt.y = *reinterpret_cast<uint32_t*>(&b2);
    *reinterpret_cast<uint2*>(dst + lane * 4) = pkt;
}

// Eight K16 steps of one product, fully unrolled: the k-step offsets are
// compile-time constants in 16-byte units (hi per group of four steps, lo
// per step), so each step costs one 64-bit add and the MMA; a single
// issuing thread can then keep pace with the tensor core.  A 128-row K-major
// tile has (hi, lo) = (1024, 2), a 16-row K-major tile (128, 2) and the
// MN-major V tile (512, 128).  A descriptor advances by adding offset >> 4
// (shared addresses fit its 14-bit field).
template <uint32_t AH, uint32_t AL, uint32_t BH, uint32_t BL>
__device__ __forceinline__ void mma8(uint32_t d, uint64_t ad, uint64_t bd, uint32_t idesc, uint32_t acc0) {
#pragma unroll
    for (int kk = 0; kk < 8; ++kk)
        mma_ss(d, ad + (uint64_t)((kk >> 2) * AH + (kk & 3) * AL), bd + (uint64_t)((kk >> 2) * BH + (kk & 3) * BL),
               idesc, kk == 0 ? acc0 : 1u);
}

// Epilogue of one 128-row M tile.  Each thread owns one row of O in TMEM.
// Rows are normalised, packed to bf16 and staged in the tile's own last P
// slot (dead once its last P.V completed) with the 16-byte chunks of row r
// XOR-swizzled by r & 15; then each warp writes two whole rows per
// instruction with coalesced 16-byte stores.  One split: rows go to
// out[token][head]; several: to the bf16 partial part_o[split][g][r]
// (r = row within the KV head) with its log-sum-exp in part_lse.
__device__ __forceinline__ void tile_epilogue(const Params& p, uint32_t o_col, unsigned char* stage, int row, int qw,
                                              int lane, int mt, int split, int g, float inv, float lse, int bar_id) {
    const int rows_head = p.group * p.n_tokens;
    {
        uint32_t r[4][32];
#pragma unroll
        for (int q = 0; q < 4; ++q) tmem_ld32(o_col + q * 32, r[q]);
        tmem_wait_ld();
#pragma unroll
        for (int q = 0; q < 4; ++q) {
#pragma unroll
            for (int v = 0; v < 4; ++v) {
                uint4 pkt;
                uint32_t* w = reinterpret_cast<uint32_t*>(&pkt);
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    __nv_bfloat162 h = __floats2bfloat162_rn(__uint_as_float(r[q][v * 8 + 2 * e]) * inv,
                                                             __uint_as_float(r[q][v * 8 + 2 * e + 1]) * inv);
                    w[e] = *reinterpret_cast<uint32_t*>(&h);
                }
                const int chunk = q * 4 + v;
                *reinterpret_cast<uint4*>(stage + row * 256 + ((chunk ^ (row & 15)) << 4)) = pkt;
            }
        }
    }
    const int rg = mt * BM + row;
    if (p.splits > 1 && rg < rows_head) p.part_lse[((int64_t)split * p.hkv + g) * rows_head + rg] = lse;
    named_bar_sync(bar_id, 128);
    const int chunk = lane & 15;
#pragma unroll 4
    for (int it = 0; it < 16; ++it) {
        const int rl = qw * 32 + it * 2 + (lane >> 4);
        const int rgl = mt * BM + rl;
        if (rgl >= rows_head) continue;
        const uint4 v = *reinterpret_cast<const uint4*>(stage + rl * 256 + ((chunk ^ (rl & 15)) << 4));
        __nv_bfloat16* dst;
        if (p.splits == 1) {
            const int token = rgl / p.group, head = g * p.group + rgl % p.group;
            dst = p.out + (int64_t)token * p.o_stride_tok + (int64_t)head * p.o_stride_head;
        } else {
            dst = p.part_o + (((int64_t)split * p.hkv + g) * rows_head + rgl) * HD;
        }
        *reinterpret_cast<uint4*>(dst + chunk * 8) = v;
    }
}

// kWindow: sliding-window layer (p.key_lo set).  A separate instance, so the
// ordinary layers' code, the transposed tail's above all, carries no window
// test.
template <bool kWindow>
__global__ void __launch_bounds__(kThreads, 1)
tree_attn_split_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tqt,
                       const __grid_constant__ CUtensorMap tk, const __grid_constant__ CUtensorMap tv,
                       const Params p) {
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    unsigned char* smem = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kBar);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + kNumBars);
    float* wmax = reinterpret_cast<float*>(smem + kRed);   // [j][4 warps][16]
    float* wsum = wmax + 128;                               // [j][4 warps][16]
    float* tmax = wsum + 128;                               // [j][16] column max of tile j
    float* wts = tmax + 32;                                 // [j][16] merge weights, then [16] lse

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int split = blockIdx.x, grp = blockIdx.y, g = blockIdx.z;
    int past, n_kt;
    runtime_keys(p, past, n_kt);
    const int kt0 = split * p.tpc;
    const int nj = min(p.tpc, n_kt - kt0);       // 1 or 2
    if (nj <= 0) return;                         // past the run-time keys (whole CTA, before any barrier)
    const int mA = 2 * grp, mB = 2 * grp + 1;
    const bool hasA = mA < p.n_mt, hasB = mB < p.n_mt;
    const bool hasT = grp == p.n_groups - 1 && p.tail_rows > 0;

    if (threadIdx.x == 0) {
        for (int i = 0; i < kNumBars; ++i) {
            const uint32_t count =
                ((i >= bP0 && i < bP0 + 4) || i == bX1 || i == bX0B || i == bPt0 || i == bPt0 + 1 || i == bStLd) ? 128 : 1;
            mbar_init(&bars[i], count);
        }
        fence_mbar_init();
    }
    if (warp == 12) {
        tmem_alloc(tmem_slot, 512);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const uint32_t s_addr = smem_u32(smem);
    // every CTA of this grid is resident: the next kernel in the stream may be
    // scheduled as SMs free up (it waits for this grid before reading our output)
    griddep_launch_dependents();

    // 512 threads x 128 registers at launch: warpgroup 2 (tail) gives 88 per
    // thread, warpgroup 3 (loads and MMA issue) 104, the two softmax
    // warpgroups take 96 each (224: a whole 128-column row of S without
    // spilling).  Each
    // role's setmaxnreg sits in its own branch so the compiler sizes that
    // role's code to the new limit; the code after the branches is trivial.
    if (warp >= 12) {
        asm volatile("setmaxnreg.dec.sync.aligned.u32 24;\n" ::: "memory");
        if (warp == 12) {
            // The whole warp runs this branch in step, so the operand
            // descriptors are warp-uniform values; one elected lane issues
            // each TMA copy, MMA and commit.
            const bool leader = elect_one_sync();
            // ------------------------------------------------------------ loads
            // K tiles that hold only stable keys (Params::stable) load before
            // the preceding kernel in the stream has finished; Q and every
            // other K tile load after it.
            // V is not needed before the first softmax ends: its tiles load
            // once Q and K_0 have landed and the first S products are queued,
            // so the S products' operands are not queued behind V in the
            // memory system.
            const uint64_t kv_policy = policy_evict_first();
            auto load_k = [&](int j) {
                const int key0 = (kt0 + j) * BN;
                unsigned char* kb = smem + (j ? kK1 : kK0);
                mbar_arrive_expect_tx(&bars[bK0 + j], kSlot);
                tma_load_3d_hint(kb, &tk, 0, key0, g, &bars[bK0 + j], kv_policy);
                tma_load_3d_hint(kb + kHalf, &tk, 64, key0, g, &bars[bK0 + j], kv_policy);
            };
            auto load_v = [&](int j) {
                const int key0 = (kt0 + j) * BN;
                unsigned char* vb = smem + (j ? kV1 : kV0);
                mbar_arrive_expect_tx(&bars[bV0 + j], kSlot);
                tma_load_3d_hint(vb, &tv, 0, key0, g, &bars[bV0 + j], kv_policy);
                tma_load_3d_hint(vb + kHalf, &tv, 64, key0, g, &bars[bV0 + j], kv_policy);
            };
            int stable = p.stable;
            if (p.stable_dev) stable = __ldg(p.stable_dev);
            stable = stable < 0 ? 0 : (stable > past ? past : stable);
            auto prefix_only = [&](int j) { return (kt0 + j + 1) * BN <= stable; };
            if (leader) {
                prefetch_tmap(&tk);
                prefetch_tmap(&tv);
                for (int j = 0; j < nj; ++j)
                    if (prefix_only(j)) load_k(j);
            }
            __syncwarp();
            griddep_wait();
            if (leader) {
                prefetch_tmap(&tq);
                const uint32_t qbytes = (hasA ? kSlot : 0) + (hasB ? kSlot : 0) + (hasT ? 2 * kTHalf : 0);
                mbar_arrive_expect_tx(&bars[bQ], qbytes);
                if (hasA) {
                    tma_load_3d(smem + kQA, &tq, 0, g * p.group, mA * p.tpt, &bars[bQ]);
                    tma_load_3d(smem + kQA + kHalf, &tq, 64, g * p.group, mA * p.tpt, &bars[bQ]);
                }
                if (hasB) {
                    tma_load_3d(smem + kQB, &tq, 0, g * p.group, mB * p.tpt, &bars[bQ]);
                    tma_load_3d(smem + kQB + kHalf, &tq, 64, g * p.group, mB * p.tpt, &bars[bQ]);
                }
                if (hasT) {
                    prefetch_tmap(&tqt);
                    tma_load_3d(smem + kQT, &tqt, 0, g * p.group, p.tail_token0, &bars[bQ]);
                    tma_load_3d(smem + kQT + kTHalf, &tqt, 64, g * p.group, p.tail_token0, &bars[bQ]);
                }
                for (int j = 0; j < nj; ++j)
                    if (!prefix_only(j)) load_k(j);
            }
            __syncwarp();
            // ------------------------------------------------------------ MMA issue
            auto desc = [&](uint32_t off, uint32_t lbo) { return smem_desc_sw128(s_addr + off, lbo, 1024); };
            // Issue order follows the order operands become ready: S products as
            // K tiles land, then each P.V as its P is written (main tiles before
            // the tail, whose result is needed last).  Waits suspend in hardware.
            auto s_main = [&](int sl, int j, uint32_t col) {
                if (leader) {
                    mma8<1024, 2, 1024, 2>(tmem + col, desc(sl ? kQB : kQA, 16), desc(j ? kK1 : kK0, 16), kIdescQK, 0u);
                    mma_commit(&bars[bS0 + 2 * sl + j]);
                }
            };
            auto pv_main = [&](int sl, int j) {
                if (leader) {
                    mma8<1024, 2, 512, 128>(tmem + (sl ? kColB : kColA), desc(p_slot(sl, j), 16), desc(j ? kV1 : kV0, kHalf),
                                            kIdescPVs, j > 0 ? 1u : 0u);
                    mma_commit(&bars[bPV0 + 2 * sl + j]);
                }
            };
            auto commit = [&](int b) {
                if (leader) mma_commit(&bars[b]);
            };
            auto wait = [&](int b) -> bool {
                const bool r = mbar_wait(&bars[b], 0);
                tc_fence_after();
                return __all_sync(DDT_FULL_MASK, r);
            };
            // the tail's S_t^T(j) = K_j Q_t^T into S(B,0)'s TMEM block
            auto s_tail = [&](int j) {
                if (leader)
                    mma8<1024, 2, 128, 2>(tmem + kColB + 16 * j, desc(j ? kK1 : kK0, 16), desc(kQT, 16), kIdescQKt, 0u);
            };
            bool ok = wait(bQ) && wait(bK0);
            if (ok) {
                if (hasA) s_main(0, 0, kColA);
                if (hasB) s_main(1, 0, kColB);
            }
            if (leader)   // issued even after a failed wait, so the drain below completes
                for (int j = 0; j < nj; ++j) load_v(j);
            if (ok && nj == 1) {
                commit(bFreeQA);
                commit(bFreeQB);
            }
            if (ok && nj > 1) {
                ok = wait(bK0 + 1);
                if (ok) {
                    if (hasA) s_main(0, 1, kCol1);
                    commit(bFreeQA);
                    if (hasB) s_main(1, 1, kColT);
                    commit(bFreeQB);
                }
            }
            // the tail's scores last: they are needed last, and every main S
            // product they would delay gates a softmax
            if (ok && hasT) {
                if (hasB) ok = wait(bX0B);
                if (ok) {
                    s_tail(0);
                    if (nj > 1) s_tail(1);
                    commit(bSt);
                }
            }
            if (ok) {
                commit(bFreeK0);
                if (nj > 1) commit(bFreeK1);
            }
            if (ok) ok = wait(bV0);
            if (ok && hasA) {
                ok = wait(bP0 + 0);
                if (ok) pv_main(0, 0);
            }
            if (ok && hasB) {
                ok = wait(bP0 + 2) && (!hasT || wait(bStLd));   // the tail has loaded S_t from O_B's columns
                if (ok) pv_main(1, 0);
            }
            if (ok && hasT) {
                // the tail's O_t^T = V^T P_t^T into S(A,1)'s TMEM block, once free
                if (hasA && nj > 1) ok = wait(bX1);
                for (int j = 0; j < nj && ok; ++j) {
                    ok = wait(bV0 + j) && wait(bPt0 + j);
                    if (ok && leader)
                        mma8<512, 128, 128, 2>(tmem + kCol1 + 16 * j, desc(j ? kV1 : kV0, kHalf), desc(kPT + j * 4096, 16),
                                               kIdescPVt, 0u);
                }
                if (ok) commit(bPVt);
            }
            if (ok && nj > 1) {
                ok = wait(bV0 + 1);
                if (ok && hasA) {
                    ok = wait(bP0 + 1);
                    if (ok) pv_main(0, 1);
                }
                if (ok && hasB) {
                    ok = wait(bP0 + 3);
                    if (ok) pv_main(1, 1);
                }
            }
            __syncwarp();
            if (!ok && leader) flag_error(p.status, 2);
            // drain: nothing this warp issued may still be in flight when the CTA exits
            if (leader) mma_commit(&bars[bDrain]);
            __syncwarp();
            mbar_wait(&bars[bDrain], 0);
            for (int j = 0; j < nj; ++j) {
                mbar_wait(&bars[bK0 + j], 0);
                mbar_wait(&bars[bV0 + j], 0);
            }
            mbar_wait(&bars[bQ], 0);
        }
    } else if (warp < 8) {
        asm volatile("setmaxnreg.inc.sync.aligned.u32 224;\n" ::: "memory");
        griddep_wait();   // nothing global is read or written before the preceding kernel is done
        // ---------------------------------------------------------------- softmax of M tile A / B
        const int slot = warp >> 2;
        const bool has = slot == 0 ? hasA : hasB;
        const int qw = warp & 3;
        const int row = qw * 32 + lane;
        const uint32_t lane_addr = (uint32_t)(qw * 32) << 16;
        const int mt = slot == 0 ? mA : mB;
        const int rows_head = p.group * p.n_tokens;
        const int rg = mt * BM + row;
        const bool valid = rg < rows_head;
        const int token = rg / p.group;
        const uint32_t o_col = tmem + lane_addr + (slot ? kColB : kColA);
        float m_ref = -INFINITY, l = 0.f;
        bool ok = true;
        if (has) {
            const uint32_t* vrow = valid ? p.vis + (int64_t)token * p.vis_words : p.vis;
            const int lo = kWindow ? row_key_lo(p.key_lo, token, valid, past) : 0;
            const float sl2 = p.scale_log2;
            for (int j = 0; j < nj; ++j) {
                const uint32_t s_col =
                    tmem + lane_addr + (j == 0 ? (slot ? kColB : kColA) : (slot == 0 ? kCol1 : kColT));
                ok = ok && mbar_wait(&bars[bS0 + 2 * slot + j], 0);
                tc_fence_after();
                const int u0 = (kt0 + j) * BN - past;
                // tiles reaching into the tree, and under a sliding window the
                // tiles holding prefix keys before this row's first visible one
                const bool masked = u0 + BN > 0 || (kWindow && u0 + past < lo);
                uint32_t r[4][32];
                uint32_t vb[4];
                if (ok) {
#pragma unroll
                    for (int q = 0; q < 4; ++q) tmem_ld32(s_col + q * 32, r[q]);
#pragma unroll
                    for (int q = 0; q < 4; ++q)
                        vb[q] = !masked ? 0xffffffffu
                                : kWindow ? vis_bits(vrow, p.vis_words, u0 + q * 32, p.n_tokens, valid) &
                                                window_bits(past + u0 + q * 32, lo, past)
                                          : vis_bits(vrow, p.vis_words, u0 + q * 32, p.n_tokens, valid);
                    tmem_wait_ld();
                }
                if (hasT && slot == 0 && j == 1) {   // S(A,1)'s TMEM block may now take the tail's P.V
                    tc_fence_before();
                    mbar_arrive(&bars[bX1]);
                }
                if (hasT && slot == 1 && j == 0) {   // S(B,0)'s TMEM block may now take the tail's S
                    tc_fence_before();
                    mbar_arrive(&bars[bX0B]);
                }
                if (!ok) break;
                float mk[8];
#pragma unroll
                for (int e = 0; e < 8; ++e) mk[e] = -INFINITY;
                if (masked) {
#pragma unroll
                    for (int q = 0; q < 4; ++q)
#pragma unroll
                        for (int c = 0; c < 32; ++c)
                            mk[c & 7] = fmaxf(mk[c & 7], ((vb[q] >> c) & 1u) ? __uint_as_float(r[q][c]) : -INFINITY);
                } else {
#pragma unroll
                    for (int q = 0; q < 4; ++q)
#pragma unroll
                        for (int c = 0; c < 32; ++c) mk[c & 7] = fmaxf(mk[c & 7], __uint_as_float(r[q][c]));
                }
                const float mx = fmaxf(fmaxf(fmaxf(mk[0], mk[1]), fmaxf(mk[2], mk[3])),
                                       fmaxf(fmaxf(mk[4], mk[5]), fmaxf(mk[6], mk[7])));
                const float m_new = fmaxf(m_ref, mx * sl2);
                // rare: a row's running max grew by more than 2^8; O is
                // rescaled once P.V of tile 0 is done.  tcgen05.ld / st are
                // warp-collective, so the warp takes the rescale together when
                // any of its rows needs it; the other rows scale by exactly 1
                const bool grow = j > 0 && m_new > m_ref + 8.0f;
                if (j == 0) {
                    m_ref = m_new;
                } else if (__any_sync(__activemask(), grow)) {
                    const float alpha = grow ? ex2_approx(m_ref - m_new) : 1.f;
                    ok = mbar_wait(&bars[bPV0 + 2 * slot], 0);
                    if (!ok) break;
                    tc_fence_after();
#pragma unroll
                    for (int q = 0; q < 4; ++q) {
                        uint32_t o[32];
                        tmem_ld32(o_col + q * 32, o);
                        tmem_wait_ld();
#pragma unroll
                        for (int c = 0; c < 32; ++c) o[c] = __float_as_uint(__uint_as_float(o[c]) * alpha);
                        tmem_st32(o_col + q * 32, o);
                    }
                    tmem_wait_st();
                    tc_fence_before();
                    if (grow) {
                        l *= alpha;
                        m_ref = m_new;
                    }
                }
                const float neg_m = m_ref == -INFINITY ? 0.f : -m_ref;
                ok = mbar_wait(&bars[free_bar(slot, j)], 0);
                if (!ok) break;
                unsigned char* pdst = smem + p_slot(slot, j) + (row >> 3) * 1024 + (row & 7) * 128;
                float ls[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    uint32_t pk[16];
#pragma unroll
                    for (int c = 0; c < 32; c += 2) {
                        float p0 = ex2_approx(fmaf(__uint_as_float(r[q][c]), sl2, neg_m));
                        float p1 = ex2_approx(fmaf(__uint_as_float(r[q][c + 1]), sl2, neg_m));
                        if (masked) {
                            p0 = ((vb[q] >> c) & 1u) ? p0 : 0.f;
                            p1 = ((vb[q] >> (c + 1)) & 1u) ? p1 : 0.f;
                        }
                        ls[(c >> 1) & 3] += p0 + p1;
                        __nv_bfloat162 h = __floats2bfloat162_rn(p0, p1);
                        pk[c >> 1] = *reinterpret_cast<uint32_t*>(&h);
                    }
                    // keys 32q .. 32q+31: half q >> 1, 16-byte chunks (q & 1) * 4 .. + 3
                    unsigned char* hb = pdst + (q >> 1) * kHalf;
#pragma unroll
                    for (int v = 0; v < 4; ++v) {
                        const int chunk = (q & 1) * 4 + v;
                        *reinterpret_cast<uint4*>(hb + ((chunk ^ (row & 7)) << 4)) =
                            make_uint4(pk[4 * v], pk[4 * v + 1], pk[4 * v + 2], pk[4 * v + 3]);
                    }
                }
                l += (ls[0] + ls[1]) + (ls[2] + ls[3]);
                fence_proxy_async_smem();
                mbar_arrive(&bars[bP0 + 2 * slot + j]);
            }
            if (ok) ok = mbar_wait(&bars[bPV0 + 2 * slot + nj - 1], 0);
            if (!ok) flag_error(p.status, 3);
            tc_fence_after();
            // every thread of the warpgroup reaches the named barrier inside
            if (ok)
                tile_epilogue(p, o_col, smem + p_slot(slot, nj - 1), row, qw, lane, mt, split, g,
                              l > 0.f ? 1.f / l : 0.f, l > 0.f ? m_ref + log2f(l) : -INFINITY, 2 + slot);
            else
                named_bar_sync(2 + slot, 128);
        }
    } else {
        asm volatile("setmaxnreg.dec.sync.aligned.u32 40;\n" ::: "memory");
        griddep_wait();
        // ---------------------------------------------------------------- tail rows, warps 8-11
        // The <= 4 tail rows (one token of a group of <= 4 heads) against this
        // CTA's key tiles.  Both products are transposed tensor-core MMAs with
        // 16 columns: thread k reads key k's scores of every tail row from
        // S_t^T, runs the softmax column-wise (column max and sum by warp-wide
        // redux and one exchange across the 4 warps), writes P_t as the B
        // operand of O_t^T = V^T P_t^T, and finally reads dim k of every tail
        // row from O_t^T; the key tiles merge there.
        const int tw = warp - 8;
        const int k = tw * 32 + lane;
        if (hasT) {
            const int nt = p.tail_rows;
            const float sl2 = p.scale_log2;
            // rows 4..15 of both P_t tiles are zero (the product runs on 16 rows)
            for (int i = k; i < 2 * 4096 / 16; i += 128) {
                const int row = (i >> 3) & 15;
                if (row >= 4) reinterpret_cast<uint4*>(smem + kPT)[i] = make_uint4(0u, 0u, 0u, 0u);
            }
            // S_t^T(j) in TMEM: lane = key k, column 16 j + r = tail row r
            float sc0[4] = {0.f, 0.f, 0.f, 0.f}, sc1[4] = {0.f, 0.f, 0.f, 0.f};
            bool ok = __all_sync(DDT_FULL_MASK, mbar_wait(&bars[bSt], 0));
            tc_fence_after();
            if (ok) {
                const uint32_t lane_addr = (uint32_t)(tw * 32) << 16;
                uint32_t r0[4], r1[4];
                tmem_ld4(tmem + lane_addr + kColB, r0);
                if (nj > 1) tmem_ld4(tmem + lane_addr + kColB + 16, r1);
                tmem_wait_ld();
#pragma unroll
                for (int r = 0; r < 4; ++r) {
                    sc0[r] = __uint_as_float(r0[r]);
                    sc1[r] = nj > 1 ? __uint_as_float(r1[r]) : 0.f;
                }
            }
            tc_fence_before();
            mbar_arrive(&bars[bStLd]);
            for (int j = 0; j < nj; ++j) {
                float sc[4];
#pragma unroll
                for (int r = 0; r < 4; ++r) sc[r] = j ? sc1[r] : sc0[r];
                const int u = (kt0 + j) * BN + k - past;
#pragma unroll
                for (int r = 0; r < 4; ++r) {
                    bool vis = false;
                    if (r < nt && ok) {
                        const int token = p.tail_token0 + r / p.group;
                        if (u < 0)
                            vis = !kWindow || (int64_t)(u + past) >= __ldg(p.key_lo + token);
                        else if (u < p.n_tokens)
                            vis = (__ldg(p.vis + (int64_t)token * p.vis_words + (u >> 5)) >> (u & 31)) & 1u;
                    }
                    sc[r] = vis ? sc[r] * sl2 : -INFINITY;
                }
                // column max: one redux per warp, one exchange across the 4 warps
                float* wm = wmax + j * 64;
#pragma unroll
                for (int r = 0; r < 4; ++r) {
                    if (r < nt) {
                        const float v = warp_max(sc[r]);
                        if (lane == 0) wm[tw * 16 + r] = v;
                    }
                }
                named_bar_sync(1, 128);
                float* ws = wsum + j * 64;
                float pr[4];
#pragma unroll
                for (int r = 0; r < 4; ++r) {
                    pr[r] = 0.f;
                    if (r < nt) {
                        const float mt = fmaxf(fmaxf(wm[r], wm[16 + r]), fmaxf(wm[32 + r], wm[48 + r]));
                        pr[r] = ex2_approx(sc[r] - (mt == -INFINITY ? 0.f : mt));   // -inf gives 0
                        // column sum in 2^-24 fixed point: every p <= 1, so a warp's sum fits 32 bits
                        const uint32_t sum = warp_sum_u32(__float2uint_rn(pr[r] * kFix));
                        if (lane == 0) ws[tw * 16 + r] = (float)sum * (1.f / kFix);
                        if (k == 0) tmax[j * 16 + r] = mt;
                    }
                }
                // P_t(j) as the [16 rows x 128 keys] K-major, 128-byte-swizzled B
                // operand of the transposed P.V product (rows >= 4 stay zero)
                unsigned char* ptb = smem + kPT + j * 4096 + (k >> 6) * kTHalf;
                const int kk = k & 63;
#pragma unroll
                for (int r = 0; r < 4; ++r)
                    *reinterpret_cast<__nv_bfloat16*>(ptb + r * 128 + ((((kk >> 3) ^ r) & 7) << 4) + (kk & 7) * 2) =
                        __float2bfloat16_rn(pr[r]);
                fence_proxy_async_smem();
                mbar_arrive(&bars[bPt0 + j]);
            }
            // thread r < nt merges row r's per-tile statistics into the weights of
            // each tile's P.V and the row's log-sum-exp
            named_bar_sync(1, 128);
            if (k < nt) {
                const float m0 = tmax[k], m1 = nj > 1 ? tmax[16 + k] : -INFINITY;
                const float l0 = wsum[k] + wsum[16 + k] + wsum[32 + k] + wsum[48 + k];
                const float l1 = nj > 1 ? wsum[64 + k] + wsum[80 + k] + wsum[96 + k] + wsum[112 + k] : 0.f;
                const float mm = fmaxf(m0, m1);
                const float w0 = m0 == -INFINITY ? 0.f : ex2_approx(m0 - mm);
                const float w1 = m1 == -INFINITY ? 0.f : ex2_approx(m1 - mm);
                const float L = w0 * l0 + w1 * l1;
                const float inv = L > 0.f ? 1.f / L : 0.f;
                wts[k] = w0 * inv;
                wts[16 + k] = w1 * inv;
                wts[32 + k] = L > 0.f ? mm + log2f(L) : -INFINITY;
            }
            named_bar_sync(1, 128);
            // O_t^T(j) in TMEM: lane = dim k, column = tail row
            ok = __all_sync(DDT_FULL_MASK, ok && mbar_wait(&bars[bPVt], 0));
            tc_fence_after();
            float o0[16], o1[16];
            {
                const uint32_t lane_addr = (uint32_t)(tw * 32) << 16;
                uint32_t r0[16], r1[16];
                if (ok) {
                    tmem_ld16(tmem + lane_addr + kCol1, r0);
                    if (nj > 1) tmem_ld16(tmem + lane_addr + kCol1 + 16, r1);
                    tmem_wait_ld();
                }
#pragma unroll
                for (int c = 0; c < 16; ++c) {
                    o0[c] = ok ? __uint_as_float(r0[c]) : 0.f;
                    o1[c] = (ok && nj > 1) ? __uint_as_float(r1[c]) : 0.f;
                }
            }
            if (!ok) {
                if (k == 0) flag_error(p.status, 4);
            } else {
                const int rows_head = p.group * p.n_tokens;
                const int d = k;
#pragma unroll
                for (int r = 0; r < 4; ++r) {
                    if (r < nt) {
                        const int token = p.tail_token0 + r / p.group;
                        const int head = g * p.group + r % p.group;
                        if (token < p.n_tokens) {
                            const float w0 = wts[r], w1 = nj > 1 ? wts[16 + r] : 0.f;
                            const __nv_bfloat16 h = __float2bfloat16_rn(w0 * o0[r] + w1 * o1[r]);
                            __nv_bfloat16* dst;
                            if (p.splits == 1) {
                                dst = p.out + (int64_t)token * p.o_stride_tok + (int64_t)head * p.o_stride_head;
                            } else {
                                const int64_t prow =
                                    ((int64_t)split * p.hkv + g) * rows_head + p.tail_token0 * p.group + r;
                                dst = p.part_o + prow * HD;
                                if (d == 0) p.part_lse[prow] = wts[32 + r];
                            }
                            dst[d] = h;
                        }
                    }
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 12) {
        tc_fence_after();
        tmem_dealloc(tmem, 512);
    }
}

// Merge of the split partials: one warp per row over hkv * rows_head rows,
// CHUNK splits per memory round trip.  The host picks the smallest CHUNK of
// 8, 12 and 17 that covers the splits in one round trip (at most 117
// registers, so four CTAs fit on an SM and the grid of the verify shapes is
// one wave), or 16 per pass beyond that.
template <int CHUNK>
__global__ void __launch_bounds__(128)
combine_kernel(const __nv_bfloat16* __restrict__ part_o, const float* __restrict__ part_lse, int splits, int hkv,
               int group, int n_tokens, __nv_bfloat16* out, int64_t o_stride_tok, int64_t o_stride_head,
               const int32_t* past_dev, int past_max, int tpc) {
    griddep_launch_dependents();
    griddep_wait();   // the partials come from the split kernel just before
    if (past_dev) {   // only the splits that held run-time keys wrote partials
        const int v = __ldg(past_dev);
        const int past = v < 0 ? 0 : (v > past_max ? past_max : v);
        const int n_kt = (past + n_tokens + BN - 1) / BN;
        splits = min(splits, (n_kt + tpc - 1) / tpc);
    }
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int rows_head = group * n_tokens;
    const int64_t row = (int64_t)blockIdx.x * 4 + warp;
    if (row >= (int64_t)hkv * rows_head) return;
    const int g = (int)(row / rows_head), r = (int)(row % rows_head);
    const int token = r / group, head = g * group + r % group;
    merge_row<CHUNK>(part_o, part_lse, splits, (int64_t)hkv * rows_head, (int64_t)g * rows_head + r, lane,
              out + (int64_t)token * o_stride_tok + (int64_t)head * o_stride_head);
}

}  // namespace split

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

// Split-kernel workspace: status word, then the partials.
constexpr size_t kSplitPartOffset = 256;

struct SplitPlan {
    int group, tpt, n_kt, tpc, splits, n_mt, n_groups, tail_rows, tail_token0;
    bool usable;
    size_t ws_bytes;
};

// The split kernel applies when the rows of a KV head are too few to fill
// the GPU without splitting keys (fewer M tiles x KV heads than SMs), the
// tail fits the 16-column transposed pass, and at most 16 waves of CTAs of
// at most two key tiles each cover the keys.
static SplitPlan plan_split(int64_t n_tokens, int64_t hq, int64_t hkv, int64_t past, int sms) {
    SplitPlan pl = {};
    if (sms <= 0) sms = 148;
    pl.group = (int)(hq / hkv);
    pl.tpt = BM / pl.group;
    const int64_t rows = (int64_t)pl.group * n_tokens;
    int64_t n_mt = rows / BM, rem = rows % BM, tail = 0;
    if (rem > 4 || (rem > 0 && 16 % pl.group != 0))
        n_mt += 1;
    else
        tail = rem;
    pl.n_mt = (int)n_mt;
    pl.tail_rows = (int)tail;
    pl.tail_token0 = (int)((rows - tail) / pl.group);
    pl.n_groups = (int)(n_mt > 0 ? (n_mt + 1) / 2 : 1);
    pl.n_kt = (int)ceil_div(past + n_tokens, BN);
    const int64_t units = hkv * pl.n_groups;
    pl.tpc = (int64_t)pl.n_kt * units <= sms ? 1 : 2;
    pl.splits = (int)ceil_div(pl.n_kt, pl.tpc);
    const int64_t ctas = (int64_t)pl.splits * units;
    pl.usable = ceil_div(rows, (int64_t)BM) * hkv < sms && ctas <= 16 * (int64_t)sms;
    size_t o = kSplitPartOffset;
    if (pl.splits > 1) {
        o += sizeof(__nv_bfloat16) * (size_t)pl.splits * n_tokens * hq * HD;
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

// Launch of the split kernel (and, with several key splits, the merge).
// past_dev (nullable): run-time prefix length; a->past_length is then its
// upper bound, the grid is planned for it, and the K/V maps span all
// kv_rows (rows past the run-time tree are masked by the tree bits and hold
// the caller's finite cache contents, so P = 0 never meets a NaN).
static int launch_split(const ddt_attention_args* a, const int64_t* key_lo, const int32_t* past_dev,
                        const int32_t* stable_dev, const SplitPlan& sp, void* workspace, size_t workspace_bytes,
                        ddt_stream_t stream) {
    if (!workspace || workspace_bytes < sp.ws_bytes || reinterpret_cast<uintptr_t>(workspace) % 256)
        return set_error(DDT_EWORKSPACE, "attention workspace needs %zu bytes (256-aligned), got %zu", sp.ws_bytes,
                         workspace_bytes);
    const int64_t group = a->hq / a->hkv;
    const int64_t kv_len = past_dev ? a->kv_rows : a->past_length + a->n_tokens;
    // Without past_dev the K/V maps end at past + n_tokens: rows of a larger
    // cache past the tree read as zeros, so whatever they hold never reaches P.V.
    CUtensorMap tq, tqt, tk, tv;
    int rc = make_map(&tq, a->q, HD, a->hq, a->n_tokens, a->q_stride_head * 2, a->q_stride_tok * 2, 64,
                      (uint32_t)group, (uint32_t)sp.tpt);
    if (!rc && sp.tail_rows > 0)
        rc = make_map(&tqt, a->q, HD, a->hq, a->n_tokens, a->q_stride_head * 2, a->q_stride_tok * 2, 64,
                      (uint32_t)group, (uint32_t)(16 / group));
    else
        tqt = tq;
    if (!rc) rc = make_map(&tk, a->k, HD, kv_len, a->hkv, a->kv_stride_row * 2, a->kv_stride_head * 2, 64, BN, 1);
    if (!rc) rc = make_map(&tv, a->v, HD, kv_len, a->hkv, a->kv_stride_row * 2, a->kv_stride_head * 2, 64, BN, 1);
    if (rc) return rc;
    static std::once_flag once;
    static cudaError_t attr_err = cudaSuccess;
    std::call_once(once, [] {
        attr_err = cudaFuncSetAttribute(split::tree_attn_split_kernel<false>,
                                        cudaFuncAttributeMaxDynamicSharedMemorySize, (int)split::kSmemBytes);
        if (attr_err == cudaSuccess)
            attr_err = cudaFuncSetAttribute(split::tree_attn_split_kernel<true>,
                                            cudaFuncAttributeMaxDynamicSharedMemorySize, (int)split::kSmemBytes);
    });
    if (attr_err != cudaSuccess) return set_error(DDT_ECUDA, "cudaFuncSetAttribute: %s", cudaGetErrorString(attr_err));
    unsigned char* ws = static_cast<unsigned char*>(workspace);
    split::Params q;
    q.n_tokens = (int)a->n_tokens;
    q.hq = (int)a->hq;
    q.hkv = (int)a->hkv;
    q.group = sp.group;
    q.tpt = sp.tpt;
    q.past = (int)a->past_length;
    q.n_kt = sp.n_kt;
    q.tpc = sp.tpc;
    q.splits = sp.splits;
    q.n_mt = sp.n_mt;
    q.n_groups = sp.n_groups;
    q.tail_rows = sp.tail_rows;
    q.tail_token0 = sp.tail_token0;
    q.vis = a->visibility;
    q.key_lo = key_lo;
    q.vis_words = (int)a->vis_words;
    q.scale_log2 = a->scale * 1.4426950408889634f;
    q.out = static_cast<__nv_bfloat16*>(a->out);
    q.o_stride_tok = a->o_stride_tok;
    q.o_stride_head = a->o_stride_head;
    q.status = reinterpret_cast<int*>(ws);
    q.past_dev = past_dev;
    // Host-length calls: the whole prefix is stable unless this library's
    // own kernels may be running ahead of this one (ddt_set_pdl), when no
    // key loads early.  Device-length calls: what the caller states.
    q.stable_dev = stable_dev;
    q.stable = (past_dev || pdl_enabled()) ? 0 : (int)a->past_length;
    q.part_o = nullptr;
    q.part_lse = nullptr;
    if (sp.splits > 1) {
        size_t o = kSplitPartOffset;
        q.part_o = reinterpret_cast<__nv_bfloat16*>(ws + o);
        o += sizeof(__nv_bfloat16) * (size_t)sp.splits * a->n_tokens * a->hq * HD;
        o = (o + 255) & ~size_t(255);
        q.part_lse = reinterpret_cast<float*>(ws + o);
    }
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    dim3 grid((unsigned)sp.splits, (unsigned)sp.n_groups, (unsigned)a->hkv);
    // Both kernels are launched as programmatic dependents of whatever precedes
    // them in the stream: their prologues (and the prefix K/V loads) overlap
    // the previous kernel's tail; each waits for it before touching its data.
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = dim3(split::kThreads);
    cfg.dynamicSmemBytes = split::kSmemBytes;
    cfg.stream = st;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaError_t le = key_lo ? cudaLaunchKernelEx(&cfg, split::tree_attn_split_kernel<true>, tq, tqt, tk, tv, q)
                            : cudaLaunchKernelEx(&cfg, split::tree_attn_split_kernel<false>, tq, tqt, tk, tv, q);
    if (le != cudaSuccess) return set_error(DDT_ECUDA, "tree_attn_split_kernel: %s", cudaGetErrorString(le));
    rc = check_launch("tree_attn_split_kernel");
    if (rc) return rc;
    if (sp.splits > 1) {
        const int64_t rows = a->n_tokens * a->hq;
        cfg.gridDim = dim3((unsigned)ceil_div(rows, 4));
        cfg.blockDim = dim3(128);
        cfg.dynamicSmemBytes = 0;
        auto ck = sp.splits <= 8 ? split::combine_kernel<8>
                  : sp.splits <= 12 ? split::combine_kernel<12>
                  : sp.splits <= 17 ? split::combine_kernel<17>
                                    : split::combine_kernel<16>;
        le = cudaLaunchKernelEx(&cfg, ck, (const __nv_bfloat16*)q.part_o, (const float*)q.part_lse, sp.splits,
                                (int)a->hkv, sp.group, (int)a->n_tokens, q.out, a->o_stride_tok, a->o_stride_head,
                                past_dev, (int)a->past_length, sp.tpc);
        if (le != cudaSuccess) return set_error(DDT_ECUDA, "split_combine_kernel: %s", cudaGetErrorString(le));
        rc = check_launch("split_combine_kernel");
    }
    return rc;
}

extern "C" size_t ddt_tree_attention_workspace_size(int64_t n_tokens, int64_t hq, int64_t hkv, int64_t past_length,
                                                    int device) {
    if (n_tokens <= 0 || hq <= 0 || hkv <= 0 || hq % hkv || past_length < 0) return 256;
    const int sms = ddt_sm_count(device);
    const size_t a = plan_for(n_tokens, hq, hkv, past_length, sms > 0 ? sms : 148).ws_bytes;
    const SplitPlan sp = plan_split(n_tokens, hq, hkv, past_length, sms);
    return sp.usable && sp.ws_bytes > a ? sp.ws_bytes : a;
}

static int tree_attention_impl(const ddt_attention_args* a, const int64_t* key_lo, const int32_t* past_dev,
                               const int32_t* stable_dev, void* workspace, size_t workspace_bytes,
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
    const SplitPlan sp = plan_split(a->n_tokens, a->hq, a->hkv, a->past_length, ddt_sm_count(dev));
    if (past_dev) {
        if (reinterpret_cast<uintptr_t>(past_dev) % alignof(int32_t))
            return set_error(DDT_EINVAL, "past_dev must be 4-byte aligned");
        if (!sp.usable)
            return set_error(DDT_EUNSUPPORTED, "a run-time prefix needs the split kernel: %lld rows x %lld KV heads "
                             "at prefix <= %lld do not fit it", (long long)(a->n_tokens * group),
                             (long long)a->hkv, (long long)a->past_length);
        return launch_split(a, key_lo, past_dev, stable_dev, sp, workspace, workspace_bytes, stream);
    }
    const Plan pl = plan_for(a->n_tokens, a->hq, a->hkv, a->past_length, ddt_sm_count(dev));
    if (!workspace || workspace_bytes < pl.ws_bytes || reinterpret_cast<uintptr_t>(workspace) % 256)
        return set_error(DDT_EWORKSPACE, "attention workspace needs %zu bytes (256-aligned), got %zu", pl.ws_bytes,
                         workspace_bytes);
    if (sp.usable) return launch_split(a, key_lo, nullptr, nullptr, sp, workspace, workspace_bytes, stream);
    CUtensorMap tq, tk, tv;
    int rc = make_map(&tq, a->q, HD, a->hq, a->n_tokens, a->q_stride_head * 2, a->q_stride_tok * 2, 64,
                      (uint32_t)group, (uint32_t)pl.tpt);
    if (rc) return rc;
    // K/V maps end at past + n_tokens: cache rows past the tree read as zeros
    rc = make_map(&tk, a->k, HD, a->past_length + a->n_tokens, a->hkv, a->kv_stride_row * 2, a->kv_stride_head * 2, 64, BN, 1);
    if (rc) return rc;
    rc = make_map(&tv, a->v, HD, a->past_length + a->n_tokens, a->hkv, a->kv_stride_row * 2, a->kv_stride_head * 2, 64, BN, 1);
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
    p.key_lo = key_lo;
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

extern "C" int ddt_tree_attention(const ddt_attention_args* a, void* workspace, size_t workspace_bytes,
                                  ddt_stream_t stream) {
    return tree_attention_impl(a, nullptr, nullptr, nullptr, workspace, workspace_bytes, stream);
}

extern "C" int ddt_tree_attention_window(const ddt_attention_args* a, const int64_t* key_lo, void* workspace,
                                         size_t workspace_bytes, ddt_stream_t stream) {
    if (!key_lo) return set_error(DDT_EINVAL, "key_lo is null");
    if (reinterpret_cast<uintptr_t>(key_lo) % alignof(int64_t)) return set_error(DDT_EINVAL, "key_lo must be 8-byte aligned");
    return tree_attention_impl(a, key_lo, nullptr, nullptr, workspace, workspace_bytes, stream);
}

extern "C" int ddt_tree_attention_dev(const ddt_attention_args* a, const int64_t* key_lo, const int32_t* past_dev,
                                      const int32_t* stable_dev, void* workspace, size_t workspace_bytes,
                                      ddt_stream_t stream) {
    if (!past_dev) return set_error(DDT_EINVAL, "past_dev is null");
    if (key_lo && reinterpret_cast<uintptr_t>(key_lo) % alignof(int64_t))
        return set_error(DDT_EINVAL, "key_lo must be 8-byte aligned");
    if (stable_dev && reinterpret_cast<uintptr_t>(stable_dev) % alignof(int32_t))
        return set_error(DDT_EINVAL, "stable_dev must be 4-byte aligned");
    return tree_attention_impl(a, key_lo, past_dev, stable_dev, workspace, workspace_bytes, stream);
}
