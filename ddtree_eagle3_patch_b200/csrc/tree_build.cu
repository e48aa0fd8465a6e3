// Kernel (1): DDTree tree build on sm_100a.
//
// Restates build_ddtree_tree (ddtree.py:114-196) as one launch:
//   phase A  (rows x chunks CTAs)  per chunk of a draft row, staged in shared
//            memory: max, sum of exp, and the chunk's top-k on 64-bit keys
//            (value, then lower token id), written sorted - ddtree.py:136-138:
//            a warp-sorted lower bound gathers a few candidates, ranked by
//            counting (radix select when there are many);
//   phase B  (last CTA of a row)   the row's top-k from the sorted chunk
//            lists: the keys at or above the largest list tail, ranked by
//            counting; log-normaliser, lp = top - log_z  (ddtree.py:139);
//   phase C  (last CTA overall)    the best-first expansion, restated exactly
//            with one warp doing the frontier arg-min each step
//            (ddtree.py:146-177), then parents / depths / tokens, the packed
//            ancestor bitmask (ddtree.py:181-188) and the verify ids /
//            positions (ddtree.py:233-242).
// The hand-off between phases uses the "last block done" pattern (a fence
// and an atomic counter); no CTA ever waits on another.

#include <cstdio>
#include <mutex>

#include "common.cuh"

namespace ddt {
namespace tree {

constexpr int kThreads = 512;
constexpr int kWarps = kThreads / 32;
constexpr int kValsPerThread = 40;
constexpr int kMaxChunk = kThreads * kValsPerThread;  // 20480 elements: a 151936-wide row in 8 chunks
constexpr int kCandCap = 2048;
constexpr int kHeadCandCap = kMaxChunk / 2;   // head-statistics mode: candidates held in the staging area
constexpr int kMaxRows = 32;
constexpr int kMaxBudget = 1024;
constexpr int kMergeCap = 16384;  // chunks * topk keys held by the merging CTA
constexpr int kRankCap = 256;     // candidate counts ranked directly (rank = number of larger keys)

struct SelectScratch {
    uint32_t hist[256];
    unsigned long long prefix;
    int need;
    int done;
    int count;
    int flag;
};

// Workspace layout (all offsets 256-byte aligned).
struct WsLayout {
    size_t row_cnt, done_cnt, part_m, part_s, part_keys, top_ids, top_lp, total;
};

__host__ __device__ inline size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

__host__ __device__ inline WsLayout ws_layout(int64_t rows, int64_t chunks, int64_t topk) {
    WsLayout w;
    size_t o = 0;
    w.row_cnt = o;
    o = align256(o + sizeof(uint32_t) * kMaxRows);
    w.done_cnt = o;
    o = align256(o + sizeof(uint32_t) * 4);
    w.part_m = o;
    o = align256(o + sizeof(float) * rows * chunks);
    w.part_s = o;
    o = align256(o + sizeof(double) * rows * chunks);
    w.part_keys = o;
    o = align256(o + sizeof(uint64_t) * rows * chunks * topk);
    w.top_ids = o;
    o = align256(o + sizeof(int64_t) * rows * topk);
    w.top_lp = o;
    o = align256(o + sizeof(float) * rows * topk);
    w.total = o;
    return w;
}

__host__ inline void choose_chunks(int64_t rows, int64_t vocab, int64_t topk, int sms, int64_t* chunks,
                                   int64_t* chunk_len) {
    int64_t c_min = ceil_div(vocab, kMaxChunk);
    int64_t c_fill = rows > 0 ? (int64_t)sms / rows : 1;
    int64_t c_small = ceil_div(vocab, 2048);
    int64_t c = c_fill < c_small ? c_fill : c_small;
    if (c < c_min) c = c_min;
    if (c < 1) c = 1;
    while (c > c_min && c * topk > kMergeCap) --c;
    int64_t len = ceil_div(vocab, c);
    len = (len + 7) & ~int64_t(7);
    *chunk_len = len;
    *chunks = ceil_div(vocab, len);
}

// ---------------------------------------------------------------------------
// block-wide helpers
// ---------------------------------------------------------------------------
__device__ __forceinline__ float block_max(float v, float* red) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(DDT_FULL_MASK, v, o));
    __syncthreads();
    if (lane == 0) red[warp] = v;
    __syncthreads();
    if (warp == 0) {
        v = lane < kWarps ? red[lane] : -INFINITY;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(DDT_FULL_MASK, v, o));
        if (lane == 0) red[0] = v;
    }
    __syncthreads();
    return red[0];
}

__device__ __forceinline__ double block_sum_d(double v, double* red) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(DDT_FULL_MASK, v, o);
    __syncthreads();
    if (lane == 0) red[warp] = v;
    __syncthreads();
    if (warp == 0) {
        v = lane < kWarps ? red[lane] : 0.0;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(DDT_FULL_MASK, v, o);
        if (lane == 0) red[0] = v;
    }
    __syncthreads();
    return red[0];
}

// Warp 0 picks the 8-bit bin that holds the need-th largest key.
__device__ __forceinline__ void pick_bin(SelectScratch* s, int shift) {
    const int lane = threadIdx.x & 31;
    // lane l owns bins 255-8l ... 248-8l (descending)
    uint32_t c[8];
    uint32_t tot = 0;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        c[j] = s->hist[255 - (lane * 8 + j)];
        tot += c[j];
    }
    uint32_t incl = tot;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        uint32_t t = __shfl_up_sync(DDT_FULL_MASK, incl, o);
        if (lane >= o) incl += t;
    }
    uint32_t before = incl - tot;
    const uint32_t need = (uint32_t)s->need;
    bool mine = before < need && need <= incl;
    if (mine) {
        uint32_t acc = before;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            if (acc < need && need <= acc + c[j]) {
                const uint32_t bin = 255 - (lane * 8 + j);
                s->prefix |= (unsigned long long)bin << shift;
                s->need = (int)(need - acc);
                s->done = (c[j] == need - acc) ? 1 : 0;
            }
            acc += c[j];
        }
    }
}

// K-th largest of n distinct 64-bit keys held in shared or global memory.
// Returns T with "key >= T" selecting exactly K keys.  All threads call it.
__device__ unsigned long long block_kth_largest(const unsigned long long* keys, int n, int K, SelectScratch* s) {
    if (threadIdx.x == 0) {
        s->prefix = 0ull;
        s->need = K;
        s->done = 0;
    }
    unsigned long long mask = 0ull;
    for (int shift = 56; shift >= 0; shift -= 8) {
        for (int i = threadIdx.x; i < 256; i += kThreads) s->hist[i] = 0;
        __syncthreads();
        const unsigned long long prefix = s->prefix;
        for (int i = threadIdx.x; i < n; i += kThreads) {
            const unsigned long long k = keys[i];
            if ((k & mask) == prefix) atomicAdd(&s->hist[(k >> shift) & 255u], 1u);
        }
        __syncthreads();
        if (threadIdx.x < 32) pick_bin(s, shift);
        __syncthreads();
        mask |= 0xffull << shift;
        if (s->done) break;
    }
    const unsigned long long t = s->prefix;
    __syncthreads();
    return t;
}

// Same, over keys produced by key_at(j), j < kValsPerThread, per thread (0 = empty).
template <typename KeyAt>
__device__ __forceinline__ unsigned long long block_kth_largest_regs(KeyAt key_at, int K, SelectScratch* s) {
    if (threadIdx.x == 0) {
        s->prefix = 0ull;
        s->need = K;
        s->done = 0;
    }
    unsigned long long mask = 0ull;
    for (int shift = 56; shift >= 0; shift -= 8) {
        for (int i = threadIdx.x; i < 256; i += kThreads) s->hist[i] = 0;
        __syncthreads();
        const unsigned long long prefix = s->prefix;
#pragma unroll
        for (int j = 0; j < kValsPerThread; ++j) {
            const unsigned long long k = key_at(j);
            if (k != 0ull && (k & mask) == prefix) atomicAdd(&s->hist[(k >> shift) & 255u], 1u);
        }
        __syncthreads();
        if (threadIdx.x < 32) pick_bin(s, shift);
        __syncthreads();
        mask |= 0xffull << shift;
        if (s->done) break;
    }
    const unsigned long long t = s->prefix;
    __syncthreads();
    return t;
}

__device__ __forceinline__ unsigned long long make_key(float v, int64_t idx) { return topk_key(v, idx); }
__device__ __forceinline__ int64_t key_index(unsigned long long k) {
    return (int64_t)(0xffffffffu - (uint32_t)(k & 0xffffffffull));
}
__device__ __forceinline__ float key_value(unsigned long long k) { return unord_f32((uint32_t)(k >> 32)); }
// Key of a chunk value at chunk-local index loc (0 past the chunk).
__device__ __forceinline__ unsigned long long chunk_key(float v, int loc, int n_valid, int64_t c0) {
    return loc < n_valid ? make_key(v, c0 + loc) : 0ull;
}

// Runs BODY with X = each value this thread holds in the staged chunk `cv`,
// LOC = its chunk-local index and J = its slot (0 .. kValsPerThread-1), in
// index order: a rolled loop over the thread's 16-byte vectors, unrolled
// within one.  Each CTA runs a pass over ~17K values, so every instruction
// per value costs ~130 issue cycles of its SM: the bodies are kept to a few.
#define DDT_FOR_VALS(X, LOC, J, BODY)                                                             \
    _Pragma("unroll 1") for (int jv_ = 0; jv_ < kNv; ++jv_) {                                     \
        const int l0_ = (jv_ * kThreads + tid) * kEpv;                                            \
        _Pragma("unroll") for (int h_ = 0; h_ < kEpv; h_ += 4) {                                  \
            const float4 q_ = *reinterpret_cast<const float4*>(cv + l0_ + h_);                   \
            const float qv_[4] = {q_.x, q_.y, q_.z, q_.w};                                       \
            _Pragma("unroll") for (int e_ = 0; e_ < 4; ++e_) {                                    \
                const float X = qv_[e_];                                                          \
                const int LOC = l0_ + h_ + e_;                                                    \
                const int J = jv_ * kEpv + h_ + e_;                                               \
                (void)LOC;                                                                        \
                (void)J;                                                                          \
                BODY                                                                              \
            }                                                                                     \
        }                                                                                         \
    }

// ---------------------------------------------------------------------------
// phase C: best-first expansion (ddtree.py:146-189)
// ---------------------------------------------------------------------------
struct ExpandSmem {
    float* lp;           // [rows * topk]
    double* f_logw;      // frontier: path score
    int32_t* f_parent;   //           parent node index
    int32_t* f_dr;       //           depth << 16 | rank
    int32_t* n_parent;   // node i: parent        (i in [0, budget])
    int32_t* n_dr;       //         depth << 16 | rank
    int32_t* scalars;    // [4]
    unsigned char* par;  // table of the parallel expansion, or null
};

// the parallel expansion's limits (its table is sized for them)
__host__ __device__ inline bool par_expand_fits(int64_t rows, int64_t budget) {
    return budget <= 64 && rows <= 16;
}

__host__ __device__ inline size_t expand_smem_bytes(int64_t rows, int64_t topk, int64_t budget) {
    size_t o = 0;
    o += align256(sizeof(float) * rows * topk);
    o += align256(sizeof(double) * (budget + 1));
    o += align256(sizeof(int32_t) * (budget + 1)) * 4;
    o += 256;
    if (par_expand_fits(rows, budget)) o += 96 * 1024;   // >= par_smem_bytes(), checked below
    return o;
}

__device__ inline ExpandSmem carve_expand(unsigned char* base, int64_t rows, int64_t topk, int64_t budget) {
    ExpandSmem e;
    size_t o = 0;
    e.lp = reinterpret_cast<float*>(base + o);
    o += align256(sizeof(float) * rows * topk);
    e.f_logw = reinterpret_cast<double*>(base + o);
    o += align256(sizeof(double) * (budget + 1));
    e.f_parent = reinterpret_cast<int32_t*>(base + o);
    o += align256(sizeof(int32_t) * (budget + 1));
    e.f_dr = reinterpret_cast<int32_t*>(base + o);
    o += align256(sizeof(int32_t) * (budget + 1));
    e.n_parent = reinterpret_cast<int32_t*>(base + o);
    o += align256(sizeof(int32_t) * (budget + 1));
    e.n_dr = reinterpret_cast<int32_t*>(base + o);
    o += align256(sizeof(int32_t) * (budget + 1));
    e.scalars = reinterpret_cast<int32_t*>(base + o);
    o += 256;
    e.par = par_expand_fits(rows, budget) ? base + o : nullptr;
    return e;
}

// Ranks tuple of a frontier slot (ddtree.py:148): ranks of its parent's path, then its own rank.
__device__ int slot_path(const ExpandSmem& e, int slot, int* out) {
    const int dr = e.f_dr[slot];
    const int depth = dr >> 16;
    out[depth - 1] = dr & 0xffff;
    int node = e.f_parent[slot];
    for (int k = depth - 2; k >= 0; --k) {
        out[k] = e.n_dr[node] & 0xffff;
        node = e.n_parent[node];
    }
    return depth;
}

// Python tuple order of the ranks tuples of two slots.
__device__ bool slot_tuple_less(const ExpandSmem& e, int a, int b) {
    int pa[kMaxRows], pb[kMaxRows];
    const int na = slot_path(e, a, pa), nb = slot_path(e, b, pb);
    const int n = na < nb ? na : nb;
    for (int k = 0; k < n; ++k)
        if (pa[k] != pb[k]) return pa[k] < pb[k];
    return na < nb;
}

// Frontier in shared memory, any budget: one warp, lane-strided scan of the
// slots each step.
__device__ int expand_smem(const ExpandSmem& e, int rows, int topk, int budget, int lane) {
    int fsize = 1;
    if (lane == 0) {
        e.f_logw[0] = (double)e.lp[0];
        e.f_parent[0] = 0;
        e.f_dr[0] = (1 << 16) | 0;
        e.n_parent[0] = -1;
        e.n_dr[0] = 0;
    }
    __syncwarp();
    int count = 0;
    while (count < budget && fsize > 0) {
        // lane-local minimum of (-logw, ranks tuple)
        unsigned long long best_u = ~0ull;
        int best_s = -1;
        for (int s = lane; s < fsize; s += 32) {
            const unsigned long long u = ord_f64(-e.f_logw[s]);
            if (u < best_u || (u == best_u && best_s >= 0 && slot_tuple_less(e, s, best_s))) {
                best_u = u;
                best_s = s;
            }
        }
        const uint32_t hi = __reduce_min_sync(DDT_FULL_MASK, (uint32_t)(best_u >> 32));
        const uint32_t lo =
            __reduce_min_sync(DDT_FULL_MASK, ((uint32_t)(best_u >> 32) == hi) ? (uint32_t)best_u : 0xffffffffu);
        const unsigned long long umin = ((unsigned long long)hi << 32) | lo;
        const uint32_t tied = __ballot_sync(DDT_FULL_MASK, best_s >= 0 && best_u == umin);
        int w;
        if (__popc(tied) == 1) {
            w = __shfl_sync(DDT_FULL_MASK, best_s, __ffs(tied) - 1);
        } else {
            // exact float64 tie across lanes: decide by the ranks tuples
            int pick = -1;
            if (lane == 0) {
                for (int s = 0; s < fsize; ++s) {
                    if (ord_f64(-e.f_logw[s]) != umin) continue;
                    if (pick < 0 || slot_tuple_less(e, s, pick)) pick = s;
                }
            }
            w = __shfl_sync(DDT_FULL_MASK, pick, 0);
        }
        if (lane == 0) {
            const double logw = e.f_logw[w];
            const int parent = e.f_parent[w];
            const int dr = e.f_dr[w];
            const int depth = dr >> 16, rank = dr & 0xffff;
            const int cur = count + 1;
            e.n_parent[cur] = parent;
            e.n_dr[cur] = dr;
            const bool sib = rank + 1 < topk;
            const bool child = depth < rows;
            int nf = fsize;
            if (sib) {
                const double a = (double)e.lp[(depth - 1) * topk + rank];
                const double b = (double)e.lp[(depth - 1) * topk + rank + 1];
                const double s = __dadd_rn(__dadd_rn(logw, -a), b);
                e.f_logw[w] = s;
                e.f_parent[w] = parent;
                e.f_dr[w] = (depth << 16) | (rank + 1);
            }
            if (child) {
                const double c = __dadd_rn(logw, (double)e.lp[depth * topk]);
                const int slot = sib ? nf++ : w;
                e.f_logw[slot] = c;
                e.f_parent[slot] = cur;
                e.f_dr[slot] = (depth + 1) << 16;
            }
            if (!sib && !child) {
                nf -= 1;
                if (w != nf) {
                    e.f_logw[w] = e.f_logw[nf];
                    e.f_parent[w] = e.f_parent[nf];
                    e.f_dr[w] = e.f_dr[nf];
                }
            }
            e.scalars[0] = nf;
        }
        __syncwarp();
        fsize = *(volatile int32_t*)&e.scalars[0];
        count += 1;
    }
    return count;
}

// Ranks tuple of a frontier entry packed as parent << 17 | depth << 11 | rank.
__device__ int packed_path(const ExpandSmem& e, uint32_t pk, int* out) {
    const int depth = (pk >> 11) & 63;
    out[depth - 1] = pk & 2047;
    int node = (int)(pk >> 17);
    for (int k = depth - 2; k >= 0; --k) {
        out[k] = e.n_dr[node] & 0xffff;
        node = e.n_parent[node];
    }
    return depth;
}
__device__ bool packed_tuple_less(const ExpandSmem& e, uint32_t a, uint32_t b) {
    int pa[kMaxRows], pb[kMaxRows];
    const int na = packed_path(e, a, pa), nb = packed_path(e, b, pb);
    const int n = na < nb ? na : nb;
    for (int k = 0; k < n; ++k)
        if (pa[k] != pb[k]) return pa[k] < pb[k];
    return na < nb;
}

// Frontier in registers for budgets below 32 * S: slot i lives in lane i % 32,
// register i / 32, as (path score, parent << 17 | depth << 11 | rank).  A step
// is a register min per lane, a warp min of the 64-bit order key, and a
// broadcast of the winner; every lane computes the sibling and child scores
// (same fp64 operations and order as the reference, ddtree.py:171, 176) and
// the owning lanes update their registers.  Exact fp64 ties between slots go
// through shared memory and are decided by the ranks tuples.
template <int S>
__device__ int expand_regs(const ExpandSmem& e, int rows, int topk, int budget, int lane) {
    double lw[S];
    uint32_t pk[S];
    unsigned long long key[S];   // ord_f64(-lw): smaller key = higher score; ~0 marks an empty slot
#pragma unroll
    for (int s = 0; s < S; ++s) {
        lw[s] = 0.0;
        pk[s] = 0u;
        key[s] = ~0ull;
    }
    if (lane == 0) {
        lw[0] = (double)e.lp[0];
        pk[0] = (0u << 17) | (1u << 11) | 0u;
        key[0] = ord_f64(-lw[0]);
        e.n_parent[0] = -1;
        e.n_dr[0] = 0;
    }
    int* tie_buf = reinterpret_cast<int*>(e.f_logw);   // tie candidates: (slot, packed) pairs
    int fsize = 1, count = 0;
    while (count < budget && fsize > 0) {
        // lane minimum, then the warp minimum of the high word; the low word
        // is only reduced when high words tie
        unsigned long long best = key[0];
        int bs = 0;
#pragma unroll
        for (int s = 1; s < S; ++s)
            if (key[s] < best) {
                best = key[s];
                bs = s;
            }
        const uint32_t bhi = (uint32_t)(best >> 32);
        const uint32_t hi = __reduce_min_sync(DDT_FULL_MASK, bhi);
        uint32_t cand = __ballot_sync(DDT_FULL_MASK, bhi == hi);
        unsigned long long umin = best;
        if (__popc(cand) != 1) {
            const uint32_t lo = __reduce_min_sync(DDT_FULL_MASK, bhi == hi ? (uint32_t)best : 0xffffffffu);
            umin = ((unsigned long long)hi << 32) | lo;
            cand = __ballot_sync(DDT_FULL_MASK, best == umin);
        } else {
            umin = __shfl_sync(DDT_FULL_MASK, best, __ffs(cand) - 1);
        }
        // a slot tie inside a lane also needs the tuple rule
        int mine = 0;
#pragma unroll
        for (int s = 0; s < S; ++s) mine += key[s] == umin ? 1 : 0;
        const bool unique = __popc(cand) == 1 && __ballot_sync(DDT_FULL_MASK, mine > 1) == 0;
        int wl, ws;
        if (unique) {
            wl = __ffs(cand) - 1;
            ws = __shfl_sync(DDT_FULL_MASK, bs, wl);
        } else {
            int pre = mine;   // inclusive prefix of the per-lane tie counts
            for (int o = 1; o < 32; o <<= 1) {
                const int v = __shfl_up_sync(DDT_FULL_MASK, pre, o);
                if (lane >= o) pre += v;
            }
            const int total = __shfl_sync(DDT_FULL_MASK, pre, 31);
            int k = pre - mine;
#pragma unroll
            for (int s = 0; s < S; ++s) {
                if (key[s] == umin) {
                    tie_buf[2 * k] = s * 32 + lane;
                    tie_buf[2 * k + 1] = (int)pk[s];
                    ++k;
                }
            }
            __syncwarp();
            if (lane == 0) {
                int pick = 0;
                for (int c = 1; c < total; ++c)
                    if (packed_tuple_less(e, (uint32_t)tie_buf[2 * c + 1], (uint32_t)tie_buf[2 * pick + 1])) pick = c;
                e.scalars[3] = tie_buf[2 * pick];
            }
            __syncwarp();
            const int widx = *(volatile int32_t*)&e.scalars[3];
            __syncwarp();
            wl = widx & 31;
            ws = widx >> 5;
        }
        double wlw = 0.0;
        uint32_t wpk = 0u;
#pragma unroll
        for (int s = 0; s < S; ++s)
            if (s == ws) {
                wlw = lw[s];
                wpk = pk[s];
            }
        wlw = __shfl_sync(DDT_FULL_MASK, wlw, wl);
        wpk = __shfl_sync(DDT_FULL_MASK, wpk, wl);
        const uint32_t parent = wpk >> 17;
        const int depth = (int)((wpk >> 11) & 63), rank = (int)(wpk & 2047);
        const int cur = count + 1;
        if (lane == 0) {
            e.n_parent[cur] = (int)parent;
            e.n_dr[cur] = (depth << 16) | rank;
        }
        const bool sib = rank + 1 < topk;
        const bool child = depth < rows;
        double sv = 0.0, cv = 0.0;
        if (sib) {
            const double a = (double)e.lp[(depth - 1) * topk + rank];
            const double b = (double)e.lp[(depth - 1) * topk + rank + 1];
            sv = __dadd_rn(__dadd_rn(wlw, -a), b);
        }
        if (child) cv = __dadd_rn(wlw, (double)e.lp[depth * topk]);
        const uint32_t spk = (parent << 17) | ((uint32_t)depth << 11) | (uint32_t)(rank + 1);
        const uint32_t cpk = ((uint32_t)cur << 17) | ((uint32_t)(depth + 1) << 11);
        double nv = sv;
        uint32_t npk = spk;
        unsigned long long nkey;
        if (sib) {
            nkey = ord_f64(-sv);
        } else if (child) {
            nv = cv;
            npk = cpk;
            nkey = ord_f64(-cv);
        } else {
            // remove the winner: the last slot moves into its place
            const int li = fsize - 1, ll = li & 31, ls = li >> 5;
            double lv = 0.0;
            uint32_t lpk = 0u;
            unsigned long long lk = ~0ull;
#pragma unroll
            for (int s = 0; s < S; ++s)
                if (s == ls) {
                    lv = lw[s];
                    lpk = pk[s];
                    lk = key[s];
                }
            nv = __shfl_sync(DDT_FULL_MASK, lv, ll);
            npk = __shfl_sync(DDT_FULL_MASK, lpk, ll);
            nkey = __shfl_sync(DDT_FULL_MASK, lk, ll);
        }
        if (lane == wl) {
#pragma unroll
            for (int s = 0; s < S; ++s)
                if (s == ws) {
                    lw[s] = nv;
                    pk[s] = npk;
                    key[s] = nkey;
                }
        }
        if (!sib && !child) {   // the last slot empties (after the move, which it may be the source of)
            const int li = fsize - 1;
            if (lane == (li & 31)) {
#pragma unroll
                for (int s = 0; s < S; ++s)
                    if (s == (li >> 5)) key[s] = ~0ull;
            }
        }
        if (sib && child) {
            const int al = fsize & 31, as = fsize >> 5;
            const unsigned long long ckey = ord_f64(-cv);
            if (lane == al) {
#pragma unroll
                for (int s = 0; s < S; ++s)
                    if (s == as) {
                        lw[s] = cv;
                        pk[s] = cpk;
                        key[s] = ckey;
                    }
            }
            fsize += 1;
        } else if (!sib && !child) {
            fsize -= 1;
        }
        ++count;
    }
    return count;
}

// ---------------------------------------------------------------------------
// Parallel form of the same expansion (budget <= 64, rows <= 16).
//
// Every frontier entry is created from the entry just popped: its sibling
// fl(fl(S - a_r) + a_{r+1}) or its first child fl(S + a_0), where a is a
// row of log-probs sorted descending and S <= a_r <= 0 is the popped path
// score.  Both are never above S: a child adds a_0 <= 0; for a sibling,
// S - a_r lies in [S, 0] on S's grid (a_r's float32 grid is no finer while
// |S| < 2^29 |a_r|), so the first sum is exact and the second rounds
// S - a_r + a_{r+1} <= S, a value below the representable S, to at most S.
// With keys that never improve along the generating edges, the heap pops
// the nodes in the global order of (score desc, ranks tuple asc), so the
// popped set is the best `budget` nodes of the whole rank tree.
//
// Those are found depth by depth: the pool holds the best `budget` nodes
// seen so far, sorted; each depth-(d-1) pool node (the root at d = 1)
// generates its children's scores with the reference's sibling recurrence,
// one thread per parent, while the child beats the pool's current last
// entry (later siblings only get worse) and has fewer than `budget` nodes
// on its generating path; the new nodes are merged into the pool by rank
// counting.  A node dropped from the pool has `budget` better nodes, and so
// has every node under it.  The ranks tuple is kept as a left-aligned
// string of 7-bit fields (rank + 1 per depth), compared as two integers, so
// ties of the score are decided exactly as Python's tuple order does.
//
// Each computed step is checked (no increase, finite); on a failed check,
// or more nodes than the table holds, the serial loop below runs instead.
// ---------------------------------------------------------------------------
constexpr int kParMaxBudget = 64;
constexpr int kParNodes = 1024;
constexpr int kScratchStride = kParMaxBudget + 1;   // odd stride: the slots' rows fall in different banks

struct ParSmem {
    double* score;                 // [kParNodes] path score
    unsigned long long* key;       //             ord_f64(-score): smaller = pops first
    unsigned long long* phi;       //             ranks tuple, depths 1..9
    unsigned long long* plo;       //             ranks tuple, depths 10..16
    int32_t* parent;               //             node id of the parent, -1 = root
    int32_t* dr;                   //             depth << 16 | rank
    int32_t* acnt;                 //             nodes on the generating path before it
    int32_t* pos;                  //             position in the final pool
    int32_t* pool;                 // [kParMaxBudget] node ids, in pop order
    int32_t* pool2;                // [kParMaxBudget] the next pool
    double* scratch;               // [kParMaxBudget][kScratchStride] one depth's chain scores per pool slot
    int32_t* ctl;                  // [4] flags, then [kParMaxBudget + 1] chain offsets
};

__host__ __device__ constexpr size_t par_smem_bytes() {
    return ((sizeof(double) + 3 * sizeof(unsigned long long) + 4 * sizeof(int32_t)) * kParNodes + 255) / 256 * 256 +
           (2 * sizeof(int32_t) * kParMaxBudget + 255) / 256 * 256 +
           (sizeof(double) * kParMaxBudget * kScratchStride + 255) / 256 * 256 +
           (sizeof(int32_t) * (4 + kParMaxBudget + 1) + 255) / 256 * 256;
}
static_assert(par_smem_bytes() <= 96 * 1024, "parallel expansion table exceeds its shared-memory share");

__device__ inline ParSmem carve_par(unsigned char* base) {
    ParSmem P;
    size_t o = 0;
    P.score = reinterpret_cast<double*>(base + o);
    o += sizeof(double) * kParNodes;
    P.key = reinterpret_cast<unsigned long long*>(base + o);
    o += sizeof(unsigned long long) * kParNodes;
    P.phi = reinterpret_cast<unsigned long long*>(base + o);
    o += sizeof(unsigned long long) * kParNodes;
    P.plo = reinterpret_cast<unsigned long long*>(base + o);
    o += sizeof(unsigned long long) * kParNodes;
    P.parent = reinterpret_cast<int32_t*>(base + o);
    o += sizeof(int32_t) * kParNodes;
    P.dr = reinterpret_cast<int32_t*>(base + o);
    o += sizeof(int32_t) * kParNodes;
    P.acnt = reinterpret_cast<int32_t*>(base + o);
    o += sizeof(int32_t) * kParNodes;
    P.pos = reinterpret_cast<int32_t*>(base + o);
    o += sizeof(int32_t) * kParNodes;
    o = align256(o);
    P.pool = reinterpret_cast<int32_t*>(base + o);
    P.pool2 = P.pool + kParMaxBudget;
    o = align256(o + 2 * sizeof(int32_t) * kParMaxBudget);
    P.scratch = reinterpret_cast<double*>(base + o);
    o = align256(o + sizeof(double) * kParMaxBudget * kScratchStride);
    P.ctl = reinterpret_cast<int32_t*>(base + o);
    return P;
}

// (key, ranks tuple) order of two (key, hi, lo) triples
__device__ __forceinline__ bool par_before(unsigned long long ka, unsigned long long ha, unsigned long long la,
                                           unsigned long long kb, unsigned long long hb, unsigned long long lb) {
    if (ka != kb) return ka < kb;
    if (ha != hb) return ha < hb;
    return la < lb;
}
__device__ __forceinline__ bool par_node_before(const ParSmem& P, int a, int b) {
    return par_before(P.key[a], P.phi[a], P.plo[a], P.key[b], P.phi[b], P.plo[b]);
}

// Ranks tuple of a node at depth d with rank r under a parent's tuple.
__device__ __forceinline__ void par_path(unsigned long long& h, unsigned long long& l, int d, int r) {
    const unsigned long long f = (unsigned long long)(r + 1);
    if (d <= 9)
        h |= f << (56 - 7 * (d - 1));
    else
        l |= f << (56 - 7 * (d - 10));
}

__device__ __forceinline__ void par_store(const ParSmem& P, int id, double c, unsigned long long h,
                                          unsigned long long l, int parent, int d, int r, int acnt) {
    P.score[id] = c;
    P.key[id] = ord_f64(-c);
    P.phi[id] = h;
    P.plo[id] = l;
    P.parent[id] = parent;
    P.dr[id] = (d << 16) | r;
    P.acnt[id] = acnt;
}

// Scores of the children of pool node `parent` at depth d, best first, into
// out[0..n) while they can still enter the pool (the reference's child and
// sibling recurrences, ddtree.py:171, 176); returns n, or -1 on a step that
// increases the score.  Only the score chain is serial: the entries are
// written afterwards by all threads.
__device__ int par_chain(const ExpandSmem& e, const ParSmem& P, int parent, int d, int topk, int budget, int tau,
                         double* out) {
    const float* row = e.lp + (d - 1) * topk;
    const double S = P.score[parent];
    const int a_p = P.acnt[parent];
    double c = __dadd_rn(S, (double)row[0]);
    if (!(c <= S)) return -1;
    const bool full = tau >= 0;
    unsigned long long th = 0ull, tl = 0ull, tk = 0ull;
    unsigned long long h0 = P.phi[parent], l0 = P.plo[parent];
    if (full) {
        tk = P.key[tau];
        th = P.phi[tau];
        tl = P.plo[tau];
    }
    int n = 0;
    for (int r = 0; r < topk && a_p + 1 + r < budget; ++r) {
        if (full) {
            unsigned long long h = h0, l = l0;
            par_path(h, l, d, r);
            if (!par_before(ord_f64(-c), h, l, tk, th, tl)) break;   // and so every later sibling
        }
        out[r] = c;
        n = r + 1;
        if (r + 1 < topk) {
            const double c2 = __dadd_rn(__dadd_rn(c, -(double)row[r]), (double)row[r + 1]);
            if (!(c2 <= c)) return -1;
            c = c2;
        }
    }
    return n;
}

// Runs on all threads of the CTA; returns the node count, or -1 when the
// serial loop has to run instead.  Fills e.n_parent / e.n_dr like it.
__device__ int expand_par(const ExpandSmem& e, const ParSmem& P, int rows, int topk, int budget) {
    const int tid = threadIdx.x;
    // finite log-probs, and row 0 sorted (the depth-1 scores below rely on it)
    bool bad = false;
    for (int i = tid; i < rows * topk; i += kThreads) {
        const float v = e.lp[i];
        bad |= !(fabsf(v) <= 3.402823466e38f);
        if (i + 1 < topk) bad |= !(e.lp[i + 1] <= v);
    }
    if (__syncthreads_or(bad)) return -1;
    if (tid == 0) P.ctl[2] = 0;
    // Depth 1: the reference's first entry is lp[0,0] and each sibling step
    // fl(fl(S - a_r) + a_{r+1}) with S = a_r gives a_{r+1} exactly, so node r
    // scores lp[0, r]; that order (scores non-increasing, tuples increasing)
    // is already the pop order.
    int np = topk < budget ? topk : budget;
    for (int r = tid; r < np; r += kThreads) {
        unsigned long long h = 0ull, l = 0ull;
        par_path(h, l, 1, r);
        par_store(P, r, (double)e.lp[r], h, l, -1, 1, r, r);
        P.pool[r] = r;
    }
    int nb = np;
    double* scratch = P.scratch;
    int* soff = P.ctl + 4;
    __syncthreads();
    for (int d = 2; d <= rows; ++d) {
        const int tau = np == budget ? P.pool[budget - 1] : -1;
        // (a) each depth-(d-1) pool node's chain, one thread per pool slot
        if (tid < kParMaxBudget) {
            int n = 0;
            if (tid < np) {
                const int id = P.pool[tid];
                if ((P.dr[id] >> 16) == d - 1) n = par_chain(e, P, id, d, topk, budget, tau,
                                                             scratch + tid * kScratchStride);
            }
            if (n < 0) atomicOr(&P.ctl[2], 1);
            soff[tid + 1] = n < 0 ? 0 : n;
        }
        __syncthreads();
        // (b) offsets of the chains (one warp)
        if (tid < 32) {
            const int a = soff[2 * tid + 1], b = soff[2 * tid + 2];
            int s = a + b;
            for (int o = 1; o < 32; o <<= 1) {
                const int v = __shfl_up_sync(DDT_FULL_MASK, s, o);
                if (tid >= o) s += v;
            }
            soff[2 * tid + 1] = s - b;
            soff[2 * tid + 2] = s;
            if (tid == 0) soff[0] = 0;
        }
        __syncthreads();
        if (P.ctl[2]) return -1;
        const int m = soff[kParMaxBudget];
        if (m == 0) break;   // no node at depth d: none deeper either
        if (nb + m > kParNodes) return -1;
        const int ne = nb + m;
        // (c) the new entries, all threads
        for (int x = tid; x < m; x += kThreads) {
            int lo_s = 0, hi_s = kParMaxBudget - 1;   // the slot s with soff[s] <= x < soff[s + 1]
            while (lo_s < hi_s) {
                const int mid = (lo_s + hi_s + 1) >> 1;
                if (soff[mid] <= x)
                    lo_s = mid;
                else
                    hi_s = mid - 1;
            }
            const int r = x - soff[lo_s];
            const int parent = P.pool[lo_s];
            unsigned long long h = P.phi[parent], l = P.plo[parent];
            par_path(h, l, d, r);
            par_store(P, nb + x, scratch[lo_s * kScratchStride + r], h, l, parent, d, r, P.acnt[parent] + 1 + r);
        }
        __syncthreads();
        const int total = np + m;
        for (int x = tid; x < total; x += kThreads) {
            int id, rank;
            if (x < np) {
                id = P.pool[x];
                rank = x;
                for (int j = nb; j < ne; ++j) rank += par_node_before(P, j, id) ? 1 : 0;
            } else {
                id = nb + (x - np);
                int lo_i = 0, hi_i = np;   // pool entries before it (the pool is sorted)
                while (lo_i < hi_i) {
                    const int mid = (lo_i + hi_i) >> 1;
                    if (par_node_before(P, P.pool[mid], id))
                        lo_i = mid + 1;
                    else
                        hi_i = mid;
                }
                rank = lo_i;
                for (int j = nb; j < ne; ++j) rank += (j != id && par_node_before(P, j, id)) ? 1 : 0;
            }
            if (rank < budget) P.pool2[rank] = id;
        }
        __syncthreads();
        np = total < budget ? total : budget;
        for (int x = tid; x < np; x += kThreads) P.pool[x] = P.pool2[x];
        nb = ne;
        __syncthreads();
    }
    // pop order = pool order; a parent's position comes first
    for (int x = tid; x < nb; x += kThreads) P.pos[x] = -1;
    __syncthreads();
    for (int x = tid; x < np; x += kThreads) P.pos[P.pool[x]] = x;
    __syncthreads();
    for (int x = tid; x < np; x += kThreads) {
        const int id = P.pool[x];
        const int par = P.parent[id];
        const int pidx = par < 0 ? 0 : P.pos[par] + 1;
        if (par >= 0 && (P.pos[par] < 0 || P.pos[par] >= x)) atomicOr(&P.ctl[2], 4);
        e.n_parent[x + 1] = pidx;
        e.n_dr[x + 1] = P.dr[id];
    }
    if (tid == 0) {
        e.n_parent[0] = -1;
        e.n_dr[0] = 0;
    }
    __syncthreads();
    return P.ctl[2] ? -1 : np;
}

// Runs on all threads of one CTA.  lp / ids: [rows, topk] in global memory.
__device__ void expand_tree(const float* lp_g, const int64_t* ids_g, int rows, int topk, int budget,
                            const int64_t* root_token, int64_t start, const ddt_tree_outputs out, ExpandSmem e) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    for (int i = tid; i < rows * topk; i += kThreads) e.lp[i] = __ldcg(lp_g + i);
    __syncthreads();

    const int par_count = e.par ? expand_par(e, carve_par(e.par), rows, topk, budget) : -1;
    if (par_count >= 0) {
        if (tid == 0) e.scalars[1] = par_count;
    } else if (warp == 0) {
        int count;
        // before pop t the frontier holds at most t + 1 <= budget entries, so
        // 32 * S >= budget slots suffice; the last pop's appended entry may
        // fall past them and is dropped, as nothing is popped after it
        if (budget <= 32)
            count = expand_regs<1>(e, rows, topk, budget, lane);
        else if (budget <= 64)
            count = expand_regs<2>(e, rows, topk, budget, lane);
        else if (budget <= 96)
            count = expand_regs<3>(e, rows, topk, budget, lane);
        else if (budget <= 128)
            count = expand_regs<4>(e, rows, topk, budget, lane);
        else
            count = expand_smem(e, rows, topk, budget, lane);
        if (lane == 0) e.scalars[1] = count;
    }
    __syncthreads();
    const int n = e.scalars[1];
    int max_depth = 0;
    for (int i = 1 + tid; i <= n; i += kThreads) {
        const int dr = e.n_dr[i];
        const int depth = dr >> 16, rank = dr & 0xffff;
        const int64_t tok = __ldcg(ids_g + (int64_t)(depth - 1) * topk + rank);
        out.node_token_ids[i - 1] = tok;
        out.node_depths[i - 1] = depth;
        if (out.verify_ids) out.verify_ids[i] = tok;
        if (out.verify_pos) out.verify_pos[i] = start + depth;
        max_depth = max(max_depth, depth);
    }
    for (int i = tid; i <= n; i += kThreads) out.parents[i] = e.n_parent[i];
    if (tid == 0) {
        if (out.verify_ids) out.verify_ids[0] = root_token ? *root_token : 0;
        if (out.verify_pos) out.verify_pos[0] = start;
    }
    if (out.visibility) {
        const int W = (int)out.vis_words;
        for (int i = tid; i <= n; i += kThreads) {
            int anc[kMaxRows + 1];
            int na = 0;
            for (int a = i; a >= 0; a = e.n_parent[a]) anc[na++] = a;
            uint32_t* row = out.visibility + (int64_t)i * W;
            for (int wd = 0; wd < W; ++wd) {
                uint32_t bits = 0;
                for (int k = 0; k < na; ++k)
                    if ((anc[k] >> 5) == wd) bits |= 1u << (anc[k] & 31);
                row[wd] = bits;
            }
        }
    }
    // max depth (warp reduce then smem)
    for (int o = 16; o > 0; o >>= 1) max_depth = max(max_depth, __shfl_xor_sync(DDT_FULL_MASK, max_depth, o));
    __syncthreads();
    if (lane == 0) atomicMax(&e.scalars[2], max_depth);
    __syncthreads();
    if (tid == 0 && out.info) {
        out.info[0] = n;
        out.info[1] = e.scalars[2];
        out.info[3] = topk;
    }
}

// ---------------------------------------------------------------------------
// phases A + B (+ C on the last CTA)
// ---------------------------------------------------------------------------
template <typename T, bool kVec>
__global__ void __launch_bounds__(kThreads, 1)
tree_build_kernel(const T* __restrict__ logits, int rows, int64_t vocab, int64_t row_stride, int topk, int chunks,
                  int64_t chunk_len, int budget, const int64_t* root_token, int64_t start, ddt_tree_outputs out,
                  unsigned char* ws, const unsigned char* __restrict__ hstats) {
    extern __shared__ __align__(256) unsigned char smem[];
    __shared__ SelectScratch sel;
    __shared__ unsigned long long s_offer[kWarps];
    __shared__ double red_d[kWarps];
    __shared__ float red_f[kWarps];
    __shared__ int s_flag;

    const WsLayout L = ws_layout(rows, chunks, topk);
    uint32_t* row_cnt = reinterpret_cast<uint32_t*>(ws + L.row_cnt);
    uint32_t* done_cnt = reinterpret_cast<uint32_t*>(ws + L.done_cnt);
    float* part_m = reinterpret_cast<float*>(ws + L.part_m);
    double* part_s = reinterpret_cast<double*>(ws + L.part_s);
    unsigned long long* part_keys = reinterpret_cast<unsigned long long*>(ws + L.part_keys);
    int64_t* top_ids = reinterpret_cast<int64_t*>(ws + L.top_ids);
    float* top_lp = reinterpret_cast<float*>(ws + L.top_lp);

    const int tid = threadIdx.x;
    const int d = blockIdx.y, c = blockIdx.x;
    const T* rowp = logits + (int64_t)d * row_stride;
    const int64_t c0 = (int64_t)c * chunk_len;
    const int64_t c1 = min(c0 + chunk_len, vocab);

    // ---- load the chunk into shared memory -------------------------------
    // Thread tid holds the 16-byte vectors tid, tid + kThreads, ... of the
    // chunk; the values stay in shared memory (chunk-local index) and each
    // thread reads back only its own, in index order, with 16-byte loads (a
    // warp reads 512 consecutive bytes: no bank conflicts).  The passes are
    // rolled loops: this code runs once per CTA, and the same passes fully
    // unrolled over register-held values spent most of their time waiting
    // for instruction fetch.  Slots past the chunk hold -inf.
    constexpr int kEpv = 16 / sizeof(T);          // elements per 16-byte vector
    constexpr int kNv = kValsPerThread / kEpv;    // vectors per thread
    unsigned long long* cand = reinterpret_cast<unsigned long long*>(smem);
    unsigned long long* top = cand + kCandCap;
    float* cv = reinterpret_cast<float*>(top + kMaxBudget);
    const int n_valid = (int)(c1 - c0);
    // Keys are (value order, then lower token id) and distinct.  The chunk's
    // top kc keys go to part_keys in descending order, padded with zeros.
    const int kc = min(topk, n_valid);
    const int lane = tid & 31, warp = tid >> 5;
    unsigned long long* dst = part_keys + ((int64_t)d * chunks + c) * topk;
    auto loc_of = [&](int j) -> int { return ((j / kEpv) * kThreads + tid) * kEpv + (j % kEpv); };
    auto key_at = [&](int j) -> unsigned long long {   // (the rare radix-select path)
        const int loc = loc_of(j);
        return chunk_key(cv[loc], loc, n_valid, c0);
    };
    float m = -INFINITY;
    double sum_c = 0.0;
    int cand_cap = kCandCap;
    if (hstats) {
        // ---- phase A from the draft head's block statistics ---------------
        // (ddt_tree_build_head).  The chunk is a run of whole 128-row blocks.
        // Its max and sum of exp come from the blocks' (max, sum), rescaled
        // in float64.  Its top kc keys lie in the kc blocks with the largest
        // block keys (a block holding a key of the top kc has a block key at
        // least that large; the kc-th largest block key t0 is at most the
        // kc-th largest key, since the kc best blocks hold kc keys >= t0).
        // Those blocks are read from the logits for their keys >= t0: the
        // candidates, few unless many values are equal.  The staging area
        // `cv` is unused in this mode and holds them.
        cand = reinterpret_cast<unsigned long long*>(cv);
        cand_cap = kHeadCandCap;
        const int nblk = (int)(vocab / kHeadBlock);
        const HeadStatsLayout hl = head_stats_layout(rows, nblk);
        const float* hm = reinterpret_cast<const float*>(hstats + hl.m) + (int64_t)d * nblk;
        const float* hs = reinterpret_cast<const float*>(hstats + hl.s) + (int64_t)d * nblk;
        const unsigned long long* hk = reinterpret_cast<const unsigned long long*>(hstats + hl.keys) + (int64_t)d * nblk;
        const int b0 = (int)(c0 / kHeadBlock), b1 = (int)((c1 + kHeadBlock - 1) / kHeadBlock);
        const int nb = b1 - b0;                                   // <= kMaxBudget (host)
        unsigned long long* bkey = top;                           // the chunk's block keys
        int* pick = reinterpret_cast<int*>(top + kMaxBudget / 2); // the blocks to read (<= kc <= 4 * kMaxBudget / 2)
        float mloc = -INFINITY;
        bool nan_l = false;
        for (int b = tid; b < nb; b += kThreads) {
            const float mb = __ldcg(hm + b0 + b);
            nan_l |= mb != mb;
            mloc = fmaxf(mloc, mb);
            bkey[b] = __ldcg(hk + b0 + b);
        }
        if (tid == 0) {
            s_flag = 0;
            sel.count = 0;   // candidates
            sel.need = 0;    // blocks picked
        }
        __syncthreads();
        if (nan_l) s_flag = 1;
        m = block_max(mloc, red_f);
        double sl = 0.0;
        if (m != -INFINITY && m == m) {
            for (int b = b0 + tid; b < b1; b += kThreads) {
                const float mb = __ldcg(hm + b);
                if (mb != -INFINITY) sl += (double)__ldcg(hs + b) * exp((double)mb - (double)m);
            }
        }
        sum_c = block_sum_d(sl, red_d);   // (its barriers order the bkey writes and sel's reset)
        // rank of each block key by counting; the block of rank kc - 1 gives t0
        __shared__ unsigned long long s_t0;
        if (tid == 0) s_t0 = 0ull;
        __syncthreads();
        for (int b = tid; b < nb; b += kThreads) {
            const unsigned long long kb = bkey[b];
            int r = 0;
            for (int q = 0; q < nb; ++q) r += bkey[q] > kb ? 1 : 0;
            if (r < kc) pick[atomicAdd(&sel.need, 1)] = b;
            if (r == kc - 1) s_t0 = kb;
        }
        __syncthreads();
        const unsigned long long t0h = nb > kc ? s_t0 : 0ull;
        const int npick = sel.need;
        const T* rowh = logits + (int64_t)d * row_stride;
        for (int j = warp; j < npick; j += kWarps) {
            const int64_t base = (int64_t)(b0 + pick[j]) * kHeadBlock;
            for (int i = lane; i < kHeadBlock; i += 32) {
                const unsigned long long k = make_key(to_f32<T>(rowh[base + i]), base + i);
                if (k >= t0h) {
                    const int pos = atomicAdd(&sel.count, 1);
                    if (pos < kHeadCandCap) cand[pos] = k;
                }
            }
        }
        __syncthreads();
    } else {
#pragma unroll
    for (int j = 0; j < kNv; ++j) {
        const int loc = (j * kThreads + tid) * kEpv;
        float x[kEpv];
        if (kVec && loc + kEpv <= n_valid) {
            const uint4 raw = __ldcs(reinterpret_cast<const uint4*>(rowp + c0 + loc));
            const T* pv = reinterpret_cast<const T*>(&raw);
#pragma unroll
            for (int e = 0; e < kEpv; ++e) x[e] = to_f32<T>(pv[e]);
        } else {
#pragma unroll
            for (int e = 0; e < kEpv; ++e) x[e] = loc + e < n_valid ? to_f32<T>(rowp[c0 + loc + e]) : -INFINITY;
        }
#pragma unroll
        for (int e = 0; e < kEpv; e += 4)
            *reinterpret_cast<float4*>(cv + loc + e) = make_float4(x[e], x[e + 1], x[e + 2], x[e + 3]);
    }

    // ---- max and sum of exp (logsumexp pieces, ddtree.py:138) ----------
    // (a slot past the chunk adds exp(-inf) = +0 to the sum: no change)
    // The same pass keeps the thread's largest value and its first index
    // (values run in index order, so the lowest index among equal values).
    float best = -INFINITY;
    int bloc = -1;
    bool nan_seen = false;
    DDT_FOR_VALS(x, loc, j, {
        nan_seen |= (x != x);
        m = fmaxf(m, x);
        if (x > best) {
            best = x;
            bloc = loc;
        }
    })
    if (tid == 0) s_flag = 0;
    __syncthreads();
    if (nan_seen) s_flag = 1;
    m = block_max(m, red_f);
    const bool any_nan = s_flag != 0;   // (set before block_max's barriers)
    float sum_t = 0.f;
    if (m != -INFINITY && m == m) {
        DDT_FOR_VALS(x, loc, j, { sum_t += expf(x - m); })
    }
    sum_c = block_sum_d((double)sum_t, red_d);

    // ---- chunk top-k candidates ----------------------------------------
    // The thread's largest key.  Without NaN it is that of its first largest
    // value (up to the order of +0 and -0, which only lowers it: the bound
    // below stays a lower bound, built from keys the thread holds).
    unsigned long long tmax = 0ull;
    if (!any_nan) {
        if (bloc >= 0) tmax = chunk_key(best, bloc, n_valid, c0);
    } else {
        DDT_FOR_VALS(x, loc, j, {
            const unsigned long long k = chunk_key(x, loc, n_valid, c0);
            tmax = k > tmax ? k : tmax;
        })
    }
    if (tid == 0) sel.count = 0;
    __syncthreads();
    // A lower bound t0 on the kc-th largest key: each warp sorts its 32
    // thread maxima (distinct: every thread holds a valid value here) and
    // offers its q-th largest, q = ceil(kc / kWarps); at least q * kWarps >= kc
    // keys are >= the smallest offer, so every key of the top kc is too.
    unsigned long long t0 = 0ull;
    if (n_valid > kCandCap && kc <= kThreads) {
        const int q = (kc + kWarps - 1) / kWarps;
        unsigned long long x = tmax;
#pragma unroll
        for (int k = 2; k <= 32; k <<= 1) {
#pragma unroll
            for (int jj = k >> 1; jj > 0; jj >>= 1) {
                const unsigned long long y = __shfl_xor_sync(DDT_FULL_MASK, x, jj);
                const bool keep_max = ((lane & jj) == 0) == ((lane & k) == 0);
                x = keep_max ? (x > y ? x : y) : (x < y ? x : y);
            }
        }
        const unsigned long long offer = __shfl_sync(DDT_FULL_MASK, x, q - 1);   // lane i: (i+1)-th largest
        if (lane == 0) s_offer[warp] = offer;
        __syncthreads();
        t0 = s_offer[0];
#pragma unroll
        for (int w = 1; w < kWarps; ++w) t0 = s_offer[w] < t0 ? s_offer[w] : t0;
    }
    // gather keys >= t0: each thread counts its own, a warp scan places them,
    // one atomic per warp reserves the warp's slots.  Without NaN and with a
    // bound, the test is on the float value (greater: taken; equal: the key
    // decides, which also orders +0 / -0); else on the key.
    // The thread's candidates are bits of a 64-bit mask over its slots; the
    // write below visits only the set bits.
    const bool by_value = !any_nan && t0 != 0ull;
    const float t0v = key_value(t0);
    unsigned long long cmask = 0ull;
    if (by_value) {
        bool eq = false;
        DDT_FOR_VALS(x, loc, j, {
            cmask |= (unsigned long long)(x > t0v) << j;
            eq |= (x == t0v);
        })
        if (eq) {   // values equal to the bound's: the key decides
            DDT_FOR_VALS(x, loc, j, {
                if (x == t0v && chunk_key(x, loc, n_valid, c0) >= t0) cmask |= 1ull << j;
            })
        }
    } else {
        DDT_FOR_VALS(x, loc, j, {
            const unsigned long long kx = chunk_key(x, loc, n_valid, c0);
            if (kx != 0ull && kx >= t0) cmask |= 1ull << j;
        })
    }
    const int cnt = __popcll(cmask);
    int incl = cnt;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int t = __shfl_up_sync(DDT_FULL_MASK, incl, o);
        if (lane >= o) incl += t;
    }
    int wbase = 0;
    if (lane == 31 && incl > 0) wbase = atomicAdd(&sel.count, incl);
    wbase = __shfl_sync(DDT_FULL_MASK, wbase, 31);
    int pos = wbase + incl - cnt;
    for (unsigned long long mk = cmask; mk; mk &= mk - 1, ++pos) {
        const int loc = loc_of(__ffsll((long long)mk) - 1);
        if (pos < kCandCap) cand[pos] = chunk_key(cv[loc], loc, n_valid, c0);
    }
    __syncthreads();
    }   // phase A from the logits
    const int ncand = sel.count;
    __syncthreads();
    if (tid == 0) sel.count = 0;
    if (ncand <= kRankCap) {
        // few candidates: a candidate's rank is the number of larger ones
        for (int i = tid; i < ncand; i += kThreads) {
            const unsigned long long k = cand[i];
            int r = 0;
            for (int q = 0; q < ncand; ++q) r += cand[q] > k ? 1 : 0;
            if (r < kc) dst[r] = k;
        }
    } else {
        // radix select of the kc-th largest, the selected keys into `top`,
        // then ranked among themselves
        if (ncand <= cand_cap) {
            const unsigned long long t1 = block_kth_largest(cand, ncand, kc, &sel);
            for (int i = tid; i < ncand; i += kThreads) {
                const unsigned long long k = cand[i];
                if (k >= t1) {
                    const int pos = atomicAdd(&sel.count, 1);
                    if (pos < kc) top[pos] = k;
                }
            }
        } else {
            const unsigned long long t1 = block_kth_largest_regs(key_at, kc, &sel);
#pragma unroll
            for (int j = 0; j < kValsPerThread; ++j) {
                const unsigned long long kj = key_at(j);
                if (kj != 0ull && kj >= t1) {
                    const int pos = atomicAdd(&sel.count, 1);
                    if (pos < kc) top[pos] = kj;
                }
            }
        }
        __syncthreads();
        for (int i = tid; i < kc; i += kThreads) {
            const unsigned long long k = top[i];
            int r = 0;
            for (int q = 0; q < kc; ++q) r += top[q] > k ? 1 : 0;
            dst[r] = k;
        }
    }
    for (int i = kc + tid; i < topk; i += kThreads) dst[i] = 0ull;
    if (tid == 0) {
        part_m[d * chunks + c] = s_flag ? __int_as_float(0x7fc00000) : m;
        part_s[d * chunks + c] = sum_c;
    }

    // ---- hand-off to the row merge ---------------------------------------
    // The barrier orders every thread's writes before thread 0's fence and
    // count (the grid-barrier pattern: one fence per CTA, cumulative through
    // the barrier); the CTA that completes the count fences once more
    // before its threads read the other chunks' results.
    __syncthreads();
    if (tid == 0) {
        __threadfence();
        s_flag = (atomicAdd(&row_cnt[d], 1u) == (uint32_t)(chunks - 1)) ? 1 : 0;
        if (s_flag) __threadfence();
    }
    __syncthreads();
    if (!s_flag) return;

    // ---- phase B: merge the row ------------------------------------------
    // Every chunk list is sorted (descending, zero-padded) and the nonzero
    // keys of a row are distinct, so a key's rank in the row is its index in
    // its own list plus, for each other list, the number of its keys above
    // it (a binary search).  Each list lies entirely at or above its last
    // entry, so the largest last entry is at most the row's topk-th key and
    // only keys at or above it are ranked.  Warps 1.. rank; warp 0 computes
    // the log-normaliser meanwhile.
    {
        const int n = chunks * topk;
        unsigned long long* mk = reinterpret_cast<unsigned long long*>(smem);
        unsigned long long* sk = mk + n;
        const unsigned long long* src = part_keys + (int64_t)d * chunks * topk;
        for (int i = tid; i < n; i += kThreads) mk[i] = __ldcg(src + i);
        for (int i = tid; i < topk; i += kThreads) sk[i] = 0ull;
        __syncthreads();
        const int lane_b = tid & 31;
        __shared__ float s_logz;
        if (tid >= 32) {
            unsigned long long lb = 0ull;
            for (int q = 0; q < chunks; ++q) {
                const unsigned long long e = mk[q * topk + topk - 1];
                lb = e > lb ? e : lb;
            }
            for (int i = tid - 32; i < n; i += kThreads - 32) {
                const unsigned long long x = mk[i];
                if (x == 0ull || x < lb) continue;
                const int qx = i / topk;
                int r = i - qx * topk;
                for (int q = 0; q < chunks; ++q) {
                    if (q == qx) continue;
                    const unsigned long long* lst = mk + q * topk;
                    int lo = 0, hi = topk;   // keys of list q above x: a prefix
                    while (lo < hi) {
                        const int mid = (lo + hi) >> 1;
                        if (lst[mid] > x)
                            lo = mid + 1;
                        else
                            hi = mid;
                    }
                    r += lo;
                    if (r >= topk) break;
                }
                if (r < topk) sk[r] = x;
            }
        } else {
            float M = -INFINITY;
            bool nan_row = false;
            for (int q = lane_b; q < chunks; q += 32) {
                const float mq = __ldcg(part_m + d * chunks + q);
                nan_row |= (mq != mq);
                M = fmaxf(M, mq);
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) M = fmaxf(M, __shfl_xor_sync(DDT_FULL_MASK, M, o));
            nan_row = __any_sync(DDT_FULL_MASK, nan_row);
            double S = 0.0;
            if (!nan_row && !isinf(M)) {
                for (int q = lane_b; q < chunks; q += 32) {
                    const float mq = __ldcg(part_m + d * chunks + q);
                    const double sq = __ldcg(part_s + d * chunks + q);
                    if (mq != -INFINITY) S += sq * exp((double)mq - (double)M);
                }
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) S += __shfl_xor_sync(DDT_FULL_MASK, S, o);
            }
            if (lane_b == 0) {
                float lz;
                if (nan_row)
                    lz = __int_as_float(0x7fc00000);
                else if (isinf(M))
                    lz = M;
                else
                    lz = (float)((double)M + log(S));
                s_logz = lz;
                if (!isfinite(lz)) atomicOr(&done_cnt[1], DDT_INFO_NONFINITE);
            }
        }
        __syncthreads();
        const float lz = s_logz;
        bool bad = false;
        for (int i = tid; i < topk; i += kThreads) {
            const unsigned long long k = sk[i];
            const float v = key_value(k);
            const float lp = __fsub_rn(v, lz);
            bad |= !isfinite(lp);
            const int64_t id = key_index(k);
            top_ids[(int64_t)d * topk + i] = id;
            top_lp[(int64_t)d * topk + i] = lp;
            if (out.top_ids) out.top_ids[(int64_t)d * topk + i] = id;
            if (out.top_lp) out.top_lp[(int64_t)d * topk + i] = lp;
        }
        if (bad) atomicOr(&done_cnt[1], DDT_INFO_NONFINITE);
    }
    __syncthreads();   // (the same one-fence hand-off as above)
    if (tid == 0) {
        row_cnt[d] = 0u;
        __threadfence();
        s_flag = (atomicAdd(&done_cnt[0], 1u) == (uint32_t)(rows - 1)) ? 1 : 0;
        if (s_flag) __threadfence();
    }
    __syncthreads();
    if (!s_flag) return;

    // ---- phase C: expansion on the last CTA --------------------------------
    ExpandSmem e = carve_expand(smem, rows, topk, budget);
    if (tid == 0) {
        e.scalars[2] = 0;
    }
    __syncthreads();
    expand_tree(top_lp, top_ids, rows, topk, budget, root_token, start, out, e);
    if (tid == 0) {
        if (out.info) out.info[2] = (int32_t)atomicExch(&done_cnt[1], 0u);
        done_cnt[0] = 0u;
    }
}

// Expansion alone from given (lp, ids).
__global__ void __launch_bounds__(kThreads, 1)
tree_expand_kernel(const float* lp, const int64_t* ids, int rows, int topk, int budget, const int64_t* root_token,
                   int64_t start, ddt_tree_outputs out) {
    extern __shared__ __align__(256) unsigned char smem[];
    ExpandSmem e = carve_expand(smem, rows, topk, budget);
    if (threadIdx.x == 0) e.scalars[2] = 0;
    __syncthreads();
    expand_tree(lp, ids, rows, topk, budget, root_token, start, out, e);
    if (threadIdx.x == 0 && out.info) out.info[2] = 0;
}

// Root-only tree (budget <= 0 or no draft rows, ddtree.py:120-130).
__global__ void tree_root_only_kernel(const int64_t* root_token, int64_t start, ddt_tree_outputs out) {
    out.parents[0] = -1;
    if (out.visibility) {
        out.visibility[0] = 1u;
        for (int w = 1; w < out.vis_words; ++w) out.visibility[w] = 0u;
    }
    if (out.verify_ids) out.verify_ids[0] = root_token ? *root_token : 0;
    if (out.verify_pos) out.verify_pos[0] = start;
    if (out.info) {
        out.info[0] = 0;
        out.info[1] = 0;
        out.info[2] = 0;
        out.info[3] = 0;
    }
}

}  // namespace tree
}  // namespace ddt

using namespace ddt;
using namespace ddt::tree;

static size_t phase_smem(int64_t rows, int64_t chunks, int64_t topk, int64_t budget) {
    // phase A: candidates, selected keys, the chunk's values
    size_t a = sizeof(uint64_t) * (kCandCap + kMaxBudget) + sizeof(float) * kMaxChunk;
    size_t b = sizeof(uint64_t) * (2 * chunks * topk + topk);
    size_t c = expand_smem_bytes(rows, topk, budget);
    size_t m = a > b ? a : b;
    return m > c ? m : c;
}

static int validate_outputs(const ddt_tree_outputs* out, int64_t budget) {
    if (!out) return set_error(DDT_EINVAL, "tree outputs struct is null");
    if (budget > 0 && (!out->node_token_ids || !out->node_depths))
        return set_error(DDT_EINVAL, "node_token_ids / node_depths are required");
    if (!out->parents) return set_error(DDT_EINVAL, "parents is required");
    if (out->visibility && out->vis_words < ceil_div(budget + 1, 32))
        return set_error(DDT_EINVAL, "vis_words %lld < ceil((budget+1)/32)", (long long)out->vis_words);
    return DDT_OK;
}

extern "C" size_t ddt_tree_build_workspace_size(int64_t rows, int64_t vocab, int64_t budget) {
    if (rows <= 0 || vocab <= 0 || budget <= 0) return 256;
    int dev = 0;
    cudaGetDevice(&dev);
    const int sms = ddt_sm_count(dev);
    const int64_t topk = budget < vocab ? budget : vocab;
    int64_t chunks, len;
    choose_chunks(rows, vocab, topk, sms > 0 ? sms : 148, &chunks, &len);
    // sized for the largest chunk count any device could pick
    int64_t chunks_max, len2;
    choose_chunks(rows, vocab, topk, 1024, &chunks_max, &len2);
    if (chunks_max < chunks) chunks_max = chunks;
    return ws_layout(rows, chunks_max, topk).total;
}

static int tree_build_run(const void* logits, int dtype, int64_t rows, int64_t vocab, int64_t row_stride,
                          int64_t budget, const int64_t* root_token, int64_t start, const ddt_tree_outputs* out,
                          void* workspace, size_t workspace_bytes, ddt_stream_t stream,
                          const unsigned char* hstats);

extern "C" int ddt_tree_build(const void* logits, int dtype, int64_t rows, int64_t vocab, int64_t row_stride,
                              int64_t budget, const int64_t* root_token, int64_t start, const ddt_tree_outputs* out,
                              void* workspace, size_t workspace_bytes, ddt_stream_t stream) {
    return tree_build_run(logits, dtype, rows, vocab, row_stride, budget, root_token, start, out, workspace,
                          workspace_bytes, stream, nullptr);
}

extern "C" int ddt_tree_build_head(const void* logits, int64_t rows, int64_t vocab, int64_t row_stride,
                                   const void* head_stats, int64_t budget, const int64_t* root_token, int64_t start,
                                   const ddt_tree_outputs* out, void* workspace, size_t workspace_bytes,
                                   ddt_stream_t stream) {
    if (budget > 0 && rows > 0) {
        if (!head_stats) return set_error(DDT_EINVAL, "head_stats is null");
        if (vocab % kHeadBlock) return set_error(DDT_EINVAL, "vocab=%lld is not a multiple of %d", (long long)vocab,
                                                 kHeadBlock);
        if (reinterpret_cast<uintptr_t>(head_stats) % 256)
            return set_error(DDT_EINVAL, "head_stats must be 256-byte aligned");
    }
    return tree_build_run(logits, DDT_BF16, rows, vocab, row_stride, budget, root_token, start, out, workspace,
                          workspace_bytes, stream, static_cast<const unsigned char*>(head_stats));
}

static int tree_build_run(const void* logits, int dtype, int64_t rows, int64_t vocab, int64_t row_stride,
                          int64_t budget, const int64_t* root_token, int64_t start, const ddt_tree_outputs* out,
                          void* workspace, size_t workspace_bytes, ddt_stream_t stream,
                          const unsigned char* hstats) {
    int rc = validate_outputs(out, budget);
    if (rc) return rc;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    if (budget <= 0 || rows == 0) {
        tree_root_only_kernel<<<1, 1, 0, st>>>(root_token, start, *out);
        return check_launch("tree_root_only_kernel");
    }
    if (!logits) return set_error(DDT_EINVAL, "logits is null");
    if (rows < 0 || rows > kMaxRows) return set_error(DDT_EUNSUPPORTED, "rows=%lld outside [0, %d]", (long long)rows, kMaxRows);
    if (vocab <= 0 || vocab >= (int64_t)1 << 31) return set_error(DDT_EINVAL, "vocab=%lld", (long long)vocab);
    if (budget > kMaxBudget) return set_error(DDT_EUNSUPPORTED, "budget=%lld > %d", (long long)budget, kMaxBudget);
    if (row_stride < vocab) return set_error(DDT_EINVAL, "row_stride < vocab");
    if (dtype != DDT_F32 && dtype != DDT_BF16 && dtype != DDT_F16) return set_error(DDT_EINVAL, "dtype %d", dtype);
    int dev = 0;
    cudaGetDevice(&dev);
    const int sms = ddt_sm_count(dev);
    const int64_t topk = budget < vocab ? budget : vocab;
    int64_t chunks, chunk_len;
    choose_chunks(rows, vocab, topk, sms, &chunks, &chunk_len);
    if (hstats) {
        // whole 128-row blocks per chunk (never more chunks than above, so
        // ddt_tree_build_workspace_size covers this mode too); the topk
        // blocks read from the logits must fit the candidate area
        const int64_t nblk = vocab / kHeadBlock;
        const int64_t bpc = ceil_div(nblk, chunks);
        chunk_len = bpc * kHeadBlock;
        chunks = ceil_div(nblk, bpc);
        if (topk * kHeadBlock > kHeadCandCap || bpc > kMaxBudget / 2)
            return set_error(DDT_EUNSUPPORTED, "ddt_tree_build_head: budget %lld (top-k %lld) or %lld blocks per "
                             "chunk beyond its limits (%d, %d); use ddt_tree_build", (long long)budget,
                             (long long)topk, (long long)bpc, kHeadCandCap / kHeadBlock, kMaxBudget / 2);
    }
    const WsLayout L = ws_layout(rows, chunks, topk);
    if (!workspace || workspace_bytes < L.total)
        return set_error(DDT_EWORKSPACE, "tree build workspace needs %zu bytes, got %zu", L.total, workspace_bytes);
    if (reinterpret_cast<uintptr_t>(workspace) % 256) return set_error(DDT_EINVAL, "workspace must be 256-byte aligned");
    const size_t smem = phase_smem(rows, chunks, topk, budget);
    if (smem > 227 * 1024) return set_error(DDT_EUNSUPPORTED, "tree build needs %zu bytes of shared memory", smem);
    const size_t esz = dtype == DDT_F32 ? 4 : 2;
    const bool vec = (reinterpret_cast<uintptr_t>(logits) % 16 == 0) && ((row_stride * esz) % 16 == 0);
    dim3 grid((unsigned)chunks, (unsigned)rows);
    unsigned char* ws = static_cast<unsigned char*>(workspace);
#define DDT_LAUNCH_TB(T, V)                                                                                        \
    do {                                                                                                           \
        auto k = tree_build_kernel<T, V>;                                                                          \
        if (cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)        \
            return check_launch("cudaFuncSetAttribute(tree_build_kernel)");                                        \
        k<<<grid, kThreads, smem, st>>>(static_cast<const T*>(logits), (int)rows, vocab, row_stride, (int)topk,    \
                                        (int)chunks, chunk_len, (int)budget, root_token, start, *out, ws, hstats); \
    } while (0)
    if (dtype == DDT_F32) {
        if (vec) DDT_LAUNCH_TB(float, true); else DDT_LAUNCH_TB(float, false);
    } else if (dtype == DDT_BF16) {
        if (vec) DDT_LAUNCH_TB(__nv_bfloat16, true); else DDT_LAUNCH_TB(__nv_bfloat16, false);
    } else {
        if (vec) DDT_LAUNCH_TB(__half, true); else DDT_LAUNCH_TB(__half, false);
    }
#undef DDT_LAUNCH_TB
    return check_launch("tree_build_kernel");
}

extern "C" int ddt_tree_from_log_probs(const float* lp, const int64_t* ids, int64_t rows, int64_t topk,
                                       int64_t budget, const int64_t* root_token, int64_t start,
                                       const ddt_tree_outputs* out, ddt_stream_t stream) {
    int rc = validate_outputs(out, budget);
    if (rc) return rc;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    if (budget <= 0 || rows == 0) {
        tree_root_only_kernel<<<1, 1, 0, st>>>(root_token, start, *out);
        return check_launch("tree_root_only_kernel");
    }
    if (!lp || !ids) return set_error(DDT_EINVAL, "lp / ids are null");
    if (rows < 0 || rows > kMaxRows) return set_error(DDT_EUNSUPPORTED, "rows=%lld outside [0, %d]", (long long)rows, kMaxRows);
    if (topk <= 0 || topk > 0xffff) return set_error(DDT_EINVAL, "topk=%lld", (long long)topk);
    if (budget > kMaxBudget) return set_error(DDT_EUNSUPPORTED, "budget=%lld > %d", (long long)budget, kMaxBudget);
    const size_t smem = expand_smem_bytes(rows, topk, budget);
    if (smem > 227 * 1024) return set_error(DDT_EUNSUPPORTED, "expansion needs %zu bytes of shared memory", smem);
    if (cudaFuncSetAttribute(tree_expand_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
        return check_launch("cudaFuncSetAttribute(tree_expand_kernel)");
    tree_expand_kernel<<<1, kThreads, smem, st>>>(lp, ids, (int)rows, (int)topk, (int)budget, root_token, start, *out);
    return check_launch("tree_expand_kernel");
}

// ---------------------------------------------------------------------------
// Tree build for callers that cannot allocate device memory.
//
// Some callers of this library cannot call cudaMalloc: a plugin that is
// handed only its input and output buffers, or a host application whose
// device memory is owned by another allocator (a serving framework's memory
// pool, a game engine budget) and that must not grow it behind that
// allocator's back.  For them
// ddt_tree_build_noalloc runs the same kernel as ddt_tree_build, with its
// scratch in a fixed 1 MiB array that lives in this library's device image.
// Every GPU that loads the library holds that MiB until the process exits.
// 1 MiB covers 15 draft rows x 151936 vocabulary up to a node budget of 512;
// larger shapes are rejected with DDT_EUNSUPPORTED.
// ---------------------------------------------------------------------------
namespace ddt {
namespace tree {

constexpr size_t kNoAllocScratchBytes = size_t(1) << 20;
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

// Device address of g_noalloc_scratch on `dev`.  In host code the symbol is
// only a host-side stand-in, so the address is looked up with
// cudaGetSymbolAddress once per device (with that device current) and cached.
static int noalloc_scratch(int dev, void** out) {
    static std::mutex mu;
    static void* addr[64] = {nullptr};
    if (dev < 0 || dev >= 64) return set_error(DDT_EUNSUPPORTED, "device %d out of range", dev);
    std::lock_guard<std::mutex> lock(mu);
    if (!addr[dev]) {
        void* p = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess || !p) {
            cudaGetLastError();
            return set_error(DDT_ECUDA, "cudaGetSymbolAddress(no-alloc scratch): %s", cudaGetErrorString(e));
        }
        addr[dev] = p;
    }
    *out = addr[dev];
    return DDT_OK;
}

}  // namespace tree
}  // namespace ddt

extern "C" int ddt_tree_build_noalloc(const void* logits, int dtype, int64_t rows, int64_t vocab, int64_t row_stride,
                                      int64_t budget, const int64_t* root_token, int64_t start,
                                      const ddt_tree_outputs* out, ddt_stream_t stream) {
    if (budget > 0 && rows > 0 && vocab > 0 && rows <= kMaxRows) {
        int dev = 0;
        cudaGetDevice(&dev);
        const int64_t topk = budget < vocab ? budget : vocab;
        int64_t chunks, chunk_len;
        choose_chunks(rows, vocab, topk, ddt_sm_count(dev), &chunks, &chunk_len);
        const size_t need = ws_layout(rows, chunks, topk).total;
        if (need > kNoAllocScratchBytes)
            return set_error(DDT_EUNSUPPORTED,
                             "ddt_tree_build_noalloc: rows=%lld vocab=%lld budget=%lld needs %zu bytes of scratch, "
                             "more than its fixed %zu; use ddt_tree_build with a caller workspace",
                             (long long)rows, (long long)vocab, (long long)budget, need, kNoAllocScratchBytes);
    }
    int dev = 0;
    cudaGetDevice(&dev);
    void* scratch = nullptr;
    int rc = noalloc_scratch(dev, &scratch);
    if (rc) return rc;
    // The array keeps whatever the previous call left.  The kernel's
    // hand-off counters and error flags (the first 512 bytes) must start at
    // zero, so they are cleared on the caller's stream before every launch.
    if (cudaMemsetAsync(scratch, 0, 512, reinterpret_cast<cudaStream_t>(stream)) != cudaSuccess)
        return check_launch("cudaMemsetAsync(no-alloc scratch)");
    return ddt_tree_build(logits, dtype, rows, vocab, row_stride, budget, root_token, start, out, scratch,
                          kNoAllocScratchBytes, stream);
}
