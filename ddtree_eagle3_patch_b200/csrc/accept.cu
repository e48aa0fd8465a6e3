// Kernel (3): greedy acceptance and KV-cache compaction on sm_100a.
//
// accept:  row-wise argmax of the verify logits (model/utils.py:28-30) with
//          (rows x chunks) CTAs streaming the logits once with 16-byte
//          loads; each CTA folds its chunk winner into its row's 64-bit word
//          (atomicMax), and the last CTA of the launch decodes every row,
//          then walks the tree (ddtree.py:290-301) or evaluates the EAGLE3
//          paths (eagle3.py:46-79).
// compact: one launch moves the accepted rows of every cache tensor
//          (ddtree.py:61-88, 304-369), staging reads in shared memory before
//          any write so the in-place gather matches index_select + copy_.

#include "common.cuh"

namespace ddt {
namespace accept {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kMaxNodes = 2048;

// argmax key: value order (NaN above everything, -0 == +0), then lower index.
__device__ __forceinline__ unsigned long long argmax_key(float v, int64_t idx) {
    uint32_t o;
    if (v != v) {
        o = 0xffffffffu;
    } else {
        if (v == 0.0f) v = 0.0f;
        o = ord_f32(v);
    }
    return ((unsigned long long)o << 32) | (unsigned long long)(0xffffffffu - (uint32_t)idx);
}

__device__ __forceinline__ unsigned long long warp_max_u64(unsigned long long k) {
    const uint32_t hi = __reduce_max_sync(DDT_FULL_MASK, (uint32_t)(k >> 32));
    const uint32_t lo = __reduce_max_sync(DDT_FULL_MASK, ((uint32_t)(k >> 32) == hi) ? (uint32_t)k : 0u);
    return ((unsigned long long)hi << 32) | lo;
}

// Workspace layout.  The per-row winner words and the counter sit at fixed
// offsets for every shape (never data in another call's layout), so a
// zero-filled workspace stays valid across calls of any shape: every
// completed call leaves them at zero again.
constexpr int64_t kMaxRowsPerLaunch = 4096;
struct WsLayout {
    size_t row_best, done_cnt, post, total;
};
__host__ __device__ inline size_t align256(size_t x) { return (x + 255) & ~size_t(255); }
__host__ __device__ inline WsLayout ws_layout(int64_t rows) {
    WsLayout w;
    w.row_best = 0;
    w.done_cnt = sizeof(unsigned long long) * kMaxRowsPerLaunch;
    size_t o = align256(w.done_cnt + sizeof(uint32_t) * 4);
    w.post = o;
    o = align256(o + sizeof(int64_t) * rows);
    w.total = o;
    return w;
}

// Chunks per row: as many CTAs as fit on the GPU at once (one wave),
// chunks of at least 4096 elements.
__host__ inline int64_t choose_chunks(int64_t rows, int64_t vocab, int64_t resident_ctas) {
    int64_t want = resident_ctas / rows;
    int64_t cap = ceil_div(vocab, 4096);
    int64_t c = want < cap ? want : cap;
    return c < 1 ? 1 : c;
}

// Shared memory of the walk: node tokens and posterior (int64), parents
// (int32), one entry per verify row.
struct WalkSmem {
    int64_t* tok;
    int64_t* post;
    int32_t* par;
};
__host__ __device__ inline size_t walk_smem_bytes(int64_t n_rows) {
    return (2 * sizeof(int64_t) + sizeof(int32_t)) * (size_t)n_rows;
}
__device__ inline WalkSmem carve_walk(unsigned char* smem, int64_t n_rows) {
    WalkSmem w;
    w.tok = reinterpret_cast<int64_t*>(smem);
    w.post = w.tok + n_rows;
    w.par = reinterpret_cast<int32_t*>(w.post + n_rows);
    return w;
}
__host__ inline int64_t chunk_len_for(int64_t vocab, int64_t chunks) {
    int64_t len = ceil_div(vocab, chunks);
    return (len + 7) & ~int64_t(7);
}

enum Mode { kArgmaxOnly = 0, kTreeWalk = 1, kEagle3 = 2 };

struct TailArgs {
    // tree walk
    const int32_t* parents;
    const int64_t* node_tokens;
    const int32_t* n_nodes_dev;
    int64_t* accepted;
    int64_t max_accept;
    int64_t* accept_info;
    // eagle3
    const int64_t* draft_tokens;
    const int64_t* retrieve;
    int64_t leaves, width;
    int64_t* e3_info;
    int64_t* e3_accepted;
};

// The walk (ddtree.py:290-301).  Parents, node tokens and the posterior go
// to shared memory first (the posterior may already be there), so no step
// waits on a global load.
__device__ void tree_walk(const int64_t* post, int64_t n_rows, const TailArgs& a, unsigned char* smem,
                          bool post_in_smem) {
    const WalkSmem w = carve_walk(smem, n_rows);
    int64_t* s_tok = w.tok;
    int64_t* s_post = w.post;
    int32_t* s_par = w.par;
    int n = (int)(n_rows - 1);
    if (a.n_nodes_dev) n = min(n, (int)*a.n_nodes_dev);
    n = min(n, kMaxNodes - 1);
    for (int i = threadIdx.x; i <= n; i += kThreads) {
        s_par[i] = i == 0 ? -1 : __ldcg(a.parents + i);
        s_tok[i] = i == 0 ? -1 : __ldcg(a.node_tokens + i - 1);
        if (!post_in_smem) s_post[i] = __ldcg(post + i);
    }
    __syncthreads();
    if (threadIdx.x < 32) {
        const int lane = threadIdx.x;
        int cur = 0;
        int64_t nxt = s_post[0];
        int64_t count = 1;
        if (lane == 0 && a.max_accept > 0) a.accepted[0] = 0;
        for (;;) {
            int child = -1;
            for (int base = 1; base <= n; base += 32) {
                const int j = base + lane;
                const bool hit = j <= n && s_par[j] == cur && s_tok[j] == nxt;
                const uint32_t b = __ballot_sync(DDT_FULL_MASK, hit);
                if (b) {
                    child = base + __ffs(b) - 1;
                    break;
                }
            }
            if (child < 0) break;
            cur = child;
            if (lane == 0 && count < a.max_accept) a.accepted[count] = cur;
            count += 1;
            nxt = s_post[cur];
        }
        if (lane == 0) {
            a.accept_info[0] = count;
            a.accept_info[1] = nxt;
        }
    }
}

__device__ void eagle3_eval(const int64_t* post, const TailArgs& a, unsigned char* smem) {
    __shared__ unsigned long long s_best;
    if (threadIdx.x == 0) s_best = 0ull;
    __syncthreads();
    unsigned long long mine = 0ull;
    for (int64_t l = threadIdx.x; l < a.leaves; l += kThreads) {
        const int64_t* r = a.retrieve + l * a.width;
        int64_t len = 0;
        for (int64_t w = 0; w + 1 < a.width; ++w) {
            const int64_t nxt = r[w + 1];
            if (nxt < 0) break;
            const int64_t g = r[w] < 0 ? 0 : r[w];
            if (a.draft_tokens[nxt] != __ldcg(post + g)) break;
            len += 1;
        }
        // larger length first, then lower leaf index (first argmax)
        const unsigned long long k =
            ((unsigned long long)(len + 1) << 32) | (unsigned long long)(0xffffffffu - (uint32_t)l);
        mine = k > mine ? k : mine;
    }
    mine = warp_max_u64(mine);
    if ((threadIdx.x & 31) == 0) atomicMax(&s_best, mine);
    __syncthreads();
    if (threadIdx.x == 0) {
        const unsigned long long k = s_best;
        int64_t len = (int64_t)(k >> 32) - 1;
        int64_t best = (int64_t)(0xffffffffu - (uint32_t)(k & 0xffffffffu));
        if (len <= 0) {
            len = 0;
            best = 0;
        }
        for (int64_t w = 0; w <= len; ++w) a.e3_accepted[w] = a.retrieve[best * a.width + w];
        a.e3_info[0] = best;
        a.e3_info[1] = len;
        a.e3_info[2] = __ldcg(post + a.retrieve[best * a.width + len]);
        a.e3_info[3] = 0;
    }
}

template <typename T, bool kVec>
__global__ void __launch_bounds__(kThreads)
argmax_kernel(const T* __restrict__ logits, int64_t n_rows, int64_t vocab, int64_t row_stride, int64_t chunk_len,
              int64_t* posterior, unsigned char* ws, int mode, TailArgs tail) {
    extern __shared__ __align__(16) unsigned char smem[];
    __shared__ unsigned long long s_red[kWarps];
    __shared__ int s_flag;
    const WsLayout L = ws_layout(n_rows);
    unsigned long long* row_best = reinterpret_cast<unsigned long long*>(ws + L.row_best);
    uint32_t* done_cnt = reinterpret_cast<uint32_t*>(ws + L.done_cnt);
    int64_t* post = reinterpret_cast<int64_t*>(ws + L.post);

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int64_t r = blockIdx.y;
    const int c = blockIdx.x;
    const T* rowp = logits + r * row_stride;
    const int64_t c0 = (int64_t)c * chunk_len;
    const int64_t c1 = min(c0 + chunk_len, vocab);
    constexpr int kEpv = 16 / sizeof(T);

    unsigned long long best = 0ull;
    const int64_t step = (int64_t)kThreads * kEpv;
    int64_t base = c0 + (int64_t)tid * kEpv;
    auto scan_vec = [&](const uint4& raw, int64_t b) {
        const T* pv = reinterpret_cast<const T*>(&raw);
#pragma unroll
        for (int e = 0; e < kEpv; ++e) {
            const unsigned long long k = argmax_key(to_f32<T>(pv[e]), b + e);
            best = k > best ? k : best;
        }
    };
    if (kVec) {
        // batches of eight independent 16-byte loads per thread (the scan is
        // bound by memory latency otherwise), then one predicated batch for
        // the rest of this thread's whole vectors and at most one partial
        // vector; the max is order-independent
        // A full batch first takes its float max; v * 0 turns NaN when any
        // element is NaN or infinite, and such a batch takes the exact key
        // path.  Otherwise the batch can only win with a larger value (this
        // thread's earlier batches hold lower indices), and only then is the
        // lowest index holding the max looked up.
        constexpr int U = 8;
        for (; base + (U - 1) * step + kEpv <= c1; base += U * step) {
            uint4 raw[U];
#pragma unroll
            for (int u = 0; u < U; ++u) raw[u] = __ldcs(reinterpret_cast<const uint4*>(rowp + base + u * step));
            float bmax = -INFINITY, inf_nan = 0.f;
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const T* pv = reinterpret_cast<const T*>(&raw[u]);
#pragma unroll
                for (int e = 0; e < kEpv; ++e) {
                    const float v = to_f32<T>(pv[e]);
                    bmax = fmaxf(bmax, v);
                    inf_nan = fmaf(v, 0.f, inf_nan);
                }
            }
            if (inf_nan != inf_nan) {
#pragma unroll
                for (int u = 0; u < U; ++u) scan_vec(raw[u], base + u * step);
            } else if (ord_f32(bmax == 0.f ? 0.f : bmax) > (uint32_t)(best >> 32)) {
                int64_t first = base;
#pragma unroll
                for (int u = U - 1; u >= 0; --u) {
                    const T* pv = reinterpret_cast<const T*>(&raw[u]);
#pragma unroll
                    for (int e = kEpv - 1; e >= 0; --e)
                        if (to_f32<T>(pv[e]) == bmax) first = base + u * step + e;
                }
                best = argmax_key(bmax, first);
            }
        }
        uint4 raw[U];
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int64_t b = base + u * step;
            raw[u] = b + kEpv <= c1 ? __ldcs(reinterpret_cast<const uint4*>(rowp + b)) : make_uint4(0u, 0u, 0u, 0u);
        }
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int64_t b = base + u * step;
            if (b + kEpv <= c1) {
                scan_vec(raw[u], b);
            } else if (b < c1) {
                for (int64_t i = b; i < c1; ++i) {
                    const unsigned long long k = argmax_key(to_f32<T>(rowp[i]), i);
                    best = k > best ? k : best;
                }
            }
        }
    } else {
        for (int64_t i = c0 + tid; i < c1; i += kThreads) {
            const unsigned long long k = argmax_key(to_f32<T>(rowp[i]), i);
            best = k > best ? k : best;
        }
    }
    best = warp_max_u64(best);
    if (lane == 0) s_red[warp] = best;
    __syncthreads();
    // one hand-off: the CTA's winner goes into its row's word, and the last
    // CTA of the launch decodes every row
    if (tid == 0) {
        unsigned long long k = 0ull;
        for (int w = 0; w < kWarps; ++w) k = s_red[w] > k ? s_red[w] : k;
        atomicMax(&row_best[r], k);
        __threadfence();
        s_flag = (atomicAdd(&done_cnt[0], 1u) == gridDim.x * gridDim.y - 1) ? 1 : 0;
    }
    __syncthreads();
    if (!s_flag) return;
    __threadfence();
    int64_t* s_post = mode == kTreeWalk ? carve_walk(smem, n_rows).post : nullptr;
    for (int64_t q = tid; q < n_rows; q += kThreads) {
        const unsigned long long k = atomicExch(&row_best[q], 0ull);   // read, and reset for the next call
        const int64_t idx = (int64_t)(0xffffffffu - (uint32_t)(k & 0xffffffffu));
        post[q] = idx;
        if (posterior) posterior[q] = idx;
        if (s_post) s_post[q] = idx;
    }
    if (tid == 0) done_cnt[0] = 0u;
    if (mode == kArgmaxOnly) return;
    __syncthreads();
    if (mode == kTreeWalk)
        tree_walk(post, n_rows, tail, smem, true);
    else
        eagle3_eval(post, tail, smem);
}

// Walk alone, from a posterior already on the device (ddtree.py:290-301).
__global__ void __launch_bounds__(kThreads) tree_walk_kernel(const int64_t* posterior, int64_t n_rows, TailArgs tail) {
    extern __shared__ __align__(16) unsigned char smem[];
    tree_walk(posterior, n_rows, tail, smem, false);
}

// ---------------------------------------------------------------------------
// commit (ddtree.py:534-548)
// ---------------------------------------------------------------------------
// CTA i copies hidden row accepted[i] to hidden_out row i (when i is below
// the accepted count); CTA 0 also writes the accepted tokens and the bonus
// token into output_ids.  The count and the bonus token are read from
// accept_info on the device.  Writes at or past output_len and accepted
// indices outside [0, n_rows) are skipped.
__global__ void __launch_bounds__(kThreads)
commit_kernel(const int64_t* __restrict__ verify_ids, int64_t n_rows, const int64_t* __restrict__ accepted,
              int64_t max_accept, const int64_t* __restrict__ accept_info, int64_t* output_ids, int64_t output_len,
              int64_t start, const unsigned char* __restrict__ hidden, int64_t hidden_stride, int64_t row_bytes,
              unsigned char* hidden_out, int64_t out_stride) {
    int64_t count = accept_info[0];
    if (count > max_accept) count = max_accept;
    if (count < 0) count = 0;
    const int64_t i = blockIdx.x;
    if (i == 0) {
        for (int64_t t = threadIdx.x; t < count; t += kThreads) {
            const int64_t row = accepted[t];
            if (row >= 0 && row < n_rows && start + t < output_len) output_ids[start + t] = verify_ids[row];
        }
        if (threadIdx.x == 0 && start + count < output_len) output_ids[start + count] = accept_info[1];
    }
    if (!hidden || i >= count) return;
    const int64_t row = accepted[i];
    if (row < 0 || row >= n_rows) return;
    const unsigned char* src = hidden + row * hidden_stride;
    unsigned char* dst = hidden_out + i * out_stride;
    const bool vec = ((reinterpret_cast<uintptr_t>(src) | reinterpret_cast<uintptr_t>(dst) | (uintptr_t)row_bytes) & 15) == 0;
    if (vec) {
        for (int64_t b = (int64_t)threadIdx.x * 16; b < row_bytes; b += (int64_t)kThreads * 16)
            *reinterpret_cast<uint4*>(dst + b) = __ldg(reinterpret_cast<const uint4*>(src + b));
    } else {
        for (int64_t b = threadIdx.x; b < row_bytes; b += kThreads) dst[b] = src[b];
    }
}

// ---------------------------------------------------------------------------
// compaction
// ---------------------------------------------------------------------------
constexpr int kCompactThreads = 256;
constexpr int kStageBytes = 32 * 1024;

__global__ void __launch_bounds__(kCompactThreads)
kv_compact_kernel(void* const* tensors, int64_t heads, int64_t row_bytes, int64_t head_stride, int64_t row_stride,
                  int64_t past, int64_t cur_len, const int64_t* keep, const int64_t* keep_count_dev,
                  int64_t max_keep) {
    __shared__ __align__(16) unsigned char stage[kStageBytes];
    int64_t count = *keep_count_dev;
    if (count <= 0 || count == cur_len) return;  // ddtree.py:80-81
    if (count > max_keep) count = max_keep;
    const int64_t t = blockIdx.x / heads, h = blockIdx.x % heads;
    unsigned char* base = static_cast<unsigned char*>(tensors[t]) + h * head_stride + past * row_stride;
    const bool vec = ((reinterpret_cast<uintptr_t>(base) | (uintptr_t)row_bytes | (uintptr_t)row_stride) & 15) == 0;
    // slabs of columns so that count * slab fits the stage buffer
    int64_t slab = row_bytes;
    while (slab > 16 && count * slab > kStageBytes) slab = (slab + 1) / 2;
    if (vec) slab = (slab + 15) & ~int64_t(15);
    if (count * slab > kStageBytes) return;  // host validation keeps count * 16 <= stage
    for (int64_t s0 = 0; s0 < row_bytes; s0 += slab) {
        const int64_t w = min(slab, row_bytes - s0);
        if (vec) {
            const int64_t nv = w / 16;
            for (int64_t i = threadIdx.x; i < count * nv; i += kCompactThreads) {
                const int64_t k = i / nv, v = i % nv;
                const int64_t src = __ldg(keep + k);
                *reinterpret_cast<uint4*>(stage + k * w + v * 16) =
                    *reinterpret_cast<const uint4*>(base + src * row_stride + s0 + v * 16);
            }
            __syncthreads();
            for (int64_t i = threadIdx.x; i < count * nv; i += kCompactThreads) {
                const int64_t k = i / nv, v = i % nv;
                *reinterpret_cast<uint4*>(base + k * row_stride + s0 + v * 16) =
                    *reinterpret_cast<const uint4*>(stage + k * w + v * 16);
            }
        } else {
            for (int64_t i = threadIdx.x; i < count * w; i += kCompactThreads) {
                const int64_t k = i / w, b = i % w;
                stage[k * w + b] = base[__ldg(keep + k) * row_stride + s0 + b];
            }
            __syncthreads();
            for (int64_t i = threadIdx.x; i < count * w; i += kCompactThreads) {
                const int64_t k = i / w, b = i % w;
                base[k * row_stride + s0 + b] = stage[k * w + b];
            }
        }
        __syncthreads();
    }
}

}  // namespace accept
}  // namespace ddt

using namespace ddt;
using namespace ddt::accept;

template <typename T, bool V>
static int launch_argmax_t(const void* logits, int64_t n_rows, int64_t vocab, int64_t row_stride, size_t esz,
                           int64_t* posterior, unsigned char* ws, int mode, const TailArgs& tail, cudaStream_t st) {
    auto k = argmax_kernel<T, V>;
    int dev = 0;
    cudaGetDevice(&dev);
    const size_t smem = mode == kTreeWalk ? walk_smem_bytes(n_rows < kMaxRowsPerLaunch ? n_rows : kMaxRowsPerLaunch) : 0;
    if (smem > 48 * 1024 && cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
        return check_launch("cudaFuncSetAttribute(argmax_kernel)");
    int occ = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, k, kThreads, smem) != cudaSuccess || occ < 1) {
        cudaGetLastError();
        occ = 1;
    }
    const char* base = static_cast<const char*>(logits);
    for (int64_t r0 = 0; r0 < n_rows; r0 += kMaxRowsPerLaunch) {
        const int64_t nr = n_rows - r0 < kMaxRowsPerLaunch ? n_rows - r0 : kMaxRowsPerLaunch;
        const int64_t chunks = choose_chunks(nr, vocab, (int64_t)occ * ddt_sm_count(dev));
        const int64_t clen = chunk_len_for(vocab, chunks);
        const int64_t nchunks = ceil_div(vocab, clen);
        const T* lg = reinterpret_cast<const T*>(base + r0 * row_stride * (int64_t)esz);
        int64_t* post_out = posterior ? posterior + r0 : nullptr;
        k<<<dim3((unsigned)nchunks, (unsigned)nr), kThreads, smem, st>>>(lg, nr, vocab, row_stride, clen, post_out, ws,
                                                                        mode, tail);
    }
    return check_launch("argmax_kernel");
}

static int launch_argmax(const void* logits, int dtype, int64_t n_rows, int64_t vocab, int64_t row_stride,
                         int64_t* posterior, void* workspace, size_t workspace_bytes, int mode, const TailArgs& tail,
                         cudaStream_t st) {
    if (!logits) return set_error(DDT_EINVAL, "logits is null");
    if (n_rows <= 0 || vocab <= 0 || vocab >= ((int64_t)1 << 31)) return set_error(DDT_EINVAL, "bad logits shape");
    if (row_stride < vocab) return set_error(DDT_EINVAL, "row_stride < vocab");
    if (dtype != DDT_F32 && dtype != DDT_BF16 && dtype != DDT_F16) return set_error(DDT_EINVAL, "dtype %d", dtype);
    if (mode != kArgmaxOnly && n_rows > kMaxRowsPerLaunch)
        return set_error(DDT_EUNSUPPORTED, "n_rows=%lld > %lld", (long long)n_rows, (long long)kMaxRowsPerLaunch);
    const WsLayout L = ws_layout(n_rows < kMaxRowsPerLaunch ? n_rows : kMaxRowsPerLaunch);
    if (!workspace || workspace_bytes < L.total)
        return set_error(DDT_EWORKSPACE, "accept workspace needs %zu bytes, got %zu", L.total, workspace_bytes);
    if (reinterpret_cast<uintptr_t>(workspace) % 256) return set_error(DDT_EINVAL, "workspace must be 256-byte aligned");
    const size_t esz = dtype == DDT_F32 ? 4 : 2;
    const bool vec = (reinterpret_cast<uintptr_t>(logits) % 16 == 0) && ((row_stride * esz) % 16 == 0);
    unsigned char* ws = static_cast<unsigned char*>(workspace);
    if (dtype == DDT_F32)
        return vec ? launch_argmax_t<float, true>(logits, n_rows, vocab, row_stride, esz, posterior, ws, mode, tail, st)
                   : launch_argmax_t<float, false>(logits, n_rows, vocab, row_stride, esz, posterior, ws, mode, tail, st);
    if (dtype == DDT_BF16)
        return vec ? launch_argmax_t<__nv_bfloat16, true>(logits, n_rows, vocab, row_stride, esz, posterior, ws, mode,
                                                          tail, st)
                   : launch_argmax_t<__nv_bfloat16, false>(logits, n_rows, vocab, row_stride, esz, posterior, ws, mode,
                                                           tail, st);
    return vec ? launch_argmax_t<__half, true>(logits, n_rows, vocab, row_stride, esz, posterior, ws, mode, tail, st)
               : launch_argmax_t<__half, false>(logits, n_rows, vocab, row_stride, esz, posterior, ws, mode, tail, st);
}

extern "C" size_t ddt_tree_accept_workspace_size(int64_t n_rows, int64_t vocab) {
    if (n_rows <= 0 || vocab <= 0) return 256;
    return ws_layout(n_rows < kMaxRowsPerLaunch ? n_rows : kMaxRowsPerLaunch).total;
}

extern "C" int ddt_argmax_rows(const void* logits, int dtype, int64_t n_rows, int64_t vocab, int64_t row_stride,
                               int64_t* posterior, void* workspace, size_t workspace_bytes, ddt_stream_t stream) {
    if (!posterior) return set_error(DDT_EINVAL, "posterior is null");
    TailArgs tail = {};
    return launch_argmax(logits, dtype, n_rows, vocab, row_stride, posterior, workspace, workspace_bytes,
                         kArgmaxOnly, tail, reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int ddt_tree_accept(const void* logits, int dtype, int64_t n_rows, int64_t vocab, int64_t row_stride,
                               const int32_t* parents, const int64_t* node_token_ids, const int32_t* n_nodes_dev,
                               int64_t* posterior, int64_t* accepted, int64_t max_accept, int64_t* accept_info,
                               void* workspace, size_t workspace_bytes, ddt_stream_t stream) {
    if (!parents || !accepted || !accept_info) return set_error(DDT_EINVAL, "parents / accepted / accept_info null");
    if (n_rows > 1 && !node_token_ids) return set_error(DDT_EINVAL, "node_token_ids is null");
    if (n_rows > kMaxNodes) return set_error(DDT_EUNSUPPORTED, "n_rows=%lld > %d", (long long)n_rows, kMaxNodes);
    if (max_accept < 1) return set_error(DDT_EINVAL, "max_accept must be >= 1");
    TailArgs tail = {};
    tail.parents = parents;
    tail.node_tokens = node_token_ids;
    tail.n_nodes_dev = n_nodes_dev;
    tail.accepted = accepted;
    tail.max_accept = max_accept;
    tail.accept_info = accept_info;
    return launch_argmax(logits, dtype, n_rows, vocab, row_stride, posterior, workspace, workspace_bytes, kTreeWalk,
                         tail, reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int ddt_tree_walk(const int64_t* posterior, int64_t n_rows, const int32_t* parents,
                             const int64_t* node_token_ids, const int32_t* n_nodes_dev, int64_t* accepted,
                             int64_t max_accept, int64_t* accept_info, ddt_stream_t stream) {
    if (!posterior || !parents || !accepted || !accept_info) return set_error(DDT_EINVAL, "null argument");
    if (n_rows > 1 && !node_token_ids) return set_error(DDT_EINVAL, "node_token_ids is null");
    if (n_rows <= 0 || n_rows > kMaxNodes) return set_error(DDT_EUNSUPPORTED, "n_rows=%lld", (long long)n_rows);
    if (max_accept < 1) return set_error(DDT_EINVAL, "max_accept must be >= 1");
    TailArgs tail = {};
    tail.parents = parents;
    tail.node_tokens = node_token_ids;
    tail.n_nodes_dev = n_nodes_dev;
    tail.accepted = accepted;
    tail.max_accept = max_accept;
    tail.accept_info = accept_info;
    const size_t smem = walk_smem_bytes(n_rows);
    tree_walk_kernel<<<1, kThreads, smem, reinterpret_cast<cudaStream_t>(stream)>>>(posterior, n_rows, tail);
    return check_launch("tree_walk_kernel");
}

extern "C" int ddt_eagle3_accept(const void* logits, int dtype, int64_t n_rows, int64_t vocab, int64_t row_stride,
                                 const int64_t* draft_tokens, const int64_t* retrieve, int64_t leaves, int64_t width,
                                 int64_t* posterior, int64_t* out_info, int64_t* accepted, void* workspace,
                                 size_t workspace_bytes, ddt_stream_t stream) {
    if (!draft_tokens || !retrieve || !out_info || !accepted) return set_error(DDT_EINVAL, "null argument");
    if (leaves <= 0 || width <= 0) return set_error(DDT_EINVAL, "retrieve shape [%lld, %lld]", (long long)leaves,
                                                    (long long)width);
    TailArgs tail = {};
    tail.draft_tokens = draft_tokens;
    tail.retrieve = retrieve;
    tail.leaves = leaves;
    tail.width = width;
    tail.e3_info = out_info;
    tail.e3_accepted = accepted;
    return launch_argmax(logits, dtype, n_rows, vocab, row_stride, posterior, workspace, workspace_bytes, kEagle3,
                         tail, reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int ddt_tree_commit(const int64_t* verify_ids, int64_t n_rows, const int64_t* accepted,
                               int64_t max_accept, const int64_t* accept_info, int64_t* output_ids, int64_t output_len,
                               int64_t start, const void* hidden, int64_t hidden_row_stride_bytes, int64_t row_bytes,
                               void* hidden_out, int64_t out_row_stride_bytes, ddt_stream_t stream) {
    if (!verify_ids || !accepted || !accept_info || !output_ids) return set_error(DDT_EINVAL, "null argument");
    if (n_rows <= 0 || max_accept < 1) return set_error(DDT_EINVAL, "n_rows and max_accept must be positive");
    if (start < 0 || output_len <= start) return set_error(DDT_EINVAL, "start %lld outside output of %lld",
                                                          (long long)start, (long long)output_len);
    if ((hidden == nullptr) != (hidden_out == nullptr))
        return set_error(DDT_EINVAL, "hidden and hidden_out go together");
    if (hidden && (row_bytes <= 0 || hidden_row_stride_bytes < row_bytes || out_row_stride_bytes < row_bytes))
        return set_error(DDT_EINVAL, "bad hidden row layout");
    commit_kernel<<<(unsigned)max_accept, kThreads, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
        verify_ids, n_rows, accepted, max_accept, accept_info, output_ids, output_len, start,
        static_cast<const unsigned char*>(hidden), hidden_row_stride_bytes, hidden ? row_bytes : 0,
        static_cast<unsigned char*>(hidden_out), out_row_stride_bytes);
    return check_launch("commit_kernel");
}

extern "C" int ddt_kv_compact(void* const* tensors, int64_t n_tensors, int64_t heads, int64_t row_bytes,
                              int64_t head_stride_bytes, int64_t row_stride_bytes, int64_t past_length,
                              int64_t cur_len, const int64_t* keep, const int64_t* keep_count_dev, int64_t max_keep,
                              ddt_stream_t stream) {
    if (n_tensors == 0 || heads == 0) return DDT_OK;
    if (!tensors || !keep || !keep_count_dev) return set_error(DDT_EINVAL, "null argument");
    if (n_tensors < 0 || heads < 0 || row_bytes <= 0 || past_length < 0 || cur_len < 0 || max_keep < 0)
        return set_error(DDT_EINVAL, "negative size");
    if (max_keep * 16 > kStageBytes)
        return set_error(DDT_EUNSUPPORTED, "max_keep=%lld exceeds %d", (long long)max_keep, kStageBytes / 16);
    if (n_tensors * heads > 0x7fffffff) return set_error(DDT_EINVAL, "too many tensors");
    kv_compact_kernel<<<(unsigned)(n_tensors * heads), kCompactThreads, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
        tensors, heads, row_bytes, head_stride_bytes, row_stride_bytes, past_length, cur_len, keep, keep_count_dev,
        max_keep);
    return check_launch("kv_compact_kernel");
}
