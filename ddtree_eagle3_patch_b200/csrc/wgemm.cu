// Weight-streaming GEMM for the decode-time projections, on tcgen05.
//
//   y[t, n] = sum_k x[t, k] * w[n, k]  (+ residual[t, n]),   t < T <= 64
//
// At batch 1 a decode round multiplies a few dozen token rows (33 verify
// rows, 16 draft rows) by weight matrices of 5-300 MB: the work is a stream
// of the weights through the tensor cores, bound by HBM.  The weight rows
// take the MMA's M side (128 per CTA) and the token rows its N side (T padded
// to 16/32/48/64), so one tcgen05.mma (M = 128, N = TP, K = 16) consumes a
// 128 x 16 slice of weights and the whole token batch:
//
//   warp 0 (one elected lane)  TMA producer: a 4-stage ring of [128 x 64]
//                              weight tiles (evict-first) and [TP x 64] token
//                              tiles (zero rows past T), 128-byte swizzle
//   warp 1 (one elected lane)  MMA issuer: 4 K16 steps per stage into a
//                              [128 lanes x TP] fp32 TMEM accumulator; each
//                              stage is released by a tcgen05.commit
//   warps 0-3                  epilogue: lane i owns weight row n0 + i; it
//                              reads its TP columns and writes y[t, n0 + i]
//                              (coalesced across the warp), adding the
//                              residual in fp32 and rounding once, as addmm
//
// Few weight-row blocks (a 2560-row output) leave SMs idle, so the K range
// is split across CTAs (grid.y, at most 8): the splits of a row block form
// one thread-block cluster, stage their fp32 partials in shared memory and
// reduce them through distributed shared memory, each CTA summing a share
// of the token rows over its peers in cluster-rank order, so the result
// does not depend on timing and no partial touches global memory.  CTAs are
// ~92 KB of shared memory (a 4-stage ring), two per SM.  Every wait is
// bounded; a wait that runs out sets the status word.
//
// Gate/up mode (ddt_wgemm_gate_up): the weight holds the MLP's gate and up
// projections interleaved in blocks of 64 rows (gate rows 64b .. 64b+63,
// then the same up rows), so a CTA's 128 rows pair each gate row with its
// up row and the epilogue writes act(gate) * up: the [T, 2I] intermediate is
// never stored and no separate elementwise kernel runs.
//
// Head mode (ddt_wgemm_head, the draft's lm_head): besides the logits, the
// epilogue leaves per token row and per block of 128 vocabulary rows the
// block's max, its sum of exp(x - max) and its largest top-k key, which the
// tree build (ddt_tree_build_head) reads instead of scanning every logit.
//
// Launched as a programmatic dependent (ddt_set_pdl), the kernel signals its
// own dependents at once and its producer puts the first ring stages' weight
// loads in flight before griddepcontrol.wait: the weights do not depend on
// the preceding kernels, so their latency overlaps those kernels' tails.
// Token rows, the residual and the output are touched only after the wait.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <mutex>

#include "common.cuh"
#include "sm100.cuh"

namespace ddt {
namespace wgemm {

using namespace ddt::sm100;

constexpr int kThreads = 128;
constexpr int BN = 128;                       // weight rows per CTA (MMA M)
constexpr int BK = 64;                        // K elements per stage (128-byte rows)
constexpr int kStages = 4;
constexpr uint32_t kWTile = BN * BK * 2;      // 16 KB
constexpr int kMaxSplits = 8;                 // portable cluster size

template <int TP>
struct Cfg {
    static constexpr uint32_t kXTile = TP * BK * 2;             // TP x 128 B, a multiple of 1 KB
    static constexpr uint32_t kStage = kWTile + kXTile;
    static constexpr uint32_t kBars = kStages * kStage;          // barriers after the ring
    static constexpr uint32_t kSmem = kBars + 256 + 1024;        // + alignment slack
    static constexpr uint32_t kTmemCols = TP <= 32 ? 32 : TP <= 64 ? 64 : 128;   // a power of two >= TP
    static_assert(TP % 16 == 0 && TP <= 128, "token tile: a multiple of 16 up to 128");
    static constexpr uint32_t kIdesc = idesc_bf16_f32(128, TP, false, false);
};

struct Params {
    int T, N, nk_total, splits;
    int gate_up;   // interleaved gate/up weight: write act(gate) * up, N / 2 columns
    // head mode (ddt_wgemm_head): per-block statistics of the rounded
    // outputs, laid out by head_stats_layout(T, N / 128); null otherwise
    float* st_m;
    float* st_s;
    unsigned long long* st_keys;
    const __nv_bfloat16* residual;
    int64_t r_stride;
    __nv_bfloat16* y;
    int64_t y_stride;
    int* status;
};

__device__ __forceinline__ void flag_error(int* status, int code) {
    if (status) atomicOr(status, 1 << code);
}

template <int TP>
__global__ void __launch_bounds__(kThreads)
wgemm_kernel(const __grid_constant__ CUtensorMap tw, const __grid_constant__ CUtensorMap tx, const Params p) {
    using C = Cfg<TP>;
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    unsigned char* smem = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::kBars);
    uint64_t* empty = full + kStages;
    uint64_t* done = empty + kStages;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nb = blockIdx.x, split = blockIdx.y;
    const int n0 = nb * BN;
    const int kb = (int)((int64_t)split * p.nk_total / p.splits);
    const int nk = (int)((int64_t)(split + 1) * p.nk_total / p.splits) - kb;   // >= 1 (splits <= nk_total)

    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        mbar_init(done, 1);
        fence_mbar_init();
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, C::kTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    // TMEM is held before dependents are released: a later kernel's CTA on
    // this SM can then only wait for this one's columns, never hold them
    griddep_launch_dependents();
    if (warp != 0) griddep_wait();   // the producer waits after its weight prefetch
    const uint32_t tmem = *tmem_slot;
    const uint32_t s_addr = smem_u32(smem);

    if (warp == 0) {
        // ---------------------------------------------------------------- TMA producer
        const bool leader = elect_one_sync();
        const uint64_t pol_w = policy_evict_first();   // weights are read once
        const uint64_t pol_x = policy_evict_last();    // token rows are read by every CTA
        // the first stages' weight tiles go out before the wait on the
        // preceding grid; their token tiles follow it
        const int pre = nk < kStages ? nk : kStages;
        if (leader) {
            for (int i = 0; i < pre; ++i) {
                mbar_arrive_expect_tx(&full[i], C::kStage);
                tma_load_2d_hint(smem + i * C::kStage, &tw, (kb + i) * BK, n0, &full[i], pol_w);
            }
        }
        griddep_wait();
        if (leader) {
            for (int i = 0; i < pre; ++i)
                tma_load_2d_hint(smem + i * C::kStage + kWTile, &tx, (kb + i) * BK, 0, &full[i], pol_x);
        }
        __syncwarp();
        int issued = pre;
        for (int i = pre; i < nk; ++i) {
            const int s = i % kStages;
            const bool ok = mbar_wait(&empty[s], (uint32_t)((i / kStages - 1) & 1));
            if (!__all_sync(DDT_FULL_MASK, ok)) {
                if (leader) flag_error(p.status, 1);
                break;
            }
            if (leader) {
                unsigned char* st = smem + s * C::kStage;
                mbar_arrive_expect_tx(&full[s], C::kStage);
                tma_load_2d_hint(st, &tw, (kb + i) * BK, n0, &full[s], pol_w);
                tma_load_2d_hint(st + kWTile, &tx, (kb + i) * BK, 0, &full[s], pol_x);
            }
            __syncwarp();
            ++issued;
        }
        // drain: every issued stage has landed before the CTA can exit
        for (int i = (issued > kStages ? issued - kStages : 0); i < issued; ++i)
            mbar_wait(&full[i % kStages], (uint32_t)((i / kStages) & 1));
    } else if (warp == 1) {
        // ---------------------------------------------------------------- MMA issuer
        const bool leader = elect_one_sync();
        for (int i = 0; i < nk; ++i) {
            const int s = i % kStages;
            const bool ok = mbar_wait(&full[s], (uint32_t)((i / kStages) & 1));
            tc_fence_after();
            if (!__all_sync(DDT_FULL_MASK, ok)) {
                if (leader) flag_error(p.status, 2);
                break;
            }
            if (leader) {
                const uint32_t base = s_addr + s * C::kStage;
                const uint64_t da = smem_desc_sw128(base, 16, 1024);
                const uint64_t db = smem_desc_sw128(base + kWTile, 16, 1024);
#pragma unroll
                for (int kk = 0; kk < BK / 16; ++kk)
                    mma_ss(tmem, da + (uint64_t)(kk * 2), db + (uint64_t)(kk * 2), C::kIdesc,
                           (i > 0 || kk > 0) ? 1u : 0u);
                mma_commit(&empty[s]);
            }
            __syncwarp();
        }
        if (leader) mma_commit(done);   // arrives once every MMA issued above has completed
        __syncwarp();
    }

    // -------------------------------------------------------------------- epilogue
    const bool ok = mbar_wait(done, 0);
    tc_fence_after();
    if (!ok && threadIdx.x == 0) flag_error(p.status, 3);
    const int row = warp * 32 + lane;
    const int n = n0 + row;
    float acc[TP];
    {
        // TP columns: 32-column loads, then a 16-column one when TP % 32 == 16
        const uint32_t taddr = tmem + ((uint32_t)(warp * 32) << 16);
#pragma unroll
        for (int c0 = 0; c0 + 32 <= TP; c0 += 32) {
            uint32_t r[32];
            tmem_ld32(taddr + c0, r);
            tmem_wait_ld();
#pragma unroll
            for (int c = 0; c < 32; ++c) acc[c0 + c] = __uint_as_float(r[c]);
        }
        if (TP % 32 == 16) {
            uint32_t r16[16];
            tmem_ld16(taddr + (TP - 16), r16);
            tmem_wait_ld();
#pragma unroll
            for (int c = 0; c < 16; ++c) acc[TP - 16 + c] = __uint_as_float(r16[c]);
        }
    }
    if (p.splits == 1 && p.gate_up) {
        // every accumulator goes through the idle ring, [TP][128], so that
        // all four warps share the SiLU products: thread (c, h) = (row % 64,
        // row / 64) writes column c at token rows h, h + 2, ...  The products
        // (an accurate exp and an IEEE divide each) are a long dependent
        // chain: unrolled by four, independent rows overlap.
        float* gu = reinterpret_cast<float*>(smem);
#pragma unroll
        for (int t = 0; t < TP; ++t) gu[t * BN + row] = acc[t];
        __syncthreads();
        const int c = row & 63, h = row >> 6;
        const int col = nb * 64 + c;
#pragma unroll 4
        for (int t = h; t < p.T; t += 2)
            p.y[(int64_t)t * p.y_stride + col] =
                silu_times(__float2bfloat16_rn(gu[t * BN + c]), __float2bfloat16_rn(gu[t * BN + 64 + c]));
    } else if (p.splits == 1) {
#pragma unroll
        for (int t = 0; t < TP; ++t) {
            if (t < p.T) {
                float v = acc[t];
                if (p.residual) v += __bfloat162float(p.residual[(int64_t)t * p.r_stride + n]);
                p.y[(int64_t)t * p.y_stride + n] = __float2bfloat16_rn(v);
            }
        }
        if (p.st_m) {
            // Head mode: the rounded logits of this block go through the idle
            // ring, [TP][128]; warp w then takes token rows w, w + 4, ...:
            // the block's max, its sum of exp(x - max) (in float64, so the
            // block's 128 terms add no rounding of their own) and its
            // largest key.
            float* xs = reinterpret_cast<float*>(smem);
#pragma unroll
            for (int t = 0; t < TP; ++t) xs[t * BN + row] = __bfloat162float(__float2bfloat16_rn(acc[t]));
            __syncthreads();
            const int nblk = p.N / BN;
            for (int t = warp; t < p.T; t += kThreads / 32) {
                float v[BN / 32];
                unsigned long long kmax = 0ull;
                bool nan = false;
                float m = -INFINITY;
#pragma unroll
                for (int i = 0; i < BN / 32; ++i) {
                    v[i] = xs[t * BN + lane + 32 * i];
                    const unsigned long long k = topk_key(v[i], (int64_t)n0 + lane + 32 * i);
                    kmax = k > kmax ? k : kmax;
                    nan |= v[i] != v[i];
                    m = fmaxf(m, v[i]);
                }
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) {
                    m = fmaxf(m, __shfl_xor_sync(DDT_FULL_MASK, m, o));
                    const unsigned long long q = __shfl_xor_sync(DDT_FULL_MASK, kmax, o);
                    kmax = q > kmax ? q : kmax;
                }
                nan = __any_sync(DDT_FULL_MASK, nan);
                double s = 0.0;
                if (!nan && m != -INFINITY) {
#pragma unroll
                    for (int i = 0; i < BN / 32; ++i) s += (double)expf(v[i] - m);
#pragma unroll
                    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(DDT_FULL_MASK, s, o);
                }
                if (lane == 0) {
                    const int64_t cell = (int64_t)t * nblk + nb;
                    p.st_m[cell] = nan ? __int_as_float(0x7fc00000) : m;
                    p.st_s[cell] = (float)s;
                    p.st_keys[cell] = kmax;
                }
            }
        }
    } else {
        // Split K: the splits of a row block are one thread-block cluster.
        // Each stages its fp32 partial [TP][128] in its own shared memory (the
        // ring is idle: every load was consumed and every MMA has completed),
        // then CTA r sums token rows r, r + S, ... over the peers' stages in
        // cluster-rank order (so the result does not depend on timing) and
        // writes them; a second cluster barrier keeps every stage alive until
        // its peers have read it.
        float* stage = reinterpret_cast<float*>(smem);
#pragma unroll
        for (int t = 0; t < TP; ++t) stage[t * BN + row] = acc[t];
        cluster_sync();
        const int r = (int)cluster_ctarank();
        float* pair = stage + TP * BN;   // gate/up mode: the reduced [TP][128] sums
        // kRows of this CTA's token rows at a time: every peer load and
        // residual load of the group is issued before the first sum, so
        // their latencies overlap instead of adding up row by row
        constexpr int kRows = 4;
        for (int t0 = r; t0 < p.T; t0 += kRows * p.splits) {
            float part[kRows][kMaxSplits];
            float res[kRows];
#pragma unroll
            for (int j = 0; j < kRows; ++j) {
                const int t = t0 + j * p.splits;
                const bool in = t < p.T;
#pragma unroll
                for (int q = 0; q < kMaxSplits; ++q)
                    part[j][q] = in && q < p.splits ? ld_dsmem_f32(stage + t * BN + row, (uint32_t)q) : 0.f;
                res[j] = in && p.residual ? __bfloat162float(p.residual[(int64_t)t * p.r_stride + n]) : 0.f;
            }
#pragma unroll
            for (int j = 0; j < kRows; ++j) {
                const int t = t0 + j * p.splits;
                if (t >= p.T) break;
                float v = 0.f;
#pragma unroll
                for (int q = 0; q < kMaxSplits; ++q) v += part[j][q];
                if (p.gate_up) {
                    pair[t * BN + row] = v;
                    continue;
                }
                if (p.residual) v += res[j];
                p.y[(int64_t)t * p.y_stride + n] = __float2bfloat16_rn(v);
            }
        }
        if (p.gate_up) {
            // the SiLU products of this CTA's token rows, over all four warps
            __syncthreads();
            const int c = row & 63, h = row >> 6;
            const int col = nb * 64 + c;
#pragma unroll 4
            for (int t = r + h * p.splits; t < p.T; t += 2 * p.splits)
                p.y[(int64_t)t * p.y_stride + col] = silu_times(__float2bfloat16_rn(pair[t * BN + c]),
                                                                __float2bfloat16_rn(pair[t * BN + 64 + c]));
        }
        cluster_sync();
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, C::kTmemCols);
    }
}

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

// 2-D bf16 map over [rows, cols] (cols innermost) with a [box_rows x 64] box.
static int make_map_2d(CUtensorMap* m, const void* base, uint64_t cols, uint64_t rows, uint64_t row_bytes,
                       uint32_t box_rows) {
    auto fn = encode_fn();
    if (!fn) return set_error(DDT_ECUDA, "cuTensorMapEncodeTiled is unavailable");
    cuuint64_t dims[2] = {cols, rows};
    cuuint64_t strides[1] = {row_bytes};
    cuuint32_t box[2] = {(cuuint32_t)BK, box_rows};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return set_error(DDT_EINVAL, "cuTensorMapEncodeTiled failed (%d)", (int)r);
    return DDT_OK;
}

// The kernel's shared-memory opt-in, once per token tile.
template <int TP>
static cudaError_t prepare() {
    static std::once_flag once;
    static cudaError_t attr = cudaSuccess;
    std::call_once(once, [] {
        attr = cudaFuncSetAttribute(wgemm_kernel<TP>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    (int)Cfg<TP>::kSmem);
    });
    return attr;
}

// CTAs of token tile TP that fit on one SM by shared memory (228 KB per SM,
// 1 KB of it reserved per CTA).
static int ctas_per_sm(int TP) {
    uint32_t smem = 0;
    switch (TP) {
        case 16: smem = Cfg<16>::kSmem; break;
        case 32: smem = Cfg<32>::kSmem; break;
        case 48: smem = Cfg<48>::kSmem; break;
        case 64: smem = Cfg<64>::kSmem; break;
        case 80: smem = Cfg<80>::kSmem; break;
        default: smem = Cfg<128>::kSmem; break;
    }
    const int n = (int)((228u * 1024u) / (smem + 1024u));
    return n < 1 ? 1 : n;
}

// About one wave of two CTAs per SM, and at most 90 % of the CTAs that fit
// at once: a grid of clusters that fills them (almost) exactly runs part of
// it as a second wave.  Measured on B200 at 33 token rows (two CTAs per SM):
// 48 row blocks x 6 splits (288 CTAs) 17.4 us, x 5 splits 10.5 us; 32 x 8
// (256 CTAs) ran in one wave.  At 16 rows (three per SM) 48 x 6 is the best.
static int choose_splits(int64_t N, int64_t K, int sms, int TP) {
    const int64_t nblocks = N / BN, nk = K / BK;
    if (sms <= 0) sms = 148;
    const int per_sm = ctas_per_sm(TP);
    const int64_t wave = (int64_t)sms * (per_sm < 2 ? per_sm : 2);
    const int64_t fit = (int64_t)sms * per_sm * 9 / 10;
    int64_t s = (wave < fit ? wave : fit) / nblocks;
    if (s > kMaxSplits) s = kMaxSplits;
    if (s > nk / 2) s = nk / 2;                            // at least two stages per split
    return s < 1 ? 1 : (int)s;
}

template <int TP>
static int launch(const CUtensorMap& tw, const CUtensorMap& tx, const Params& p, int nblocks, cudaStream_t st) {
    using C = Cfg<TP>;
    const cudaError_t attr = prepare<TP>();
    if (attr != cudaSuccess) return set_error(DDT_ECUDA, "cudaFuncSetAttribute(wgemm): %s", cudaGetErrorString(attr));
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)nblocks, (unsigned)p.splits);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = C::kSmem;
    cfg.stream = st;
    cudaLaunchAttribute attr_c[2];
    unsigned na = 0;
    if (p.splits > 1) {
        attr_c[na].id = cudaLaunchAttributeClusterDimension;   // the splits of a row block share a cluster
        attr_c[na].val.clusterDim.x = 1;
        attr_c[na].val.clusterDim.y = (unsigned)p.splits;
        attr_c[na].val.clusterDim.z = 1;
        ++na;
    }
    na += pdl_attr(&attr_c[na]);
    cfg.attrs = attr_c;
    cfg.numAttrs = na;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, wgemm_kernel<TP>, tw, tx, p);
    if (e != cudaSuccess) return set_error(DDT_ECUDA, "wgemm_kernel: %s", cudaGetErrorString(e));
    return check_launch("wgemm_kernel");
}

}  // namespace wgemm
}  // namespace ddt

using namespace ddt;

extern "C" size_t ddt_wgemm_workspace_size(int64_t T, int64_t N, int64_t K) {
    (void)T;
    (void)N;
    (void)K;
    return 256;   // the status word
}

static int wgemm_run(const void* x, int64_t x_stride, int64_t T, const void* w, int64_t w_stride, int64_t N,
                     int64_t K, const void* residual, int64_t r_stride, void* y, int64_t y_stride, int gate_up,
                     int64_t splits_hint, void* workspace, size_t workspace_bytes, ddt_stream_t stream,
                     void* stats = nullptr) {
    using namespace ddt::wgemm;
    if (!x || !w || !y) return set_error(DDT_EINVAL, "null argument");
    if (T <= 0 || T > 128) return set_error(DDT_EUNSUPPORTED, "T=%lld outside [1, 128]", (long long)T);
    if (N <= 0 || N % BN || K <= 0 || K % BK)
        return set_error(DDT_EUNSUPPORTED, "N=%lld must be a multiple of 128 and K=%lld of 64", (long long)N,
                         (long long)K);
    if (N / BN > 65535) return set_error(DDT_EUNSUPPORTED, "N too large");
    const int64_t out_cols = gate_up ? N / 2 : N;
    if (x_stride < K || w_stride < K || y_stride < out_cols || (residual && r_stride < N))
        return set_error(DDT_EINVAL, "strides smaller than the rows");
    auto mis = [](const void* ptr, int b) { return reinterpret_cast<uintptr_t>(ptr) % b != 0; };
    if (mis(x, 16) || mis(w, 16) || (x_stride * 2) % 16 || (w_stride * 2) % 16)
        return set_error(DDT_EINVAL, "x / w must be 16-byte aligned with row strides of multiples of 8 elements");
    if (!workspace || mis(workspace, 256) || workspace_bytes < ddt_wgemm_workspace_size(T, N, K))
        return set_error(DDT_EWORKSPACE, "wgemm workspace needs %zu bytes (256-aligned)",
                         ddt_wgemm_workspace_size(T, N, K));
    int dev = 0;
    cudaGetDevice(&dev);
    // token tile: the decode shapes (15 / 16 draft rows, 33 and 65 verify rows)
    // pad to 16 / 48 / 80; others to the next of 16, 32, 48, 64, 80, 128
    const int TP = T <= 16 ? 16 : T <= 32 ? 32 : T <= 48 ? 48 : T <= 64 ? 64 : T <= 80 ? 80 : 128;
    int splits = choose_splits(N, K, ddt_sm_count(dev), TP);
    if (splits_hint > 0) {   // the caller's choice, within the cluster limit and the K stages
        splits = (int)(splits_hint < kMaxSplits ? splits_hint : kMaxSplits);
        if (splits > K / BK) splits = (int)(K / BK);
    }
    if (stats) splits = 1;   // the statistics come from whole blocks
    CUtensorMap tw, tx;
    int rc = make_map_2d(&tw, w, (uint64_t)K, (uint64_t)N, (uint64_t)w_stride * 2, BN);
    if (!rc) rc = make_map_2d(&tx, x, (uint64_t)K, (uint64_t)T, (uint64_t)x_stride * 2, (uint32_t)TP);
    if (rc) return rc;
    unsigned char* ws = static_cast<unsigned char*>(workspace);
    Params p;
    p.T = (int)T;
    p.N = (int)N;
    p.nk_total = (int)(K / BK);
    p.splits = splits;
    p.gate_up = gate_up;
    p.st_m = p.st_s = nullptr;
    p.st_keys = nullptr;
    if (stats) {
        const HeadStatsLayout h = head_stats_layout(T, N / BN);
        unsigned char* sb = static_cast<unsigned char*>(stats);
        p.st_m = reinterpret_cast<float*>(sb + h.m);
        p.st_s = reinterpret_cast<float*>(sb + h.s);
        p.st_keys = reinterpret_cast<unsigned long long*>(sb + h.keys);
    }
    p.residual = static_cast<const __nv_bfloat16*>(residual);
    p.r_stride = r_stride;
    p.y = static_cast<__nv_bfloat16*>(y);
    p.y_stride = y_stride;
    p.status = reinterpret_cast<int*>(ws);
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    const int nblocks = (int)(N / BN);
    switch (TP) {
        case 16: return launch<16>(tw, tx, p, nblocks, st);
        case 32: return launch<32>(tw, tx, p, nblocks, st);
        case 48: return launch<48>(tw, tx, p, nblocks, st);
        case 64: return launch<64>(tw, tx, p, nblocks, st);
        case 80: return launch<80>(tw, tx, p, nblocks, st);
        default: return launch<128>(tw, tx, p, nblocks, st);
    }
}

extern "C" int ddt_wgemm(const void* x, int64_t x_stride, int64_t T, const void* w, int64_t w_stride, int64_t N,
                         int64_t K, const void* residual, int64_t r_stride, void* y, int64_t y_stride,
                         int64_t splits_hint, void* workspace, size_t workspace_bytes, ddt_stream_t stream) {
    return wgemm_run(x, x_stride, T, w, w_stride, N, K, residual, r_stride, y, y_stride, 0, splits_hint, workspace,
                     workspace_bytes, stream);
}

extern "C" int ddt_wgemm_gate_up(const void* x, int64_t x_stride, int64_t T, const void* w_gate_up,
                                 int64_t w_stride, int64_t N2, int64_t K, void* y, int64_t y_stride,
                                 int64_t splits_hint, void* workspace, size_t workspace_bytes, ddt_stream_t stream) {
    return wgemm_run(x, x_stride, T, w_gate_up, w_stride, N2, K, nullptr, 0, y, y_stride, 1, splits_hint, workspace,
                     workspace_bytes, stream);
}

extern "C" size_t ddt_wgemm_head_stats_size(int64_t T, int64_t N) {
    if (T <= 0 || N <= 0) return 256;
    return ddt::head_stats_layout(T, N / ddt::kHeadBlock).total;
}

extern "C" int ddt_wgemm_head(const void* x, int64_t x_stride, int64_t T, const void* w, int64_t w_stride, int64_t N,
                              int64_t K, void* y, int64_t y_stride, void* stats, size_t stats_bytes, void* workspace,
                              size_t workspace_bytes, ddt_stream_t stream) {
    if (!stats || reinterpret_cast<uintptr_t>(stats) % 256 || stats_bytes < ddt_wgemm_head_stats_size(T, N))
        return set_error(DDT_EWORKSPACE, "head statistics need %zu bytes (256-aligned)",
                         ddt_wgemm_head_stats_size(T, N));
    return wgemm_run(x, x_stride, T, w, w_stride, N, K, nullptr, 0, y, y_stride, 0, 0, workspace, workspace_bytes,
                     stream, stats);
}
