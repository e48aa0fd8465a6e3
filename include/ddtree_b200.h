/*
 * ddtree_b200.h - C ABI of the B200 (sm_100a) DDTree draft-tree hot path.
 *
 * One shared library, libddtree_b200.so, exports these entry points.  They
 * take raw device pointers, sizes and strides plus a cudaStream_t; nothing
 * in the signatures is a torch type.  Inputs are borrowed; outputs go to
 * caller-allocated device buffers.  Every entry point validates its
 * arguments on the host and returns DDT_OK or an error code; the text of
 * the last error of the calling thread is available from ddt_last_error().
 * Kernels are launched asynchronously on `stream`.  Errors that can only be
 * seen on the device (a non-finite log-normaliser, a bounded wait that ran
 * out) are reported through the `info` words of the call's outputs.
 *
 * Each entry point names the reference function it replaces
 * (kimwin2/ddtree_eagle3_patch, file:line).
 */
#ifndef DDTREE_B200_H
#define DDTREE_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st* ddt_stream_t; /* same handle as cudaStream_t */

#if defined(__GNUC__)
#define DDT_API __attribute__((visibility("default")))
#else
#define DDT_API
#endif

enum ddt_status {
    DDT_OK = 0,
    DDT_EINVAL = 1,      /* bad argument (shape, stride, alignment, null pointer) */
    DDT_ECUDA = 2,       /* a CUDA runtime call failed */
    DDT_EUNSUPPORTED = 3,/* valid but outside what this build implements */
    DDT_EWORKSPACE = 4   /* workspace missing or too small */
};

enum ddt_dtype { DDT_F32 = 0, DDT_BF16 = 1, DDT_F16 = 2, DDT_BOOL = 3 };

/* info[2] bits written by the tree-build kernels */
#define DDT_INFO_NONFINITE 1u /* a selected log-probability or log-normaliser was not finite */

DDT_API const char* ddt_last_error(void);
DDT_API int ddt_abi_version(void);
DDT_API int ddt_sm_count(int device);
/* Kernels this library has launched since it was loaded (all devices and
 * threads; a launch recorded into a CUDA graph counts once, at capture). */
DDT_API uint64_t ddt_launch_count(void);
/* Launch the decode-layer kernels (ddt_rms_norm, ddt_qk_norm_rope_append,
 * ddt_silu_mul*, ddt_kv_append, ddt_wgemm*) as programmatic dependent
 * launches: each may start while the kernel before it in the stream is
 * still running and waits (griddepcontrol.wait) before touching anything
 * that kernel may write, so launch latency and prologues overlap.  (The
 * split-key attention kernels are always launched that way; with this on,
 * host-length attention calls load no key before that wait.)  While on,
 * the WEIGHT operand of ddt_wgemm / ddt_wgemm_gate_up is read before the
 * preceding kernels complete: it must not be written by work still queued
 * on the stream.  Off at load.  Returns the previous setting.  Reference
 * counterpart: none (the reference launches cuBLAS / SDPA through torch). */
DDT_API int ddt_set_pdl(int enabled);

/* ---------------------------------------------------------------------------
 * (1) Tree build.
 * Replaces build_ddtree_tree (ddtree.py:114-196) and the id / position
 * buffer fills of compile_ddtree_tree (ddtree.py:233-245).
 *
 * logits: [rows, vocab] float32 / bf16 / fp16, row stride `row_stride`
 * elements.  budget >= 0; topk = min(budget, vocab); rows <= 32;
 * budget <= 1024.  The tree has n = min(budget, reachable) nodes; node i
 * (1-based) is the i-th entry popped by the best-first expansion.
 * ------------------------------------------------------------------------- */
typedef struct {
    int64_t* top_ids;        /* [rows, topk] int64 token ids, value desc / id asc (nullable) */
    float* top_lp;           /* [rows, topk] fp32 log-probs top - logsumexp (nullable)       */
    int64_t* node_token_ids; /* [budget] int64                                               */
    int64_t* node_depths;    /* [budget] int64 (1-based depth)                               */
    int32_t* parents;        /* [budget + 1] int32, parents[0] = -1                          */
    uint32_t* visibility;    /* [budget + 1, vis_words] ancestor bitmask: bit j of row i set
                                iff tree row j is row i or one of its ancestors (nullable)   */
    int64_t vis_words;       /* row stride of `visibility` in uint32 words, >= ceil((budget+1)/32) */
    int64_t* verify_ids;     /* [budget + 1] root token then node tokens (nullable)          */
    int64_t* verify_pos;     /* [budget + 1] start + depth (nullable)                        */
    int32_t* info;           /* [4]: node count, max depth, DDT_INFO_* flags, topk           */
} ddt_tree_outputs;

/* Workspace bytes for ddt_tree_build.  The workspace must be zero-filled
 * before its first use; every completed call leaves its counters at zero. */
DDT_API size_t ddt_tree_build_workspace_size(int64_t rows, int64_t vocab, int64_t budget);

DDT_API int ddt_tree_build(const void* logits, int dtype, int64_t rows, int64_t vocab, int64_t row_stride,
                   int64_t budget, const int64_t* root_token /* device scalar, nullable */, int64_t start,
                   const ddt_tree_outputs* out, void* workspace, size_t workspace_bytes, ddt_stream_t stream);

/* ddt_tree_build over bf16 logits written by ddt_wgemm_head, from its block
 * statistics `head_stats` (same rows and vocab): the row maxima and sums of
 * exp come from the blocks' pieces, and the top-k from the logits of only
 * the top-k blocks by their largest key.  Same outputs and workspace as
 * ddt_tree_build: the same top ids; lp within 2 ulp of the float64
 * log-softmax (another summation order than ddt_tree_build's, so the two
 * may differ in the last bits), the tree the expansion of those.  vocab a
 * multiple of 128, top-k (min(budget, vocab)) at most 80;
 * DDT_EUNSUPPORTED beyond. */
DDT_API int ddt_tree_build_head(const void* logits, int64_t rows, int64_t vocab, int64_t row_stride,
                                const void* head_stats, int64_t budget, const int64_t* root_token, int64_t start,
                                const ddt_tree_outputs* out, void* workspace, size_t workspace_bytes,
                                ddt_stream_t stream);

/* ddt_tree_build for callers that cannot allocate device memory.
 * This entry point has no counterpart in the reference.  Some callers of this
 * library cannot call cudaMalloc: a host application whose device memory is
 * owned by another allocator (a serving framework's pool) that must not grow
 * behind its back, or a plugin that is handed only its input and output
 * buffers.  This call takes the same inputs and outputs as ddt_tree_build but
 * no workspace: its scratch is a fixed 1 MiB array inside the library's
 * device image, held by every GPU that loads the library until the process
 * exits.  1 MiB covers 15 draft rows x 151936 vocabulary up to a node budget
 * of 512; larger shapes return DDT_EUNSUPPORTED.  It calls no cudaMalloc /
 * cudaFree.
 * The first call on a device looks up the array's device address
 * (cudaGetSymbolAddress, with that device current) and keeps it for the
 * process: it assumes the device's primary context and no cudaDeviceReset
 * afterwards.  Make that first call before any stream capture.  All calls
 * share the one array: calls that overlap on the GPU (different streams
 * without ordering) race.  Each call clears the counters at the start of the
 * array on `stream` before its launch. */
DDT_API int ddt_tree_build_noalloc(const void* logits, int dtype, int64_t rows, int64_t vocab, int64_t row_stride,
                                   int64_t budget, const int64_t* root_token, int64_t start,
                                   const ddt_tree_outputs* out, ddt_stream_t stream);

/* Best-first expansion only, from given log-probs and ids (ddtree.py:146-189).
 * lp: [rows, topk] fp32, ids: [rows, topk] int64, both device. */
DDT_API int ddt_tree_from_log_probs(const float* lp, const int64_t* ids, int64_t rows, int64_t topk, int64_t budget,
                            const int64_t* root_token, int64_t start, const ddt_tree_outputs* out,
                            ddt_stream_t stream);

/* Dense additive mask rows for the HF verify forward (ddtree.py:230-251):
 * clears the previous tree block [0, prev_len) x [prev_start, prev_start+prev_len)
 * to 0, then writes rows [0, n_rows) x [past, past + n_rows) as 0 where the
 * ancestor bit is set and `min_value` elsewhere.  mask: [rows_cap, row_stride]
 * of `dtype`. */
DDT_API int ddt_tree_mask_fill(void* mask, int dtype, int64_t row_stride, int64_t rows_cap, int64_t past_length,
                       int64_t n_rows, const uint32_t* visibility, int64_t vis_words, int64_t prev_start,
                       int64_t prev_len, double min_value, ddt_stream_t stream);

/* Packs the tree block of a dense bool / additive mask into the ancestor
 * bitmask layout (a visible entry is a nonzero bool or a value > min/2).
 * Used when a caller hands the verify attention a dense mask. */
DDT_API int ddt_mask_to_bits(const void* mask, int dtype, int64_t row_stride, int64_t col_offset, int64_t n_rows,
                     uint32_t* visibility, int64_t vis_words, ddt_stream_t stream);

/* ---------------------------------------------------------------------------
 * (2) Tree-masked verify attention (one layer).
 * Replaces the target's attention call inside the verify forward
 * (ddtree.py:523-531 -> transformers sdpa_attention_forward with the 4-D mask
 * from ddtree.py:247-253), i.e. softmax(Q K^T * scale + mask) V with GQA.
 *
 * q:   [n_tokens, hq, 128] bf16 (token stride q_stride_tok, head stride q_stride_head, elements)
 * k,v: [hkv, kv_rows, 128] bf16 (head stride kv_stride_head, row stride kv_stride_row)
 *      rows [0, past) are the prefix, rows [past, past + n_tokens) the tree.
 * out: [n_tokens, hq, 128] bf16.
 * visibility: [n_tokens, vis_words] ancestor bitmask of the tree rows.
 * Row t sees every prefix key and tree key j iff bit j of its mask is set.
 * ------------------------------------------------------------------------- */
typedef struct {
    const void* q;
    int64_t q_stride_tok, q_stride_head;
    const void* k;
    const void* v;
    int64_t kv_stride_head, kv_stride_row;
    int64_t kv_rows;           /* allocated rows of k / v (>= past + n_tokens) */
    void* out;
    int64_t o_stride_tok, o_stride_head;
    int64_t n_tokens, hq, hkv, head_dim, past_length;
    const uint32_t* visibility;
    int64_t vis_words;
    float scale;
} ddt_attention_args;

DDT_API size_t ddt_tree_attention_workspace_size(int64_t n_tokens, int64_t hq, int64_t hkv, int64_t past_length,
                                         int device);
DDT_API int ddt_tree_attention(const ddt_attention_args* args, void* workspace, size_t workspace_bytes,
                       ddt_stream_t stream);

/* Sliding-window layers of a hybrid model (Gemma 3/4).  Replaces the same
 * attention call when the layer gets the reference's "sliding_attention"
 * mask (ddtree.py:258-287): key_lo [n_tokens] int64 on the device gives
 * each tree row its first visible prefix key, so row t sees prefix key j
 * iff j >= key_lo[t] (the reference's query_position - window + 1; values
 * below 0 or above past_length are clamped).  Tree keys follow `visibility`
 * as in ddt_tree_attention.  Same workspace. */
DDT_API int ddt_tree_attention_window(const ddt_attention_args* args, const int64_t* key_lo, void* workspace,
                              size_t workspace_bytes, ddt_stream_t stream);

/* The same call with the prefix length read from device memory at run time,
 * so that one captured launch serves every round of a decode loop (the
 * verify attention of ddtree.py:523-531, and the draft's attention over its
 * cache, model/dflash.py:89-106, whose prefix grows every round).
 * args->past_length is the largest prefix the call may see: the launch is
 * planned for it, kv_rows >= past_length + n_tokens, and *past_dev is clamped
 * to [0, past_length].  K/V rows past the run-time tree are masked, and must
 * hold finite values (a zero-filled or previously written cache).  key_lo is
 * nullable (sliding window as in ddt_tree_attention_window).  Workspace as
 * for ddt_tree_attention at past_length.  Shapes whose rows do not fit the
 * split-key kernel (more than 147 128-row tiles x KV heads) return
 * DDT_EUNSUPPORTED.  stable_dev (nullable device int32): keys [0, *stable_dev)
 * are written by nothing still running on the stream, so their K tiles may
 * load before the preceding kernel completes (the target verify: the whole
 * prefix; the draft: the keys before this round's context rows).  Null: every
 * key loads after it. */
DDT_API int ddt_tree_attention_dev(const ddt_attention_args* args, const int64_t* key_lo, const int32_t* past_dev,
                                   const int32_t* stable_dev, void* workspace, size_t workspace_bytes,
                                   ddt_stream_t stream);

/* The same attention call for float32 targets (the reference's SDPA in the
 * target's dtype, ddtree.py:523-531): q, k, v and out are float32 with the
 * strides of ddt_attention_args counted in float elements (multiples of 4),
 * computed with fp32 FMAs and accurate exponentials on the CUDA cores (the
 * tensor cores have no float32 operand form that keeps 1e-5 accuracy).
 * key_lo (nullable) makes it a sliding-window layer as in
 * ddt_tree_attention_window.  past_dev (nullable, device int32): the prefix
 * length is read from it at run time, clamped to [0, args->past_length],
 * which is then only its upper bound (kv_rows >= past_length + n_tokens).
 * No workspace. */
DDT_API int ddt_tree_attention_f32(const ddt_attention_args* args, const int64_t* key_lo, const int32_t* past_dev,
                                   ddt_stream_t stream);

/* ---------------------------------------------------------------------------
 * (3) Greedy acceptance and KV compaction.
 * ddt_tree_accept replaces sample(logits, 0) (model/utils.py:28-30) plus
 * follow_verified_tree (ddtree.py:290-301): row-wise argmax (first max; NaN
 * counts as largest) and the walk from the root down the tree while the
 * target's token is a child of the current node.
 * logits [n_rows, vocab] with n_rows = 1 + node count; parents / node tokens
 * as produced by ddt_tree_build; n_nodes_dev (nullable) overrides n_rows-1
 * with the device-side node count info[0] of the build.
 * accepted: [max_accept] int64 tree row indices (root 0 first);
 * accept_info: [2] int64 = {accepted count, next (bonus) token}.
 * ------------------------------------------------------------------------- */
DDT_API size_t ddt_tree_accept_workspace_size(int64_t n_rows, int64_t vocab);
DDT_API int ddt_tree_accept(const void* logits, int dtype, int64_t n_rows, int64_t vocab, int64_t row_stride,
                    const int32_t* parents, const int64_t* node_token_ids, const int32_t* n_nodes_dev,
                    int64_t* posterior /* [n_rows], nullable */, int64_t* accepted, int64_t max_accept,
                    int64_t* accept_info, void* workspace, size_t workspace_bytes, ddt_stream_t stream);

/* The walk alone, from a posterior [n_rows] int64 already on the device
 * (follow_verified_tree, ddtree.py:290-301). */
DDT_API int ddt_tree_walk(const int64_t* posterior, int64_t n_rows, const int32_t* parents,
                          const int64_t* node_token_ids, const int32_t* n_nodes_dev, int64_t* accepted,
                          int64_t max_accept, int64_t* accept_info, ddt_stream_t stream);

/* Row-wise argmax alone (model/utils.py:28-30), posterior [n_rows] int64. */
DDT_API int ddt_argmax_rows(const void* logits, int dtype, int64_t n_rows, int64_t vocab, int64_t row_stride,
                    int64_t* posterior, void* workspace, size_t workspace_bytes, ddt_stream_t stream);

/* Temperature sampling of each row, the temperature > 0 branch of
 * sample(logits, temperature) (model/utils.py:31-35): one token per row drawn
 * from softmax(logits / temperature), written to posterior [n_rows] int64.
 * Drawn by the Gumbel-max rule with Philox4x32-10 uniforms keyed by `seed` and
 * counted by (element, row, `offset`): the same (seed, offset) gives the same
 * draws, and the distribution is torch.multinomial's, not its random stream.
 * NaN logits are never drawn (a row of NaN gives 0).  The posterior feeds
 * ddt_tree_walk.  n_rows <= 65535; vocab < 2^31. */
DDT_API size_t ddt_sample_rows_workspace_size(int64_t n_rows, int64_t vocab);
DDT_API int ddt_sample_rows(const void* logits, int dtype, int64_t n_rows, int64_t vocab, int64_t row_stride,
                    float temperature, uint64_t seed, uint64_t offset, int64_t* posterior, void* workspace,
                    size_t workspace_bytes, ddt_stream_t stream);

/* The commit step of a round (ddtree.py:534-548) on the device, after
 * ddt_tree_accept: output_ids[start + i] = verify_ids[accepted[i]] for
 * i < count and output_ids[start + count] = the bonus token, where count and
 * the bonus token are accept_info[0] and accept_info[1] (read on the device,
 * so the round needs no host sync).  When hidden is given, hidden_out row i
 * = hidden row accepted[i] for i < count: the accepted rows of the verify
 * hidden features (index_select(1, accepted_index_tensor)), rows of
 * row_bytes bytes at the given strides.  Writes at or past output_len and
 * accepted indices outside [0, n_rows) are skipped. */
DDT_API int ddt_tree_commit(const int64_t* verify_ids, int64_t n_rows, const int64_t* accepted, int64_t max_accept,
                            const int64_t* accept_info, int64_t* output_ids, int64_t output_len, int64_t start,
                            const void* hidden /* nullable */, int64_t hidden_row_stride_bytes, int64_t row_bytes,
                            void* hidden_out /* nullable */, int64_t out_row_stride_bytes, ddt_stream_t stream);

/* In-place compaction of the appended window of many cache tensors in one
 * launch.  Replaces compact_dynamic_cache's per-layer loop (ddtree.py:323-369)
 * over compact_tail_inplace (ddtree.py:61-88): for every tensor t and head h,
 *   rows past + keep[k] -> past + k, k < keep_count,
 * with every read done before any write (index_select then copy_).
 * tensors: device array of n_tensors base pointers; all share heads,
 * row_bytes (head_dim * element size), head and row strides (bytes).
 * keep / keep_count live on the device (keep_count may be the accept_info of
 * ddt_tree_accept); cur_len is the appended window length: the call is a
 * no-op when keep_count is 0 or equals cur_len (ddtree.py:80-81). */
DDT_API int ddt_kv_compact(void* const* tensors, int64_t n_tensors, int64_t heads, int64_t row_bytes,
                   int64_t head_stride_bytes, int64_t row_stride_bytes, int64_t past_length, int64_t cur_len,
                   const int64_t* keep, const int64_t* keep_count_dev, int64_t max_keep, ddt_stream_t stream);

/* Append of new K/V rows into a preallocated cache at a device-side row
 * offset.  Replaces DynamicCache.update's torch.cat of the whole cache
 * (transformers cache_utils.py DynamicLayer.update, reached from the verify
 * forward at ddtree.py:523-531 and the draft at ddtree.py:478-486): for every
 * head h < heads and row r < rows (r < *rows_dev when rows_dev is given),
 *   dst row (*offset_dev + r) of head h <- src row r of head h,
 * for K and V; destination rows outside [0, dst_rows) are skipped.  Strides
 * in bytes; pointers, strides and row_bytes multiples of 16. */
DDT_API int ddt_kv_append(const void* k_src, const void* v_src, int64_t src_head_stride_bytes,
                          int64_t src_row_stride_bytes, void* k_dst, void* v_dst, int64_t dst_head_stride_bytes,
                          int64_t dst_row_stride_bytes, int64_t dst_rows, int64_t heads, int64_t rows,
                          int64_t row_bytes, const int32_t* offset_dev, const int32_t* rows_dev /* nullable */,
                          ddt_stream_t stream);

/* ---------------------------------------------------------------------------
 * Fused elementwise steps of a Qwen3-style decoder layer for the verify and
 * draft forwards of a round (the target layers run by ddtree.py:523-531 and
 * the DFlash layers of model/dflash.py:36-150).  Each follows the stock
 * module's arithmetic order, rounding to the dtype where it does.
 * ------------------------------------------------------------------------- */

/* Qwen3RMSNorm of `rows` rows: y = w * to_dtype(x * rsqrt(mean(x^2) + eps)),
 * mean and rsqrt in fp32.  Strides in elements. */
DDT_API int ddt_rms_norm(const void* x, int dtype, int64_t x_row_stride, const void* weight, void* y,
                         int64_t y_row_stride, int64_t rows, int64_t cols, float eps, ddt_stream_t stream);

/* q_norm / k_norm (RMSNorm over head_dim = 128), the rotary embedding
 * (x * cos) + (rotate_half(x) * sin), and the append of the new K/V rows:
 *   - K/V rows: ctx_rows context rows (ctx_k / ctx_v) then new_rows rows
 *     (new_k / new_v), each [rows, hkv * 128]; cos / sin have one row per
 *     K/V row, in that order;
 *   - queries: q_raw [new_rows, hq * 128], one per new row; rotated queries
 *     go to q_out [new_rows, hq * 128];
 *   - cache rows (device int32 rs = {start, ctx_offset, ctx_count}): new
 *     row r goes to start + r, context row r < ctx_count to ctx_offset + r
 *     (rows >= ctx_count are not written), rows outside [0, cache_rows) are
 *     skipped.  V is written unchanged.  Strides in elements. */
DDT_API int ddt_qk_norm_rope_append(int dtype, const void* q_raw, int64_t q_row_stride, const void* ctx_k,
                                    const void* ctx_v, int64_t ctx_row_stride, int64_t ctx_rows, const void* new_k,
                                    const void* new_v, int64_t new_row_stride, int64_t new_rows,
                                    const void* q_norm_weight, const void* k_norm_weight, float eps_q, float eps_k,
                                    const void* cos, const void* sin, int64_t cs_row_stride, int64_t hq, int64_t hkv,
                                    int64_t head_dim, void* q_out, int64_t q_out_row_stride, void* cache_k,
                                    void* cache_v, int64_t cache_head_stride, int64_t cache_row_stride,
                                    int64_t cache_rows, const int32_t* rs, ddt_stream_t stream);

/* out = to_dtype(silu(gate)) * up, elementwise over n contiguous values
 * (Qwen3MLP's act_fn(gate_proj(x)) * up_proj(x)). */
DDT_API int ddt_silu_mul(const void* gate, const void* up, void* out, int dtype, int64_t n, ddt_stream_t stream);

/* The same over `rows` rows of `cols` values: gate and up share the row
 * stride in_row_stride (e.g. the two halves of one [rows, 2 * cols] gate/up
 * projection), out has out_row_stride.  Strides in elements. */
DDT_API int ddt_silu_mul_rows(const void* gate, const void* up, int64_t in_row_stride, void* out,
                              int64_t out_row_stride, int64_t rows, int64_t cols, int dtype, ddt_stream_t stream);

/* Weight-streaming GEMM for the projections of the verify and draft
 * forwards (the target's and the draft's linear layers and lm_head run by
 * ddtree.py:476-486 and :523-531), at decode sizes:
 *   y[t, n] = sum_k x[t, k] * w[n, k] (+ residual[t, n]),   0 < T <= 128,
 * bf16 in and out, fp32 accumulation on the tensor cores, the residual added
 * in fp32 before the single rounding (torch.addmm).  N a multiple of 128, K
 * of 64; x and w 16-byte aligned with row strides of multiples of 8
 * elements (strides in elements).  The K range is split across up to 8
 * CTAs of a thread-block cluster (splits 0 = chosen from the shape and the
 * SM count, else the caller's count, capped at 8 and at K / 64), whose
 * partials are summed in cluster-rank order, so results do not depend on
 * timing.  Workspace: the status word, zero-filled once,
 * ddt_wgemm_workspace_size bytes, 256-byte aligned. */
DDT_API size_t ddt_wgemm_workspace_size(int64_t T, int64_t N, int64_t K);
DDT_API int ddt_wgemm(const void* x, int64_t x_stride, int64_t T, const void* w, int64_t w_stride, int64_t N,
                      int64_t K, const void* residual /* nullable */, int64_t r_stride, void* y, int64_t y_stride,
                      int64_t splits, void* workspace, size_t workspace_bytes, ddt_stream_t stream);
/* The MLP's first half, act(x Wg^T) * (x Wu^T) with SiLU, in one launch.
 * w_gate_up: [N2, K] bf16 with the gate and up rows interleaved in blocks
 * of 64 (rows 128b .. 128b+63 = gate rows 64b .., rows 128b+64 .. = the same
 * up rows); N2 a multiple of 128.  y: [T, N2 / 2].  Each product is rounded
 * to bf16, the SiLU is rounded, then the product (the order of
 * act_fn(gate_proj(x)) * up_proj(x) in bf16, model/dflash.py and the HF
 * Qwen3 MLP).  Same limits and workspace as ddt_wgemm. */
DDT_API int ddt_wgemm_gate_up(const void* x, int64_t x_stride, int64_t T, const void* w_gate_up, int64_t w_stride,
                              int64_t N2, int64_t K, void* y, int64_t y_stride, int64_t splits, void* workspace,
                              size_t workspace_bytes, ddt_stream_t stream);
/* The draft's lm_head fused with the first step of the tree build
 * (ddtree.py:476-485 computes the draft logits, :136-139 their top-k and
 * log-softmax): ddt_wgemm's y = x w^T (bf16, no residual, no K split),
 * plus, for every token row t and every block of 128 rows of w (128 vocabulary
 * entries), the block's max logit, its sum of exp(logit - max) and its
 * largest (logit, then lower id) key, written to `stats`
 * (ddt_wgemm_head_stats_size bytes, 256-aligned).  ddt_tree_build_head reads
 * them instead of scanning the whole logits.  N a multiple of 128. */
DDT_API size_t ddt_wgemm_head_stats_size(int64_t T, int64_t N);
DDT_API int ddt_wgemm_head(const void* x, int64_t x_stride, int64_t T, const void* w, int64_t w_stride, int64_t N,
                           int64_t K, void* y, int64_t y_stride, void* stats, size_t stats_bytes, void* workspace,
                           size_t workspace_bytes, ddt_stream_t stream);

/* ---------------------------------------------------------------------------
 * EAGLE3 path acceptance.  Replaces evaluate_eagle3_posterior
 * (eagle3.py:46-79) for temperature 0: argmax of every verify row, the
 * longest accepted prefix over the rows of retrieve_indices (-1 padded),
 * first best path on ties, and the bonus token of the last accepted row.
 * out_info: [4] int64 = {best_candidate, accept_length, sample_token, -};
 * accepted: [width] int64 (first accept_length + 1 entries valid).
 * ------------------------------------------------------------------------- */
DDT_API int ddt_eagle3_accept(const void* logits, int dtype, int64_t n_rows, int64_t vocab, int64_t row_stride,
                      const int64_t* draft_tokens, const int64_t* retrieve, int64_t leaves, int64_t width,
                      int64_t* posterior /* [n_rows], nullable */, int64_t* out_info, int64_t* accepted,
                      void* workspace, size_t workspace_bytes, ddt_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* DDTREE_B200_H */
