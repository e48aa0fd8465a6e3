"""Torch-facing wrappers of the C-ABI entry points (device tensors in, device
tensors out, launched on the current CUDA stream)."""
from __future__ import annotations

import ctypes
import math
from contextlib import contextmanager
from dataclasses import dataclass

import torch

from . import _lib
from ._lib import AttentionArgs, TreeOutputs, WORKSPACES, check, dtype_code, ptr, require_cuda, stream_of


def vis_words_for(n_rows: int) -> int:
    return max(1, (int(n_rows) + 31) // 32)


@dataclass
class DeviceTree:
    """Outputs of the tree-build kernel, resident on the device.

    node i (1-based) of the tree is row i of the verify batch; row 0 is the
    root.  ``visibility`` holds one row of packed ancestor bits per verify
    row (int32 words carrying uint32 bit patterns)."""

    budget: int
    rows: int
    topk: int
    top_ids: torch.Tensor
    top_lp: torch.Tensor
    node_token_ids: torch.Tensor
    node_depths: torch.Tensor
    parents: torch.Tensor
    visibility: torch.Tensor
    verify_ids: torch.Tensor
    verify_pos: torch.Tensor
    info: torch.Tensor

    @classmethod
    def allocate(cls, rows: int, vocab: int, budget: int, device: torch.device) -> "DeviceTree":
        b = max(int(budget), 0)
        k = min(b, int(vocab)) if b > 0 else 0
        W = vis_words_for(b + 1)
        i64 = dict(dtype=torch.int64, device=device)
        return cls(
            budget=b, rows=int(rows), topk=k,
            top_ids=torch.empty((rows, max(k, 1)), **i64),
            top_lp=torch.empty((rows, max(k, 1)), dtype=torch.float32, device=device),
            node_token_ids=torch.empty((max(b, 1),), **i64),
            node_depths=torch.empty((max(b, 1),), **i64),
            parents=torch.empty((b + 1,), dtype=torch.int32, device=device),
            visibility=torch.zeros((b + 1, W), dtype=torch.int32, device=device),
            verify_ids=torch.empty((b + 1,), **i64),
            verify_pos=torch.empty((b + 1,), **i64),
            info=torch.zeros((4,), dtype=torch.int32, device=device),
        )

    def c_outputs(self) -> TreeOutputs:
        return TreeOutputs(
            top_ids=ptr(self.top_ids), top_lp=ptr(self.top_lp), node_token_ids=ptr(self.node_token_ids),
            node_depths=ptr(self.node_depths), parents=ptr(self.parents), visibility=ptr(self.visibility),
            vis_words=self.visibility.shape[1], verify_ids=ptr(self.verify_ids), verify_pos=ptr(self.verify_pos),
            info=ptr(self.info))


def tree_build(draft_logits: torch.Tensor, budget: int, root_token: torch.Tensor | None = None, start: int = 0,
               out: DeviceTree | None = None, head_stats: torch.Tensor | None = None) -> DeviceTree:
    """Kernel (1) on ``draft_logits`` [rows, vocab] (fp32 / bf16 / fp16).
    With ``head_stats`` (from ``wgemm_head`` on the same bf16 logits) it
    reads the head's block statistics instead of scanning every logit
    (``ddt_tree_build_head``)."""
    require_cuda(draft_logits, "draft_logits")
    if draft_logits.dim() != 2:
        raise ValueError("draft_logits must be [rows, vocab]")
    if draft_logits.stride(1) != 1:
        draft_logits = draft_logits.contiguous()
    rows, vocab = draft_logits.shape
    dev = draft_logits.device
    if out is None:
        out = DeviceTree.allocate(rows, vocab, budget, dev)
    lib = _lib.load()
    ws_bytes = lib.ddt_tree_build_workspace_size(rows, vocab, max(int(budget), 0))
    ws = WORKSPACES.get("tree_build", dev, ws_bytes)
    if root_token is not None:
        require_cuda(root_token, "root_token")
        if root_token.dtype != torch.int64:
            raise TypeError("root_token must be int64")
    o = out.c_outputs()
    if head_stats is not None:
        if draft_logits.dtype != torch.bfloat16:
            raise TypeError("head statistics come with bf16 logits")
        require_cuda(head_stats, "head_stats")
        rc = lib.ddt_tree_build_head(ptr(draft_logits), rows, vocab, draft_logits.stride(0), ptr(head_stats),
                                     int(budget), ptr(root_token), int(start), ctypes.byref(o), ptr(ws), ws.numel(),
                                     stream_of(dev))
        check(rc, "ddt_tree_build_head")
        return out
    rc = lib.ddt_tree_build(ptr(draft_logits), dtype_code(draft_logits.dtype), rows, vocab, draft_logits.stride(0),
                            int(budget), ptr(root_token), int(start), ctypes.byref(o), ptr(ws), ws.numel(),
                            stream_of(dev))
    check(rc, "ddt_tree_build")
    return out


def tree_from_log_probs(lp: torch.Tensor, ids: torch.Tensor, budget: int, root_token: torch.Tensor | None = None,
                        start: int = 0, out: DeviceTree | None = None) -> DeviceTree:
    """Best-first expansion alone from given [rows, topk] log-probs and ids
    (into ``out``, a DeviceTree of the same rows / topk / budget, when given)."""
    require_cuda(lp, "lp")
    require_cuda(ids, "ids")
    lp = lp.to(torch.float32).contiguous()
    ids = ids.to(torch.int64).contiguous()
    rows, topk = lp.shape
    if out is None:
        out = DeviceTree.allocate(rows, topk, budget, lp.device)
    elif out.budget != int(budget) or out.rows != rows or out.visibility.shape[1] < vis_words_for(int(budget) + 1):
        raise ValueError("out was allocated for another tree shape")
    o = out.c_outputs()
    rc = _lib.load().ddt_tree_from_log_probs(ptr(lp), ptr(ids), rows, topk, int(budget), ptr(root_token), int(start),
                                             ctypes.byref(o), stream_of(lp.device))
    check(rc, "ddt_tree_from_log_probs")
    return out


def tree_mask_fill(mask2d: torch.Tensor, past_length: int, n_rows: int, visibility: torch.Tensor,
                   prev_start: int, prev_len: int) -> None:
    """Write the additive-mask rows of a tree into ``mask2d`` [rows_cap, cols]."""
    require_cuda(mask2d, "mask")
    if mask2d.stride(1) != 1:
        raise ValueError("mask rows must be contiguous")
    min_value = torch.finfo(mask2d.dtype).min
    rc = _lib.load().ddt_tree_mask_fill(ptr(mask2d), dtype_code(mask2d.dtype), mask2d.stride(0), mask2d.shape[0],
                                        int(past_length), int(n_rows), ptr(visibility), visibility.shape[1],
                                        int(prev_start), int(prev_len), float(min_value),
                                        stream_of(mask2d.device))
    check(rc, "ddt_tree_mask_fill")


def mask_to_bits(mask2d: torch.Tensor, col_offset: int, n_rows: int, out: torch.Tensor | None = None) -> torch.Tensor:
    """Pack the [n_rows, n_rows] tree block of a dense mask at ``col_offset``."""
    require_cuda(mask2d, "mask")
    if mask2d.stride(1) != 1:
        mask2d = mask2d.contiguous()
    W = vis_words_for(n_rows)
    if out is None:
        out = torch.empty((n_rows, W), dtype=torch.int32, device=mask2d.device)
    rc = _lib.load().ddt_mask_to_bits(ptr(mask2d), dtype_code(mask2d.dtype), mask2d.stride(0), int(col_offset),
                                      int(n_rows), ptr(out), W, stream_of(mask2d.device))
    check(rc, "ddt_mask_to_bits")
    return out


_ATT_WS: dict = {}


def tree_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, past_length: int, visibility: torch.Tensor,
                   scale: float, out: torch.Tensor | None = None, key_lo: torch.Tensor | None = None,
                   past_dev: torch.Tensor | None = None, workspace: torch.Tensor | None = None,
                   stable_dev: torch.Tensor | None = None) -> torch.Tensor:
    """Kernel (2): one layer of tree-masked attention.

    q [n_tokens, hq, 128], k / v [hkv, kv_rows, 128] (bf16, last dim
    contiguous, any other strides), visibility [n_tokens, W] int32.
    Returns out [n_tokens, hq, 128] bf16.

    ``key_lo`` (int64 [n_tokens] on the device) makes it a sliding-window
    layer: row t then sees prefix key j only if j >= key_lo[t]
    (``ddt_tree_attention_window``; see ``ddtree.sliding_key_lo``).

    ``past_dev`` (int32 device scalar) makes the prefix length a run-time
    value (``ddt_tree_attention_dev``): ``past_length`` is then its upper
    bound, and one captured launch serves any prefix up to it.  ``workspace``
    (uint8, 256-aligned) is the caller's own scratch, needed when the launch
    is captured into a graph that must outlive the shared scratch.
    ``stable_dev`` (int32 device scalar, with ``past_dev``): keys below it are
    written by nothing still running on the stream, so their K tiles may load
    before the preceding kernel has finished.

    Called once per layer, so the host work is kept to one read of each
    tensor's shape and strides; the C entry point checks the rest."""
    try:
        on_gpu = q.is_cuda and k.is_cuda and v.is_cuda and visibility.is_cuda
    except AttributeError:
        on_gpu = False
    if not on_gpu:
        for t, n in ((q, "q"), (k, "k"), (v, "v"), (visibility, "visibility")):
            require_cuda(t, n)
    if q.dtype == torch.float32 and k.dtype == torch.float32 and v.dtype == torch.float32:
        return tree_attention_f32(q, k, v, past_length, visibility, scale, out=out, key_lo=key_lo, past_dev=past_dev)
    if q.dtype != torch.bfloat16 or k.dtype != torch.bfloat16 or v.dtype != torch.bfloat16:
        raise TypeError("q, k, v must all be bf16 (tensor-core path) or all float32")
    qs, ks = q.stride(), k.stride()
    kshape = k.shape
    if qs[-1] != 1 or ks[-1] != 1:
        raise ValueError("head_dim must be the contiguous dimension")
    if v.stride() != ks or v.shape != kshape:
        raise ValueError("k and v must share shape and strides")
    n_tokens, hq, d = q.shape
    hkv, kv_rows, _ = kshape
    if out is None:
        out = torch.empty((n_tokens, hq, d), dtype=torch.bfloat16, device=q.device)
    if not visibility.is_contiguous():
        visibility = visibility.contiguous()
    dev_index = q.get_device()
    past_length = int(past_length)
    lib = _lib.load()
    if workspace is not None:
        ws = (workspace, workspace.data_ptr(), workspace.numel())
    else:
        key = (n_tokens, hq, hkv, past_length, dev_index)
        ws = _ATT_WS.get(key)
        if ws is None or ws[0] is not WORKSPACES.current("attention", dev_index):
            ws_bytes = lib.ddt_tree_attention_workspace_size(n_tokens, hq, hkv, past_length, dev_index)
            buf = WORKSPACES.get("attention", q.device, ws_bytes)
            ws = (buf, buf.data_ptr(), buf.numel())
            _ATT_WS[key] = ws
    os_ = out.stride()
    a = AttentionArgs(q.data_ptr(), qs[0], qs[1], k.data_ptr(), v.data_ptr(), ks[0], ks[1], kv_rows, out.data_ptr(),
                      os_[0], os_[1], n_tokens, hq, hkv, d, past_length, visibility.data_ptr(),
                      visibility.shape[1], float(scale))
    if past_dev is not None:
        if not past_dev.is_cuda or past_dev.dtype != torch.int32:
            raise ValueError("past_dev must be an int32 CUDA tensor")
        if key_lo is not None and (not key_lo.is_cuda or key_lo.dtype != torch.int64 or not key_lo.is_contiguous()
                                   or key_lo.numel() < n_tokens):
            raise ValueError("key_lo must be a contiguous int64 CUDA tensor with one entry per token")
        if stable_dev is not None and (not stable_dev.is_cuda or stable_dev.dtype != torch.int32):
            raise ValueError("stable_dev must be an int32 CUDA tensor")
        check(lib.ddt_tree_attention_dev(ctypes.byref(a), ptr(key_lo), past_dev.data_ptr(), ptr(stable_dev), ws[1],
                                         ws[2], _lib.raw_stream(dev_index)), "ddt_tree_attention_dev")
        return out
    if key_lo is None:
        check(lib.ddt_tree_attention(ctypes.byref(a), ws[1], ws[2], _lib.raw_stream(dev_index)), "ddt_tree_attention")
        return out
    if not key_lo.is_cuda or key_lo.dtype != torch.int64 or not key_lo.is_contiguous() or key_lo.numel() < n_tokens:
        raise ValueError("key_lo must be a contiguous int64 CUDA tensor with one entry per token")
    check(lib.ddt_tree_attention_window(ctypes.byref(a), key_lo.data_ptr(), ws[1], ws[2], _lib.raw_stream(dev_index)),
          "ddt_tree_attention_window")
    return out


def tree_attention_f32(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, past_length: int,
                       visibility: torch.Tensor, scale: float, out: torch.Tensor | None = None,
                       key_lo: torch.Tensor | None = None, past_dev: torch.Tensor | None = None) -> torch.Tensor:
    """Float32 tree attention (``ddt_tree_attention_f32``): the layouts of
    ``tree_attention`` with float32 tensors.  ``past_dev`` (int32 device
    scalar) makes the prefix length a run-time value; ``past_length`` is then
    its upper bound."""
    for t, n in ((q, "q"), (k, "k"), (v, "v"), (visibility, "visibility")):
        require_cuda(t, n)
    if q.dtype != torch.float32 or k.dtype != torch.float32 or v.dtype != torch.float32:
        raise TypeError("q, k, v must be float32")
    qs, ks = q.stride(), k.stride()
    if qs[-1] != 1 or ks[-1] != 1:
        raise ValueError("head_dim must be the contiguous dimension")
    if v.stride() != ks or v.shape != k.shape:
        raise ValueError("k and v must share shape and strides")
    n_tokens, hq, d = q.shape
    hkv, kv_rows, _ = k.shape
    if out is None:
        out = torch.empty((n_tokens, hq, d), dtype=torch.float32, device=q.device)
    if out.dtype != torch.float32:
        raise TypeError("out must be float32")
    if not visibility.is_contiguous():
        visibility = visibility.contiguous()
    if key_lo is not None and (not key_lo.is_cuda or key_lo.dtype != torch.int64 or not key_lo.is_contiguous()
                               or key_lo.numel() < n_tokens):
        raise ValueError("key_lo must be a contiguous int64 CUDA tensor with one entry per token")
    if past_dev is not None and (not past_dev.is_cuda or past_dev.dtype != torch.int32):
        raise ValueError("past_dev must be an int32 CUDA tensor")
    os_ = out.stride()
    a = AttentionArgs(q.data_ptr(), qs[0], qs[1], k.data_ptr(), v.data_ptr(), ks[0], ks[1], kv_rows, out.data_ptr(),
                      os_[0], os_[1], n_tokens, hq, hkv, d, int(past_length), visibility.data_ptr(),
                      visibility.shape[1], float(scale))
    check(_lib.load().ddt_tree_attention_f32(ctypes.byref(a), ptr(key_lo), ptr(past_dev), stream_of(q.device)),
          "ddt_tree_attention_f32")
    return out


def attention_workspace(n_tokens: int, hq: int, hkv: int, max_past: int, device: torch.device) -> torch.Tensor:
    """A caller-owned, zero-filled attention workspace for prefixes up to
    ``max_past`` (status word first)."""
    index = device.index if device.index is not None else torch.cuda.current_device()
    n = _lib.load().ddt_tree_attention_workspace_size(int(n_tokens), int(hq), int(hkv), int(max_past), index)
    return torch.zeros(max(int(n), 256), dtype=torch.uint8, device=device)


def attention_status(device: torch.device, workspace: torch.Tensor | None = None) -> int:
    """Device-side status word of the attention kernel (0 = no bounded wait
    ran out), of the shared scratch or of a caller's ``workspace``."""
    ws = WORKSPACES.get("attention", device, 256) if workspace is None else workspace
    return int(ws[:4].view(torch.int32).item())


def rms_norm(x: torch.Tensor, weight: torch.Tensor, eps: float, out: torch.Tensor | None = None) -> torch.Tensor:
    """Qwen3RMSNorm over the last dim of a [rows, cols] tensor (``ddt_rms_norm``)."""
    require_cuda(x, "x")
    if x.dim() != 2 or x.stride(1) != 1 or weight.dtype != x.dtype or not weight.is_contiguous():
        raise ValueError("x must be [rows, cols] with contiguous rows; weight contiguous, same dtype")
    if out is None:
        out = torch.empty_like(x, memory_format=torch.contiguous_format)
    check(_lib.load().ddt_rms_norm(x.data_ptr(), dtype_code(x.dtype), x.stride(0), weight.data_ptr(), out.data_ptr(),
                                   out.stride(0), x.shape[0], x.shape[1], float(eps), stream_of(x.device)),
          "ddt_rms_norm")
    return out


def qk_norm_rope_append(q_raw: torch.Tensor, new_k: torch.Tensor, new_v: torch.Tensor, q_norm_w: torch.Tensor,
                        k_norm_w: torch.Tensor, eps_q: float, eps_k: float, cos: torch.Tensor, sin: torch.Tensor,
                        cache_k: torch.Tensor, cache_v: torch.Tensor, rs: torch.Tensor, hq: int, hkv: int,
                        ctx_k: torch.Tensor | None = None, ctx_v: torch.Tensor | None = None,
                        q_out: torch.Tensor | None = None) -> torch.Tensor:
    """``ddt_qk_norm_rope_append``: q_raw [T, hq*128], new_k / new_v [T,
    hkv*128] (optional ctx_k / ctx_v [C, hkv*128] before them), cos / sin
    [C + T, 128]; cache_k / cache_v [hkv, rows, 128] (any leading size-1
    dims); rs int32 device [start, ctx_offset, ctx_count].  Returns the
    rotated queries [T, hq, 128]."""
    T = q_raw.shape[0]
    C = 0 if ctx_k is None else ctx_k.shape[0]
    for t in (q_raw, new_k, new_v, cos, sin) + (() if ctx_k is None else (ctx_k, ctx_v)):
        if t.dim() != 2 or t.stride(1) != 1 or t.dtype != q_raw.dtype or not t.is_cuda:
            raise ValueError("q / k / v / cos / sin must be 2-D CUDA tensors of one dtype with contiguous rows")
    if new_k.stride() != new_v.stride() or (ctx_k is not None and ctx_k.stride() != ctx_v.stride()):
        raise ValueError("K and V must share strides")
    if cos.stride() != sin.stride() or cos.shape[0] < C + T:
        raise ValueError("cos / sin need one row per K/V row")
    ck = cache_k.reshape(-1, cache_k.shape[-2], cache_k.shape[-1])
    cv = cache_v.reshape(-1, cache_v.shape[-2], cache_v.shape[-1])
    if ck.data_ptr() != cache_k.data_ptr() or ck.stride() != cv.stride() or ck.shape[0] != hkv:
        raise ValueError("cache K/V must be [hkv, rows, 128] views sharing strides")
    if q_out is None:
        q_out = torch.empty((T, hq, 128), dtype=q_raw.dtype, device=q_raw.device)
    rc = _lib.load().ddt_qk_norm_rope_append(
        dtype_code(q_raw.dtype), q_raw.data_ptr(), q_raw.stride(0), ptr(ctx_k), ptr(ctx_v),
        0 if ctx_k is None else ctx_k.stride(0), C, new_k.data_ptr(), new_v.data_ptr(), new_k.stride(0), T,
        q_norm_w.data_ptr(), k_norm_w.data_ptr(), float(eps_q), float(eps_k), cos.data_ptr(), sin.data_ptr(),
        cos.stride(0), hq, hkv, 128, q_out.data_ptr(), q_out.stride(0), ck.data_ptr(), cv.data_ptr(), ck.stride(0),
        ck.stride(1), ck.shape[1], rs.data_ptr(), stream_of(q_raw.device))
    check(rc, "ddt_qk_norm_rope_append")
    return q_out


def silu_mul(gate: torch.Tensor, up: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """to_dtype(silu(gate)) * up: contiguous tensors (``ddt_silu_mul``) or
    2-D [rows, cols] views sharing a row stride, such as the two halves of
    one gate/up projection (``ddt_silu_mul_rows``)."""
    if gate.shape != up.shape or gate.dtype != up.dtype:
        raise ValueError("gate and up must be alike")
    if gate.is_contiguous() and up.is_contiguous():
        if out is None:
            out = torch.empty_like(gate)
        check(_lib.load().ddt_silu_mul(gate.data_ptr(), up.data_ptr(), out.data_ptr(), dtype_code(gate.dtype),
                                       gate.numel(), stream_of(gate.device)), "ddt_silu_mul")
        return out
    if gate.dim() != 2 or gate.stride(1) != 1 or gate.stride() != up.stride():
        raise ValueError("strided gate / up must be [rows, cols] views with one row stride")
    rows, cols = gate.shape
    if out is None:
        out = torch.empty((rows, cols), dtype=gate.dtype, device=gate.device)
    check(_lib.load().ddt_silu_mul_rows(gate.data_ptr(), up.data_ptr(), gate.stride(0), out.data_ptr(),
                                        out.stride(0), rows, cols, dtype_code(gate.dtype), stream_of(gate.device)),
          "ddt_silu_mul_rows")
    return out


_WGEMM_WS_BYTES = 4096
_WGEMM_WS: dict = {}


def _wgemm_workspace(device: torch.device) -> torch.Tensor:
    """One fixed, zero-filled scratch per device holding the status word of
    ``wgemm`` (split-K partials are reduced across the cluster in shared
    memory, so nothing else is needed); allocated once and never replaced,
    so launches captured into a graph keep a valid address."""
    index = device.index if device.index is not None else torch.cuda.current_device()
    ws = _WGEMM_WS.get(index)
    if ws is None:
        ws = torch.zeros(_WGEMM_WS_BYTES, dtype=torch.uint8, device=device)
        _WGEMM_WS[index] = ws
    return ws


def wgemm_supported(x: torch.Tensor, w: torch.Tensor) -> bool:
    """Shapes the weight-streaming GEMM takes: bf16, 1-128 rows of x, weight
    rows a multiple of 128, K a multiple of 64, 16-byte aligned rows."""
    return (x.dtype == torch.bfloat16 and w.dtype == torch.bfloat16 and x.dim() == 2 and w.dim() == 2
            and 1 <= x.shape[0] <= 128 and w.shape[0] % 128 == 0 and w.shape[1] % 64 == 0 and x.shape[1] == w.shape[1]
            and x.stride(1) == 1 and w.stride(1) == 1 and x.stride(0) % 8 == 0 and w.stride(0) % 8 == 0
            and x.data_ptr() % 16 == 0 and w.data_ptr() % 16 == 0 and x.is_cuda and w.is_cuda)


def wgemm(x: torch.Tensor, w: torch.Tensor, residual: torch.Tensor | None = None,
          out: torch.Tensor | None = None, splits: int = 0) -> torch.Tensor:
    """y = x @ w.T (+ residual) on the weight-streaming tcgen05 GEMM
    (``ddt_wgemm``): x [T <= 128, K], w [N, K] bf16; the residual is added in
    fp32 before the one rounding, as ``torch.addmm`` does."""
    if not wgemm_supported(x, w):
        raise ValueError("wgemm: unsupported shapes / layout (see wgemm_supported)")
    T, K = x.shape
    N = w.shape[0]
    if out is None:
        out = torch.empty((T, N), dtype=torch.bfloat16, device=x.device)
    if residual is not None and (residual.dtype != torch.bfloat16 or residual.stride(1) != 1
                                 or tuple(residual.shape) != (T, N)):
        raise ValueError("residual must be [T, N] bf16 with contiguous rows")
    if out.dtype != torch.bfloat16 or out.stride(1) != 1 or tuple(out.shape) != (T, N):
        raise ValueError("out must be [T, N] bf16 with contiguous rows")
    lib = _lib.load()
    need = lib.ddt_wgemm_workspace_size(T, N, K)
    ws = _wgemm_workspace(x.device)
    if need > ws.numel():
        raise ValueError(f"wgemm workspace of {ws.numel()} bytes is smaller than the {need} needed")
    rc = lib.ddt_wgemm(x.data_ptr(), x.stride(0), T, w.data_ptr(), w.stride(0), N, K, ptr(residual),
                       0 if residual is None else residual.stride(0), out.data_ptr(), out.stride(0), int(splits),
                       ws.data_ptr(), ws.numel(), _lib.raw_stream(x.device.index))
    check(rc, "ddt_wgemm")
    return out


def head_stats_buffer(rows: int, vocab: int, device: torch.device) -> torch.Tensor:
    """Scratch for ``wgemm_head``'s block statistics of [rows, vocab] logits."""
    return torch.empty(_lib.load().ddt_wgemm_head_stats_size(rows, vocab), dtype=torch.uint8, device=device)


def wgemm_head(x: torch.Tensor, w: torch.Tensor, stats: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """Logits y = x @ w.T of a bias-free lm_head on the weight-streaming GEMM
    (``ddt_wgemm_head``), with the per-block statistics that
    ``tree_build(..., head_stats=stats)`` reads written to ``stats`` (from
    ``head_stats_buffer``).  The logits equal ``wgemm(x, w)``'s."""
    if not wgemm_supported(x, w):
        raise ValueError("wgemm_head: unsupported shapes / layout (see wgemm_supported)")
    T, K = x.shape
    N = w.shape[0]
    if out is None:
        out = torch.empty((T, N), dtype=torch.bfloat16, device=x.device)
    if out.dtype != torch.bfloat16 or out.stride(1) != 1 or tuple(out.shape) != (T, N):
        raise ValueError("out must be [T, N] bf16 with contiguous rows")
    lib = _lib.load()
    ws = _wgemm_workspace(x.device)
    rc = lib.ddt_wgemm_head(x.data_ptr(), x.stride(0), T, w.data_ptr(), w.stride(0), N, K, out.data_ptr(),
                            out.stride(0), stats.data_ptr(), stats.numel(), ws.data_ptr(), ws.numel(),
                            _lib.raw_stream(x.device.index))
    check(rc, "ddt_wgemm_head")
    return out


def interleave_gate_up(w_gate: torch.Tensor, w_up: torch.Tensor) -> torch.Tensor:
    """[Wg; Wu] packed for ``wgemm_gate_up``: blocks of 64 gate rows, each
    followed by the same 64 up rows (I a multiple of 64)."""
    inter, k = w_gate.shape
    if w_up.shape != w_gate.shape or inter % 64:
        raise ValueError("gate and up weights must share a [I, K] shape with I a multiple of 64")
    return torch.stack([w_gate.reshape(inter // 64, 64, k), w_up.reshape(inter // 64, 64, k)], 1).reshape(2 * inter, k)


def wgemm_gate_up(x: torch.Tensor, w_packed: torch.Tensor, out: torch.Tensor | None = None,
                  splits: int = 0) -> torch.Tensor:
    """act(x Wg^T) * (x Wu^T) with SiLU in one launch (``ddt_wgemm_gate_up``):
    x [T <= 128, K] bf16, w_packed from ``interleave_gate_up`` [2I, K]; each
    product, the SiLU and the final product rounded to bf16 in the order of
    ``act_fn(gate_proj(x)) * up_proj(x)``.  Returns [T, I]."""
    if not wgemm_supported(x, w_packed):
        raise ValueError("wgemm_gate_up: unsupported shapes / layout (see wgemm_supported)")
    T, K = x.shape
    N2 = w_packed.shape[0]
    if out is None:
        out = torch.empty((T, N2 // 2), dtype=torch.bfloat16, device=x.device)
    if out.dtype != torch.bfloat16 or out.stride(1) != 1 or tuple(out.shape) != (T, N2 // 2):
        raise ValueError("out must be [T, I] bf16 with contiguous rows")
    ws = _wgemm_workspace(x.device)
    rc = _lib.load().ddt_wgemm_gate_up(x.data_ptr(), x.stride(0), T, w_packed.data_ptr(), w_packed.stride(0), N2, K,
                                       out.data_ptr(), out.stride(0), int(splits), ws.data_ptr(), ws.numel(),
                                       _lib.raw_stream(x.device.index))
    check(rc, "ddt_wgemm_gate_up")
    return out


@contextmanager
def pdl(enabled: bool = True):
    """Launch this library's decode-layer kernels as programmatic dependent
    launches (``ddt_set_pdl``) inside the block: each may start while the
    kernel before it is still running, and the weight-streaming GEMMs load
    their first weight tiles before it completes.  Weights must not be
    written by work queued in the block."""
    lib = _lib.load()
    prev = lib.ddt_set_pdl(1 if enabled else 0)
    try:
        yield
    finally:
        lib.ddt_set_pdl(prev)


def wgemm_status(device: torch.device) -> int:
    """Status word of the wgemm scratch (0 = no bounded wait ran out)."""
    return int(_wgemm_workspace(device)[:4].view(torch.int32).item())


def kv_append(k_src: torch.Tensor, v_src: torch.Tensor, k_dst: torch.Tensor, v_dst: torch.Tensor,
              offset_dev: torch.Tensor, rows_dev: torch.Tensor | None = None) -> None:
    """Copy rows [0, rows) of k_src / v_src ([..., heads, rows, dim]) into
    rows offset .. offset + rows of k_dst / v_dst ([..., heads, capacity,
    dim]) with the offset (and optionally a row count) read from device
    int32 scalars (``ddt_kv_append``)."""
    for t, n in ((k_src, "k_src"), (v_src, "v_src"), (k_dst, "k_dst"), (v_dst, "v_dst"), (offset_dev, "offset")):
        require_cuda(t, n)
    if offset_dev.dtype != torch.int32 or (rows_dev is not None and rows_dev.dtype != torch.int32):
        raise ValueError("offset_dev / rows_dev must be int32")
    ks = k_src.reshape(-1, k_src.shape[-2], k_src.shape[-1]) if k_src.dim() != 3 else k_src
    vs = v_src.reshape(-1, v_src.shape[-2], v_src.shape[-1]) if v_src.dim() != 3 else v_src
    kd = k_dst.reshape(-1, k_dst.shape[-2], k_dst.shape[-1]) if k_dst.dim() != 3 else k_dst
    vd = v_dst.reshape(-1, v_dst.shape[-2], v_dst.shape[-1]) if v_dst.dim() != 3 else v_dst
    if ks.stride() != vs.stride() or ks.shape != vs.shape or kd.stride() != vd.stride() or kd.shape != vd.shape:
        raise ValueError("K and V must share shapes and strides")
    if ks.shape[0] != kd.shape[0] or ks.shape[-1] != kd.shape[-1] or ks.dtype != kd.dtype:
        raise ValueError("source and cache heads / head_dim / dtype differ")
    if ks.stride(-1) != 1 or kd.stride(-1) != 1:
        raise ValueError("head_dim must be contiguous")
    e = ks.element_size()
    rc = _lib.load().ddt_kv_append(ks.data_ptr(), vs.data_ptr(), ks.stride(0) * e, ks.stride(1) * e, kd.data_ptr(),
                                   vd.data_ptr(), kd.stride(0) * e, kd.stride(1) * e, kd.shape[1], ks.shape[0],
                                   ks.shape[1], ks.shape[2] * e, offset_dev.data_ptr(), ptr(rows_dev),
                                   stream_of(ks.device))
    check(rc, "ddt_kv_append")


def tree_accept(logits: torch.Tensor, parents: torch.Tensor, node_token_ids: torch.Tensor,
                n_nodes_dev: torch.Tensor | None = None, max_accept: int | None = None,
                accepted: torch.Tensor | None = None, accept_info: torch.Tensor | None = None,
                posterior: torch.Tensor | None = None):
    """Kernel (3a): argmax of every verify row + walk down the tree.

    Returns (accepted [max_accept] int64, accept_info [2] int64 = {count,
    next_token}, posterior [n_rows] int64)."""
    require_cuda(logits, "logits")
    if logits.dim() == 3:
        logits = logits[0]
    if logits.stride(1) != 1:
        logits = logits.contiguous()
    n_rows, vocab = logits.shape
    dev = logits.device
    if max_accept is None:
        max_accept = n_rows
    if accepted is None:
        accepted = torch.zeros((max_accept,), dtype=torch.int64, device=dev)
    if accept_info is None:
        accept_info = torch.zeros((2,), dtype=torch.int64, device=dev)
    if posterior is None:
        posterior = torch.empty((n_rows,), dtype=torch.int64, device=dev)
    lib = _lib.load()
    ws = WORKSPACES.get("accept", dev, lib.ddt_tree_accept_workspace_size(n_rows, vocab))
    rc = lib.ddt_tree_accept(ptr(logits), dtype_code(logits.dtype), n_rows, vocab, logits.stride(0), ptr(parents),
                             ptr(node_token_ids), ptr(n_nodes_dev), ptr(posterior), ptr(accepted), int(max_accept),
                             ptr(accept_info), ptr(ws), ws.numel(), stream_of(dev))
    check(rc, "ddt_tree_accept")
    return accepted, accept_info, posterior


def tree_walk(posterior: torch.Tensor, parents: torch.Tensor, node_token_ids: torch.Tensor,
              n_nodes_dev: torch.Tensor | None = None, max_accept: int | None = None):
    """Walk alone from a device posterior [n_rows].  Returns (accepted, accept_info)."""
    require_cuda(posterior, "posterior")
    post = posterior.reshape(-1).to(torch.int64).contiguous()
    n_rows = post.numel()
    dev = post.device
    max_accept = n_rows if max_accept is None else max_accept
    accepted = torch.zeros((max_accept,), dtype=torch.int64, device=dev)
    accept_info = torch.zeros((2,), dtype=torch.int64, device=dev)
    rc = _lib.load().ddt_tree_walk(ptr(post), n_rows, ptr(parents), ptr(node_token_ids), ptr(n_nodes_dev),
                                   ptr(accepted), int(max_accept), ptr(accept_info), stream_of(dev))
    check(rc, "ddt_tree_walk")
    return accepted, accept_info


def sample_rows(logits: torch.Tensor, temperature: float, seed: int, offset: int = 0,
                out: torch.Tensor | None = None) -> torch.Tensor:
    """One token per row drawn from softmax(logits / temperature)
    (``ddt_sample_rows``): int64 of shape ``logits.shape[:-1]``.  The same
    (seed, offset) gives the same draws."""
    require_cuda(logits, "logits")
    shape = logits.shape
    x = logits.reshape(-1, shape[-1])
    if x.stride(1) != 1:
        x = x.contiguous()
    n_rows, vocab = x.shape
    if out is None:
        out = torch.empty((n_rows,), dtype=torch.int64, device=x.device)
    lib = _lib.load()
    ws = WORKSPACES.get("sample", x.device, lib.ddt_sample_rows_workspace_size(n_rows, vocab))
    rc = lib.ddt_sample_rows(ptr(x), dtype_code(x.dtype), n_rows, vocab, x.stride(0), float(temperature),
                             int(seed) & 0xFFFFFFFFFFFFFFFF, int(offset) & 0xFFFFFFFFFFFFFFFF, ptr(out), ptr(ws),
                             ws.numel(), stream_of(x.device))
    check(rc, "ddt_sample_rows")
    return out.view(shape[:-1])


def sample(logits: torch.Tensor, temperature: float = 0.0, generator: torch.Generator | None = None) -> torch.Tensor:
    """``sample(logits, temperature)`` of model/utils.py:28-35 on the device:
    row-wise argmax below temperature 1e-5, otherwise one draw per row from
    softmax(logits / temperature).  The seed of a draw comes from torch's
    CPU generator (or ``generator``), so ``torch.manual_seed`` makes runs
    repeat, as it does for the reference's ``torch.multinomial``."""
    if temperature < 1e-5:
        return argmax_rows(logits)
    seed = int(torch.randint(0, 2 ** 62, (1,), generator=generator).item())
    return sample_rows(logits, temperature, seed)


def argmax_rows(logits: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    require_cuda(logits, "logits")
    shape = logits.shape
    x = logits.reshape(-1, shape[-1])
    if x.stride(1) != 1:
        x = x.contiguous()
    n_rows, vocab = x.shape
    if out is None:
        out = torch.empty((n_rows,), dtype=torch.int64, device=x.device)
    lib = _lib.load()
    ws = WORKSPACES.get("accept", x.device, lib.ddt_tree_accept_workspace_size(n_rows, vocab))
    rc = lib.ddt_argmax_rows(ptr(x), dtype_code(x.dtype), n_rows, vocab, x.stride(0), ptr(out), ptr(ws), ws.numel(),
                             stream_of(x.device))
    check(rc, "ddt_argmax_rows")
    return out.view(shape[:-1])


def eagle3_accept(logits: torch.Tensor, draft_tokens: torch.Tensor, retrieve: torch.Tensor):
    """Kernel (3b): EAGLE3 path acceptance.  Returns (info [4] int64 =
    {best, accept_length, sample_token, 0}, accepted [width] int64, posterior)."""
    require_cuda(logits, "logits")
    x = logits[0] if logits.dim() == 3 else logits
    if x.stride(1) != 1:
        x = x.contiguous()
    n_rows, vocab = x.shape
    dev = x.device
    draft = draft_tokens.reshape(-1).to(device=dev, dtype=torch.int64).contiguous()
    r = retrieve.to(device=dev, dtype=torch.int64).contiguous()
    leaves, width = r.shape
    info = torch.zeros((4,), dtype=torch.int64, device=dev)
    accepted = torch.zeros((width,), dtype=torch.int64, device=dev)
    posterior = torch.empty((n_rows,), dtype=torch.int64, device=dev)
    lib = _lib.load()
    ws = WORKSPACES.get("accept", dev, lib.ddt_tree_accept_workspace_size(n_rows, vocab))
    rc = lib.ddt_eagle3_accept(ptr(x), dtype_code(x.dtype), n_rows, vocab, x.stride(0), ptr(draft), ptr(r), leaves,
                               width, ptr(posterior), ptr(info), ptr(accepted), ptr(ws), ws.numel(), stream_of(dev))
    check(rc, "ddt_eagle3_accept")
    return info, accepted, posterior


class PointerTable:
    """Device array of tensor base pointers, re-uploaded only when they change."""

    def __init__(self):
        self._key = None
        self._dev = None

    def get(self, tensors, device: torch.device) -> torch.Tensor:
        key = tuple(t.data_ptr() for t in tensors)
        if key != self._key or self._dev is None or self._dev.device != device:
            host = torch.tensor(key, dtype=torch.int64)
            self._dev = host.to(device)
            self._key = key
        return self._dev


_PTRS = PointerTable()


def tree_commit(verify_ids: torch.Tensor, accepted: torch.Tensor, accept_info: torch.Tensor,
                output_ids: torch.Tensor, start: int, hidden: torch.Tensor | None = None,
                hidden_out: torch.Tensor | None = None) -> torch.Tensor | None:
    """Kernel (3c): the commit step of a round (ddtree.py:534-548) on the device.

    Writes the accepted verify tokens into ``output_ids[start:start+n]`` and
    the bonus token at ``start+n``, and, with ``hidden`` ([N, H] or [1, N, H],
    last dim contiguous), returns the accepted rows of the hidden features in
    ``hidden_out`` ([max_accept, H]; rows past the count are left as they
    are).  ``n`` and the bonus token come from ``accept_info`` on the device:
    no host sync."""
    for t, n in ((verify_ids, "verify_ids"), (accepted, "accepted"), (accept_info, "accept_info"),
                 (output_ids, "output_ids")):
        require_cuda(t, n)
    vid = verify_ids.reshape(-1)
    if vid.dtype != torch.int64 or not vid.is_contiguous():
        raise ValueError("verify_ids must be contiguous int64")
    if output_ids.dtype != torch.int64 or not output_ids.is_contiguous():
        raise ValueError("output_ids must be contiguous int64")
    if accepted.dtype != torch.int64 or accept_info.dtype != torch.int64:
        raise ValueError("accepted / accept_info must be int64")
    max_accept = accepted.numel()
    row_stride = row_bytes = out_stride = 0
    if hidden is not None:
        require_cuda(hidden, "hidden")
        h = hidden.reshape(-1, hidden.shape[-1]) if hidden.dim() == 3 and hidden.shape[0] == 1 else hidden
        if h.dim() != 2 or h.stride(-1) != 1:
            raise ValueError("hidden must be [N, H] (or [1, N, H]) with a contiguous last dimension")
        if hidden_out is None:
            hidden_out = torch.empty((max_accept, h.shape[1]), dtype=h.dtype, device=h.device)
        if hidden_out.dtype != h.dtype or hidden_out.shape[-1] != h.shape[1] or hidden_out.stride(-1) != 1:
            raise ValueError("hidden_out must match hidden's dtype and width")
        esz = h.element_size()
        row_stride, row_bytes, out_stride = h.stride(0) * esz, h.shape[1] * esz, hidden_out.stride(-2) * esz
        hidden = h
    rc = _lib.load().ddt_tree_commit(ptr(vid), vid.numel(), ptr(accepted), max_accept, ptr(accept_info),
                                     ptr(output_ids), output_ids.numel(), int(start), ptr(hidden), row_stride,
                                     row_bytes, ptr(hidden_out), out_stride, stream_of(vid.device))
    check(rc, "ddt_tree_commit")
    return hidden_out


def kv_compact(tensors, past_length: int, cur_len: int, keep: torch.Tensor, keep_count: torch.Tensor,
               max_keep: int, table: PointerTable | None = None) -> None:
    """In-place compaction of many [..., heads, rows, head_dim] cache tensors
    sharing one layout: rows past+keep[k] -> past+k for k < keep_count."""
    if not tensors:
        return
    t0 = tensors[0]
    require_cuda(t0, "cache tensor")
    for t in tensors:
        if t.shape != t0.shape or t.stride() != t0.stride() or t.dtype != t0.dtype:
            raise ValueError("all cache tensors of one compaction call must share shape, strides and dtype")
    if t0.dim() < 2 or t0.stride(-1) != 1:
        raise ValueError("cache tensors must have a contiguous last dimension")
    esz = t0.element_size()
    heads = math.prod(t0.shape[:-2]) if t0.dim() > 2 else 1
    if t0.dim() > 2:
        # collapse the leading dims into one "head" dimension
        hs = t0.stride(-3)
        for i in range(t0.dim() - 3):
            if t0.stride(i) != t0.stride(i + 1) * t0.shape[i + 1]:
                raise ValueError("leading dimensions must be collapsible")
    else:
        hs = 0
    table = table or _PTRS
    ptrs = table.get(tensors, t0.device)
    rc = _lib.load().ddt_kv_compact(ptr(ptrs), len(tensors), heads, t0.shape[-1] * esz, hs * esz, t0.stride(-2) * esz,
                                    int(past_length), int(cur_len), ptr(keep), ptr(keep_count), int(max_keep),
                                    stream_of(t0.device))
    check(rc, "ddt_kv_compact")
