"""Drop-in replacements for the DDTree step functions of the reference's
``ddtree.py`` (kimwin2/ddtree_eagle3_patch), running on the B200 kernels.

Same names, arguments, return values and error behaviour as:
  build_ddtree_tree      ddtree.py:114-196
  compile_ddtree_tree    ddtree.py:199-287
  follow_verified_tree   ddtree.py:290-301
  compact_dynamic_cache  ddtree.py:323-369
  compact_tail_inplace   ddtree.py:61-88 (the reference's inline C++ op)
plus the fused device-side step ``accept_verified_tree`` (sample + follow on
the GPU, one launch) that the decode loop uses.

There is no CPU path: inputs must live on a CUDA device, and the native
library must be built.
"""
from __future__ import annotations

import time
from types import SimpleNamespace

import numpy as np
import torch

from . import kernels
from ._lib import DDT_INFO_NONFINITE, DDTreeError

DDTREE_STAGE_ORDER = ("draft", "tree_build", "tree_compile", "verify", "commit")
DDTREE_TREE_BUILD_STAGE_ORDER = ("tree_build_copy", "tree_build_heap", "tree_build_visibility")


def empty_stage_times(stage_names):
    return {name: 0.0 for name in stage_names}


class ChildMaps(list):
    """``list[dict[int, int]]`` as the reference returns it (child_maps[p][tok]
    = child index), carrying the device-resident tree it was built from so
    that follow_verified_tree can walk on the GPU."""

    device_tree: kernels.DeviceTree | None = None


def _unpack_bits(words: np.ndarray, n: int) -> np.ndarray:
    w = words.view(np.uint32)[:n]
    cols = np.arange(n)
    return ((w[:, cols // 32] >> (cols % 32).astype(np.uint32)) & 1).astype(bool)


def build_ddtree_tree(draft_logits: torch.Tensor, budget: int):
    """Best-first draft tree from per-position draft logits [L, V].

    Returns ``(node_token_ids, node_depths, parents, child_maps, visibility,
    subtimes)`` exactly as ddtree.py:114-196: CPU int64 tensors, a parents
    list with parents[0] = -1, one dict per row, a bool [1+n, 1+n] CPU
    visibility matrix and the three sub-stage timings (the fused kernel has
    no separate heap / visibility stages; its whole time is reported under
    ``tree_build_copy``)."""
    subtimes = empty_stage_times(DDTREE_TREE_BUILD_STAGE_ORDER)
    if budget <= 0 or draft_logits.shape[0] == 0:
        vis = torch.zeros((1, 1), dtype=torch.bool)
        vis[0, 0] = True
        return (torch.empty(0, dtype=torch.long), torch.empty(0, dtype=torch.long), [-1], ChildMaps([dict()]), vis,
                subtimes)
    t0 = time.perf_counter()
    tree = kernels.tree_build(draft_logits, budget)
    info = tree.info.cpu()
    n = int(info[0])
    toks = tree.node_token_ids[:n].cpu()
    depths = tree.node_depths[:n].cpu()
    parents_np = tree.parents[: n + 1].cpu().numpy()
    words = tree.visibility[: n + 1].cpu().numpy()
    subtimes["tree_build_copy"] = time.perf_counter() - t0
    if int(info[2]) & DDT_INFO_NONFINITE:
        raise DDTreeError("build_ddtree_tree: non-finite draft log-probabilities")
    parents = parents_np.astype(np.int64).tolist()
    parents[0] = -1
    child_maps = ChildMaps(dict() for _ in range(n + 1))
    tl = toks.tolist()
    for i in range(1, n + 1):
        child_maps[parents[i]][tl[i - 1]] = i
    child_maps.device_tree = tree
    visibility = torch.from_numpy(_unpack_bits(words, n + 1))
    return toks, depths, parents, child_maps, visibility, subtimes


def compile_ddtree_tree(root_token_id, start: int, node_token_ids: torch.Tensor, node_depths: torch.Tensor,
                        visibility_cpu: torch.Tensor, past_length: int, dtype: torch.dtype, device: torch.device,
                        verify_input_ids_buffer: torch.Tensor, verify_position_ids_buffer: torch.Tensor,
                        attention_mask_buffer: torch.Tensor, tree_visibility_buffer: torch.Tensor,
                        previous_tree_start: int, previous_tree_length: int, sliding_window: int | None = None,
                        sliding_attention_mask_buffer: torch.Tensor | None = None):
    """Fill the verify buffers for one tree (ddtree.py:199-287).

    Returns ``(verify_input_ids, verify_position_ids, attention_mask,
    past_length, current_length)``; ``attention_mask`` is the [1, 1, N,
    past+N] view of ``attention_mask_buffer`` (or the per-layer-type dict when
    a sliding window is given).  The mask rows are written by the mask-fill
    kernel from the packed ancestor bits, which are also attached to the
    returned mask as ``ddtree_bits`` for the tree attention kernel."""
    current_length = 1 + int(node_token_ids.numel())
    ids = verify_input_ids_buffer[:, :current_length]
    ids[0, 0] = root_token_id
    if current_length > 1:
        ids[0, 1:current_length].copy_(node_token_ids, non_blocking=False)
    pos = verify_position_ids_buffer[:, :current_length]
    pos[0, 0] = start
    if current_length > 1:
        pos[0, 1:current_length].copy_(node_depths, non_blocking=False)
        pos[0, 1:current_length].add_(start)
    vis = tree_visibility_buffer[:current_length, :current_length]
    vis.copy_(visibility_cpu, non_blocking=False)
    bits = kernels.mask_to_bits(vis, 0, current_length)
    mask2d = attention_mask_buffer[0, 0]
    kernels.tree_mask_fill(mask2d, past_length, current_length, bits, previous_tree_start,
                           previous_tree_length if previous_tree_length > 0 else 0)
    full = attention_mask_buffer[:, :, :current_length, : past_length + current_length]
    _attach_bits(full, bits, past_length)
    if sliding_window is None or sliding_attention_mask_buffer is None:
        return ids, pos, full, past_length, current_length
    # hybrid sliding-window layers (ddtree.py:258-287): same tree block, past
    # keys outside the window of each query row masked
    smask = sliding_attention_mask_buffer[0, 0]
    kernels.tree_mask_fill(smask, past_length, current_length, bits, 0, 0)
    past_block = sliding_attention_mask_buffer[0, 0, :current_length, :past_length]
    past_block.zero_()
    lower = sliding_key_lo(pos[0], sliding_window)
    if past_length > 0:
        idx = torch.arange(past_length, device=past_block.device)
        past_block.masked_fill_(idx.unsqueeze(0) < lower.unsqueeze(1), torch.finfo(dtype).min)
    sliding = sliding_attention_mask_buffer[:, :, :current_length, : past_length + current_length]
    _attach_bits(sliding, bits, past_length)
    try:
        sliding.ddtree_key_lo = lower
    except (AttributeError, RuntimeError):
        pass
    return ids, pos, {"full_attention": full, "sliding_attention": sliding}, past_length, current_length


def sliding_key_lo(position_ids: torch.Tensor, sliding_window: int) -> torch.Tensor:
    """First visible prefix key of each verify row of a sliding-window layer:
    query position - window + 1, the lower bound of the reference's
    ``sliding_attention`` mask (ddtree.py:276-283).  int64, on the device of
    ``position_ids``; pass it as ``key_lo`` to ``kernels.tree_attention``."""
    return position_ids.reshape(-1).to(torch.int64) - (int(sliding_window) - 1)


def _attach_bits(mask: torch.Tensor, bits: torch.Tensor, past_length: int) -> None:
    try:
        mask.ddtree_bits = bits
        mask.ddtree_past = int(past_length)
    except (AttributeError, RuntimeError):
        pass


def follow_verified_tree(child_maps, posterior: torch.Tensor):
    """Walk from the root while the target's token is a child of the current
    node (ddtree.py:290-301).  Returns (accepted_indices, next_token).

    With a device posterior and child maps from build_ddtree_tree the walk
    runs on the GPU (ddt_tree_walk); otherwise the child maps are uploaded
    as a parent/token table first."""
    tree = getattr(child_maps, "device_tree", None)
    if not isinstance(posterior, torch.Tensor) or not posterior.is_cuda:
        raise ValueError("posterior must be a CUDA tensor on the B200 path")
    n = len(child_maps) - 1
    if tree is None:
        parents = np.full(n + 1, -1, np.int32)
        toks = np.zeros(max(n, 1), np.int64)
        for p, m in enumerate(child_maps):
            for tok, c in m.items():
                parents[c] = p
                toks[c - 1] = tok
        par_t = torch.from_numpy(parents).to(posterior.device)
        tok_t = torch.from_numpy(toks).to(posterior.device)
        n_dev = None
    else:
        par_t, tok_t, n_dev = tree.parents, tree.node_token_ids, tree.info
    post = posterior[0] if posterior.dim() == 2 else posterior
    accepted, info = kernels.tree_walk(post[: n + 1], par_t, tok_t, n_dev, max_accept=n + 1)
    info_h = info.cpu()
    count = int(info_h[0])
    return accepted[:count].cpu().tolist(), int(info_h[1])


def accept_verified_tree(logits: torch.Tensor, tree: kernels.DeviceTree, max_accept: int | None = None):
    """Fused greedy acceptance on the device: argmax of every verify row and
    the walk, one launch (sample + follow_verified_tree, temperature 0).

    Returns device tensors (accepted [max_accept], accept_info [2] =
    {count, next_token}, posterior [N]); nothing is copied to the host."""
    return kernels.tree_accept(logits, tree.parents, tree.node_token_ids, tree.info, max_accept=max_accept)


def commit_verified_tree(verify_input_ids: torch.Tensor, accepted: torch.Tensor, accept_info: torch.Tensor,
                         output_ids: torch.Tensor, start: int, hidden: torch.Tensor | None = None):
    """The commit step of a round (ddtree.py:534-548) on the device, after
    accept_verified_tree: the accepted verify tokens go to
    ``output_ids[:, start:start+n]`` and the bonus token to ``start+n``; with
    ``hidden`` ([1, N, H] verify hidden features) the accepted rows are
    returned as [max_accept, H] (the first n are valid).  n stays on the
    device (``accept_info[0]``), so no host sync happens here."""
    return kernels.tree_commit(verify_input_ids, accepted, accept_info, output_ids, start, hidden)


# ----------------------------------------------------------------------------
# KV compaction
# ----------------------------------------------------------------------------
_CPP_COMPACT_ENABLED = True


def maybe_enable_cpp_compact(enabled: bool) -> None:
    """Kept for call compatibility with ddtree.py:107-111; compaction is
    always the native kernel here."""
    global _CPP_COMPACT_ENABLED
    _CPP_COMPACT_ENABLED = bool(enabled)


def load_cpp_compact_module():
    """The reference returns its inline C++ module (ddtree.py:52-104); this
    returns an object with the same ``compact_tail_inplace`` entry point."""
    return SimpleNamespace(compact_tail_inplace=compact_tail_inplace)


def _keep_buffer(keep_current_indices, device: torch.device) -> torch.Tensor:
    """[count, keep...] int64 on the device in one host-to-device copy."""
    host = torch.empty(1 + len(keep_current_indices), dtype=torch.int64, pin_memory=True)
    host[0] = len(keep_current_indices)
    if len(keep_current_indices):
        host[1:] = torch.as_tensor(keep_current_indices, dtype=torch.int64)
    return host.to(device, non_blocking=True)


def compact_tail_inplace(cache_tensor: torch.Tensor, past_length: int, keep_current_indices: torch.Tensor):
    """In-place ``tail.index_select(seq, keep)`` -> ``[past, past+keep)``
    (ddtree.py:61-88), with the same argument checks raising RuntimeError."""
    if cache_tensor.dim() < 2:
        raise RuntimeError("cache_tensor must have rank >= 2")
    if keep_current_indices.dim() != 1:
        raise RuntimeError("keep_current_indices must be a 1D tensor")
    if keep_current_indices.dtype != torch.long:
        raise RuntimeError("keep_current_indices must have dtype torch.long")
    if cache_tensor.device != keep_current_indices.device:
        raise RuntimeError("cache_tensor and keep_current_indices must be on the same device")
    if past_length < 0:
        raise RuntimeError("past_length must be non-negative")
    seq = cache_tensor.shape[-2]
    if past_length > seq:
        raise RuntimeError("past_length exceeds cache sequence length")
    current_length = seq - past_length
    if current_length <= 0:
        return cache_tensor
    keep_count = keep_current_indices.numel()
    if keep_count > current_length:
        raise RuntimeError("keep_count exceeds appended window length")
    if keep_count == 0 or keep_count == current_length:
        return cache_tensor
    if not cache_tensor.is_cuda:
        raise RuntimeError("compact_tail_inplace: cache_tensor must be a CUDA tensor on the B200 path")
    count = torch.full((1,), keep_count, dtype=torch.int64, device=cache_tensor.device)
    kernels.kv_compact([cache_tensor], past_length, current_length, keep_current_indices.contiguous(), count,
                       keep_count, table=kernels.PointerTable())
    return cache_tensor


def _cache_tensors(past_key_values):
    """Initialised, de-aliased K/V tensors of a DynamicCache (ddtree.py:335-367)."""
    seen = set()
    out = []

    def add(t):
        if t is None or not isinstance(t, torch.Tensor) or t.numel() == 0:
            return
        if id(t) in seen:
            return
        seen.add(id(t))
        out.append(t)

    if hasattr(past_key_values, "layers"):
        for layer in past_key_values.layers:
            if hasattr(layer, "is_initialized") and not layer.is_initialized:
                continue
            add(getattr(layer, "keys", None))
            add(getattr(layer, "values", None))
        return out, True
    if hasattr(past_key_values, "key_cache") and hasattr(past_key_values, "value_cache"):
        for i in range(len(past_key_values.key_cache)):
            add(past_key_values.key_cache[i])
            add(past_key_values.value_cache[i])
        return out, True
    return out, False


_TABLES: dict = {}


def compact_dynamic_cache(past_key_values, past_length: int, keep_current_indices) -> None:
    """Keep only the accepted rows of the appended window in every layer of a
    DynamicCache and crop it (ddtree.py:323-369).  All layers sharing a
    layout are compacted by one kernel launch."""
    keep = list(keep_current_indices)
    if len(keep) == 0:
        past_key_values.crop(past_length)
        return
    tensors, ok = _cache_tensors(past_key_values)
    if not ok:
        raise RuntimeError("Unsupported DynamicCache layout for DDTree cache compaction.")
    groups: dict = {}
    for t in tensors:
        groups.setdefault((t.device, t.dtype, tuple(t.shape), t.stride()), []).append(t)
    for (device, _, shape, _), group in groups.items():
        cur = shape[-2] - past_length
        if cur <= 0 or len(keep) == cur:
            continue
        if not group[0].is_cuda:
            raise RuntimeError("compact_dynamic_cache: cache tensors must be on a CUDA device")
        buf = _keep_buffer(keep, device)
        table = _TABLES.setdefault((device, shape, len(group)), kernels.PointerTable())
        kernels.kv_compact(group, past_length, cur, buf[1:], buf[:1], len(keep), table=table)
    past_key_values.crop(past_length + len(keep))
