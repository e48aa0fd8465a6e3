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

import os
import time
from types import SimpleNamespace

import numpy as np
import torch

from . import kernels
from ._lib import DDT_INFO_NONFINITE, DDTreeError
from .fused_layers import _wgemm_on, head_logits

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


# ----------------------------------------------------------------------------
# The decode loop
# ----------------------------------------------------------------------------
def detect_hybrid_attention(target):
    """``(layer_types, sliding_window)`` when the target interleaves
    sliding-window and full attention layers (Gemma 3/4), else ``(None,
    None)`` (ddtree.py:27-49).  The text tower's config is used when the
    model has one."""
    cfg = getattr(target, "config", None)
    if cfg is None:
        return None, None
    text_cfg = getattr(cfg, "text_config", None) or cfg
    layer_types = getattr(text_cfg, "layer_types", None)
    window = getattr(text_cfg, "sliding_window", None)
    if not layer_types or window is None or int(window) <= 0:
        return None, None
    if "sliding_attention" not in layer_types or "full_attention" not in layer_types:
        return None, None
    return list(layer_types), int(window)


def tree_node_count(budget: int, rows: int, vocab: int) -> int:
    """Nodes of the best-first tree, known before it is built.

    The expansion pops until the budget is met or the heap is empty, and
    the heap empties only after every node of the complete top-k tree of
    depth ``rows`` has been popped: each pop pushes its next sibling and its
    first child (ddtree.py:157-177).  So n = min(budget, sum_{d=1..rows}
    topk^d), topk = min(budget, vocab), and the verify batch size needs no
    read-back of the tree."""
    if budget <= 0 or rows <= 0:
        return 0
    k = min(budget, vocab)
    total, level = 0, 1
    for _ in range(rows):
        level *= k
        total += level
        if total >= budget:
            return budget
    return total


@torch.inference_mode()
def ddtree_generate(model, target, input_ids: torch.Tensor, mask_token_id: int, max_new_tokens: int,
                    block_size: int, stop_token_ids, temperature: float = 0.0, tree_budget: int | None = None,
                    save_tree_traces: bool = False) -> SimpleNamespace:
    """DDTree speculative decoding (ddtree.py:372-587), same arguments and
    same ``SimpleNamespace`` result.

    Each round: the draft predicts ``block_size - 1`` positions; the tree
    kernel builds the best-first tree, its verify ids and positions and the
    packed ancestor bits on the device; the target verifies every node in
    one forward through the tree-attention kernel (the attention layers are
    routed to it for the call); the accept kernel takes the argmax of every
    verify row (or a temperature draw) and walks the tree; the commit kernel
    writes the accepted and bonus tokens into ``output_ids`` and gathers the
    accepted rows of the target's context features; one launch compacts
    every layer's K and V.  The accepted count stays on the device until the
    round's single host read, which also returns the new tokens for the stop
    check.

    From the third round on, the draft forward and the verify forward are
    replayed from CUDA graphs captured once per call: both caches append at
    a device-side row offset and the attention reads the prefix length from
    the device, so one capture serves every round (set DDTREE_EAGER=1 to run
    every round eagerly).  The graphs need this package's DFlashDraftModel
    (other draft classes run eagerly), a target without sliding-window
    layers, and a node budget of at least ``block_size - 1``.

    Stage times come from CUDA events (``stage_times`` has the reference's
    keys; the fused tree kernel's time is booked to ``tree_build``, its three
    sub-stages read 0, and ``tree_compile`` is the host time to describe the
    tree mask).
    """
    if block_size <= 1:
        return _target_only_generate(model, target, input_ids, mask_token_id, max_new_tokens, block_size,
                                     stop_token_ids, temperature)
    import os
    from contextlib import nullcontext
    from .fused_layers import fused_decoder_layers
    from .runtime import tree_attention_for
    fuse = os.environ.get("DDTREE_FUSED", "1") != "0"
    with tree_attention_for(target), (fused_decoder_layers(target) if fuse else nullcontext()), \
            kernels.pdl(fuse and os.environ.get("DDTREE_PDL", "1") != "0"):
        budget = block_size - 1 if tree_budget is None else max(int(tree_budget), 0)
        needed = input_ids.shape[1] + max_new_tokens + (1 + budget) + 1
        dec = _decoder_session(model, target, block_size, tree_budget, needed)
        dec.start_call(input_ids, mask_token_id, max_new_tokens, stop_token_ids, temperature, save_tree_traces)
        return dec.run()


def _weights_fingerprint(*modules) -> tuple:
    """Addresses and versions of every parameter: a captured forward reads
    the weights by address, so a session is reused only while they hold."""
    return tuple((p.data_ptr(), p._version) for m in modules for p in m.parameters())


def _decoder_session(model, target, block_size, tree_budget, needed_rows: int):
    """The decode session of (draft, target, block size, budget): buffers of
    at least ``needed_rows`` cache rows and, once captured, the draft and
    verify graphs.  Kept on the target (outside its state dict) and reused
    by later calls while the weights and settings match, so a call pays no
    capture; ``release_decode_sessions(target)`` frees it."""
    import os
    eager = os.environ.get("DDTREE_EAGER", "0") == "1"
    # every DDTREE_* switch (fused layers, packing, GEMM choice, PDL) shapes the captured graphs
    switches = tuple(sorted((k, v) for k, v in os.environ.items() if k.startswith("DDTREE_")))
    key = (id(model), block_size, tree_budget, eager, switches)
    fp = _weights_fingerprint(model, target)
    held = target.__dict__.get("_ddtree_session")
    if held is not None:
        k, sess = held
        if k == key and sess.capacity >= needed_rows and sess.fingerprint == fp and sess.model is model:
            sess.target = target   # held for the call only (the session lives on the target)
            return sess
        target.__dict__.pop("_ddtree_session", None)
        del sess, held
    capacity = -(-needed_rows // 1024) * 1024
    sess = _DDTreeDecoder(model, target, block_size, tree_budget, capacity, eager)
    sess.fingerprint = fp
    target.__dict__["_ddtree_session"] = (key, sess)
    return sess


def release_decode_sessions(target) -> None:
    """Free the buffers and graphs that ddtree_generate keeps on ``target``."""
    target.__dict__.pop("_ddtree_session", None)


class _DDTreeDecoder:
    """A decode session: buffers, caches and captured forwards, reused by
    the ddtree_generate calls of one (draft, target) pair; ``start_call``
    sets the per-call state."""

    def __init__(self, model, target, block_size, tree_budget, capacity: int, eager: bool):
        from .cache import TreeAppendCache
        from .model import DFlashDraftModel
        from .runtime import Readback, TreeMask
        self.model, self.target = model, target
        self.device = device = model.device
        self.capacity = capacity
        self.block = block_size
        self.L = block_size - 1
        self.budget = self.L if tree_budget is None else max(int(tree_budget), 0)
        self.max_nodes = 1 + self.budget
        self.vocab = target.lm_head.weight.shape[0] if hasattr(target, "lm_head") else target.config.vocab_size
        self.layer_types, self.window = detect_hybrid_attention(target)
        self.output_ids = torch.zeros((1, capacity), dtype=torch.long, device=device)
        self.position_ids = torch.arange(capacity, device=device).unsqueeze(0)
        self.target_cache = TreeAppendCache(capacity, config=target.config)
        self.draft_cache = TreeAppendCache(capacity + block_size, config=model.config)
        self.tree = kernels.DeviceTree.allocate(self.L, self.vocab, self.budget, device)
        self.accepted = torch.zeros((self.max_nodes,), dtype=torch.int64, device=device)
        self.accept_info = torch.zeros((2,), dtype=torch.int64, device=device)
        self.posterior = torch.empty((self.max_nodes,), dtype=torch.int64, device=device)
        self.tree_mask = TreeMask(target.dtype, device)
        self.readback = Readback(4 + 6 * self.max_nodes, device)
        self.tables: dict = {}
        self.hidden_buf = None
        self.att_ws = None
        # static (device-length) mode: round state [start, ctx_offset, ctx_count, 0]
        self.rs_host = torch.zeros((4,), dtype=torch.int32, pin_memory=True)
        self.rs = torch.zeros((4,), dtype=torch.int32, device=device)
        self.static = (isinstance(model, DFlashDraftModel) and self.window is None
                       and self.budget >= self.L and not eager)
        # DDTREE_HEAD_TOPK=1: the draft head fused with the tree build's first
        # step: the head's GEMM leaves per-block statistics that the tree
        # build reads instead of scanning the logits (bf16 head without bias
        # or soft-capping).  Off by default: on B200 at Qwen3-4B the head's
        # epilogue costs 7.4 us and the tree build saves 2.6 us per round.
        head = getattr(target, "lm_head", None)
        self.head_stats = None
        if (self.static and os.environ.get("DDTREE_HEAD_TOPK", "0") == "1" and _wgemm_on("head")
                and isinstance(head, torch.nn.Linear) and head.bias is None
                and head.weight.dtype == torch.bfloat16 and self.vocab % 128 == 0
                and head.weight.shape[1] % 64 == 0 and 0 < self.budget <= 80
                and getattr(model, "final_logit_softcapping", None) is None):
            self.head_stats = kernels.head_stats_buffer(self.L, self.vocab, device)
        self.graphs = None
        self.graph_kernels = (0, 0)
        self.n_nodes = tree_node_count(self.budget, self.L, self.vocab)
        self.N = 1 + self.n_nodes

    def start_call(self, input_ids, mask_token_id, max_new_tokens, stop_token_ids, temperature,
                   save_tree_traces) -> None:
        from .runtime import EventClock, device_sample_seed
        self.P = input_ids.shape[1]
        self.input_ids = input_ids
        self.max_length = self.P + max_new_tokens
        # the reference's buffer length, which bounds a draft block near the end
        self.out_len = self.max_length + self.max_nodes
        self.mask_token_id = mask_token_id
        self.temperature = temperature
        self.traces = save_tree_traces
        self.stop_ids = None if stop_token_ids is None else set(int(t) for t in stop_token_ids)
        self.seed = device_sample_seed() if temperature >= 1e-5 else 0
        self.clock = EventClock(self.device)
        self.replays = 0
        self.capture_s = 0.0
        self.output_ids.fill_(mask_token_id)
        for cache in (self.target_cache, self.draft_cache):
            cache.set_static(None)
            for layer in cache.layers:
                layer.reset()

    # ------------------------------------------------------------------ setup
    def _setup_static(self, features: torch.Tensor) -> None:
        """After the prefill: both caches switch to device-offset appends; on
        the session's first call the attention workspace (sized for the
        longest prefix) and the static buffers are allocated."""
        self.target_cache.set_static(self.rs[0:1])
        self.draft_cache.set_static(self.rs[0:1])
        if self.att_ws is not None:
            return
        t, d = self.target.config, self.model.config
        hq_t, hkv_t = t.num_attention_heads, t.num_key_value_heads
        hq_d, hkv_d = d.num_attention_heads, d.num_key_value_heads
        self.past_max_t = self.target_cache.capacity - self.N
        self.past_max_d = self.draft_cache.capacity - self.block
        ws_t = kernels.attention_workspace(self.N, hq_t, hkv_t, self.past_max_t, self.device)
        ws_d = kernels.attention_workspace(self.block, hq_d, hkv_d, self.past_max_d, self.device)
        self.att_ws = ws_t if ws_t.numel() >= ws_d.numel() else ws_d
        self.ar_block = torch.arange(self.block, device=self.device)
        self.block_buf = torch.empty((1, self.block), dtype=torch.long, device=self.device)
        self.static_mask = self.tree_mask.static(self.tree.visibility[: self.N], self.rs[0:1], self.past_max_t,
                                                 self.N, self.att_ws)

    def _set_round_state(self, start: int, ctx_offset: int, ctx_count: int) -> None:
        self.rs_host[0], self.rs_host[1], self.rs_host[2] = start, ctx_offset, ctx_count
        self.rs.copy_(self.rs_host, non_blocking=True)

    # ------------------------------------------------------------------ stages
    def _draft_generic(self, start: int, target_hidden: torch.Tensor) -> torch.Tensor:
        from .model import apply_final_logit_softcapping
        block = self.output_ids[:, start: min(start + self.block, self.out_len)]
        noise = self.target.model.embed_tokens(block)
        h = self.model(target_hidden=target_hidden, noise_embedding=noise,
                       position_ids=self.position_ids[:, self.draft_cache.get_seq_length():
                                                      min(start + self.block, self.out_len)],
                       past_key_values=self.draft_cache, use_cache=True, is_causal=False)
        logits = self.target.lm_head(h[:, -self.L:, :])
        logits = apply_final_logit_softcapping(logits, self.model.final_logit_softcapping)
        self.draft_cache.crop(start)
        return logits

    def _draft_static(self, ctx_hidden: torch.Tensor) -> torch.Tensor:
        """Draft logits with every length read from ``self.rs`` (capturable)."""
        from .model import apply_final_logit_softcapping
        C = ctx_hidden.shape[1]
        start = self.rs[0:1].long()
        self.block_buf.copy_(self.output_ids[:, start + self.ar_block])
        noise = self.target.model.embed_tokens(self.block_buf)
        ar_c = self.ar_block if C == self.block else torch.arange(C, device=self.device)
        pos = torch.cat([self.rs[1:2].long() + ar_c, start + self.ar_block]).unsqueeze(0)
        h = self.model.forward_static(noise, ctx_hidden, pos, self.draft_cache, self.rs, self.past_max_d, self.att_ws)
        if self.head_stats is not None:
            return kernels.wgemm_head(h[0, -self.L:, :], self.target.lm_head.weight, self.head_stats).unsqueeze(0)
        logits = head_logits(self.target.lm_head, h[:, -self.L:, :])
        return apply_final_logit_softcapping(logits, self.model.final_logit_softcapping)

    def _verify(self, start: int, mask):
        from .model import extract_context_feature
        out = self.target(self.tree.verify_ids[: self.N].unsqueeze(0),
                          position_ids=self.tree.verify_pos[: self.N].unsqueeze(0), attention_mask=mask,
                          past_key_values=self.target_cache, use_cache=True, output_hidden_states=True)
        return out.logits, extract_context_feature(out.hidden_states, self.model.target_layer_ids)

    def _capture(self, ctx_hidden: torch.Tensor) -> None:
        """Capture the draft and verify forwards (after an eager round of the
        same shapes has warmed every path)."""
        from ._lib import load
        lib = load()
        t0 = time.perf_counter()
        pool = torch.cuda.graph_pool_handle()
        gd, gv = torch.cuda.CUDAGraph(), torch.cuda.CUDAGraph()
        n0 = lib.ddt_launch_count()
        with torch.cuda.graph(gd, pool=pool):
            draft_logits = self._draft_static(ctx_hidden)
        n1 = lib.ddt_launch_count()
        with torch.cuda.graph(gv, pool=pool):
            logits, features = self._verify(0, self.static_mask)
        n2 = lib.ddt_launch_count()
        # this library's kernels inside each graph (counted once, at capture)
        self.graph_kernels = (n1 - n0, n2 - n1)
        self.graphs = (gd, gv, draft_logits, logits, features)
        self.capture_s = time.perf_counter() - t0

    # ------------------------------------------------------------------ loop
    def run(self) -> SimpleNamespace:
        from ._lib import load
        from .model import extract_context_feature
        dev, clock = self.device, self.clock
        launches0 = load().ddt_launch_count()
        stage_times = empty_stage_times(DDTREE_STAGE_ORDER + DDTREE_TREE_BUILD_STAGE_ORDER)
        P = self.P
        ev_prefill = clock.mark()
        output = self.target(self.input_ids, position_ids=self.position_ids[:, :P], past_key_values=self.target_cache,
                             use_cache=True, logits_to_keep=1, output_hidden_states=True)
        self.output_ids[:, :P] = self.input_ids
        self.output_ids[:, P: P + 1] = kernels.sample(output.logits, self.temperature)
        target_hidden = extract_context_feature(output.hidden_states, self.model.target_layer_ids)
        F = target_hidden.shape[-1]
        if self.hidden_buf is None or self.hidden_buf.shape[-1] != F or self.hidden_buf.dtype != target_hidden.dtype:
            self.hidden_buf = torch.zeros((self.max_nodes, F), dtype=target_hidden.dtype, device=dev)
            self.graphs = None   # a captured draft reads this buffer
        if self.static:
            self._setup_static(target_hidden)
        ev_first = clock.mark()

        ev_decode = clock.mark()
        ev_round_clock = ev_decode
        start, count, rnd = P, P, 0
        acceptance, round_ends = [], []
        round_trees = [] if self.traces else None
        N, n_nodes = self.N, self.n_nodes
        while start < self.max_length:
            ev0 = clock.mark()
            if self.static:
                self._set_round_state(start, start - count, count)
                if rnd == 0:
                    draft_logits = self._draft_static(target_hidden)
                elif self.graphs is None:
                    draft_logits = self._draft_static(self.hidden_buf[None, : self.block])
                else:
                    self.graphs[0].replay()
                    self.replays += 1
                    draft_logits = self.graphs[2]
            else:
                draft_logits = self._draft_generic(start, target_hidden)
            ev1 = clock.mark()
            if rnd == 0:
                ev_decode = ev1
            else:
                clock.span("draft", ev0, ev1)

            root = self.block_buf[0, 0:1] if self.static else self.output_ids[0, start: start + 1]
            kernels.tree_build(draft_logits[0], self.budget, root_token=root, start=start, out=self.tree,
                               head_stats=self.head_stats if self.static else None)
            ev2 = clock.mark()
            clock.span("tree_build", ev1, ev2)

            bits = self.tree.visibility[:N]
            if self.static:
                mask = self.static_mask
            else:
                mask = self.tree_mask(bits, start, N)
                if self.window is not None:
                    key_lo = sliding_key_lo(self.tree.verify_pos[:N], self.window)
                    mask = {"full_attention": mask, "sliding_attention": self.tree_mask(bits, start, N, key_lo)}
            ev3 = clock.mark()
            clock.span("tree_compile", ev2, ev3)

            if self.graphs is not None:
                self.graphs[1].replay()
                logits, features = self.graphs[3], self.graphs[4]
            else:
                logits, features = self._verify(start, mask)
            ev4 = clock.mark()
            clock.span("verify", ev3, ev4)

            count = self._accept_commit(logits[0], features[0], start, rnd)
            got = self._fetch(start, count)
            count, new_tokens = int(got[0][0]), got[1][: int(got[0][0]) + 1]
            if not self.static:
                self.target_cache.crop(start + count)
            target_hidden = self.hidden_buf[None, :count]
            acceptance.append(count)
            ev5 = clock.mark()
            clock.span("commit", ev4, ev5)
            round_ends.append(ev5)
            if self.traces:
                parents = [int(p) for p in got[5]]
                parents[0] = -1
                round_trees.append({
                    "accepted_indices": [int(i) for i in got[2][:count]],
                    "tree": {"node_token_ids": [int(t) for t in got[3]], "node_depths": [int(d) for d in got[4]],
                             "parents": parents}})
            start += count
            rnd += 1
            if self.static and rnd == 2 and self.graphs is None and start < self.max_length:
                self._capture(self.hidden_buf[None, : self.block])
            if self.stop_ids is not None and any(t in self.stop_ids for t in new_tokens):
                break
        ev_end = clock.mark()

        output_ids = self.output_ids[:, : self.max_length]
        output_ids = output_ids[:, output_ids[0] != self.mask_token_id]
        if self.stop_ids is not None:
            for i, t in enumerate(output_ids[0, P:].tolist()):
                if t in self.stop_ids:
                    output_ids = output_ids[:, : P + i + 1]
                    break
        num_output_tokens = output_ids.shape[1] - P
        clock.resolve(stage_times)
        total_decode_time = clock.seconds(ev_decode, ev_end)
        # kernels of this library run by the call: eager launches plus every
        # replay of the captured ones (launches counted at a capture never ran)
        native = load().ddt_launch_count() - launches0 + self.replays * sum(self.graph_kernels) - \
            (sum(self.graph_kernels) if self.capture_s > 0 else 0)
        try:
            return SimpleNamespace(
                output_ids=output_ids.cpu(),
                num_input_tokens=P,
                num_output_tokens=num_output_tokens,
                time_to_first_token=clock.seconds(ev_prefill, ev_first),
                time_per_output_token=total_decode_time / max(num_output_tokens, 1),
                acceptance_lengths=acceptance,
                decode_rounds=len(acceptance),
                stage_times=stage_times,
                round_timestamps=[clock.seconds(ev_round_clock, e) for e in round_ends],
                round_trees=round_trees,
                native_launches=int(native),
                graph_rounds=self.replays,
                graph_capture_s=self.capture_s,
            )
        finally:
            # the session lives on the target: drop the reference back to it
            self.target = None

    def _accept_commit(self, logits: torch.Tensor, features: torch.Tensor, start: int, rnd: int) -> None:
        from .runtime import compact_on_device
        N = self.N
        if self.temperature < 1e-5:
            kernels.tree_accept(logits, self.tree.parents, self.tree.node_token_ids, self.tree.info, max_accept=N,
                                accepted=self.accepted[:N], accept_info=self.accept_info, posterior=self.posterior[:N])
        else:
            post = kernels.sample_rows(logits, self.temperature, self.seed, rnd)
            acc_t, info_t = kernels.tree_walk(post, self.tree.parents, self.tree.node_token_ids, self.tree.info,
                                              max_accept=N)
            self.accepted[:N].copy_(acc_t)
            self.accept_info.copy_(info_t)
        kernels.tree_commit(self.tree.verify_ids[:N], self.accepted[:N], self.accept_info, self.output_ids[0], start,
                            hidden=features, hidden_out=self.hidden_buf[:N])
        compact_on_device(self.target_cache, start, N, self.accepted, self.accept_info[:1], N, self.tables)

    def _fetch(self, start: int, _count) -> list:
        N, n = self.N, self.n_nodes
        pieces = [(self.accept_info, 2), (self.output_ids[0, start:], N + 1)]
        if self.traces:
            pieces += [(self.accepted, N), (self.tree.node_token_ids, n), (self.tree.node_depths, n),
                       (self.tree.parents.to(torch.int64), N)]
        return self.readback.fetch(pieces)

DFLASH_STAGE_ORDER = ("draft", "verify", "commit")


def _target_only_generate(model, target, input_ids, mask_token_id, max_new_tokens, block_size, stop_token_ids,
                          temperature):
    """``ddtree_generate`` with ``block_size <= 1`` hands over to the
    reference's ``dflash_generate`` (ddtree.py:383-393), which then decodes
    one target token per round without a draft (dflash.py:18-143 with a
    one-token block).  That is what this does, with the same result fields."""
    if block_size < 1:
        raise ValueError("block_size must be at least 1")
    from .cache import TreeAppendCache
    from .runtime import EventClock, Readback, tree_attention_for

    device = model.device
    num_input_tokens = input_ids.shape[1]
    max_length = num_input_tokens + max_new_tokens
    output_ids = torch.full((1, max_length + block_size), mask_token_id, dtype=torch.long, device=device)
    position_ids = torch.arange(output_ids.shape[1], device=device).unsqueeze(0)
    stop_ids = None if stop_token_ids is None else set(int(t) for t in stop_token_ids)
    cache = TreeAppendCache(max_length + 2, config=target.config)
    stage_times = empty_stage_times(DFLASH_STAGE_ORDER)
    clock = EventClock(device)
    readback = Readback(4, device)
    with tree_attention_for(target):
        ev_prefill = clock.mark()
        out = target(input_ids, position_ids=position_ids[:, :num_input_tokens], past_key_values=cache,
                     use_cache=True, logits_to_keep=1)
        output_ids[:, :num_input_tokens] = input_ids
        output_ids[:, num_input_tokens: num_input_tokens + 1] = kernels.sample(out.logits, temperature)
        ev_first = clock.mark()
        ev_decode = clock.mark()
        start = num_input_tokens
        acceptance_lengths, round_ends = [], []
        while start < max_length:
            ev0 = clock.mark()
            out = target(output_ids[:, start: start + 1], position_ids=position_ids[:, start: start + 1],
                         past_key_values=cache, use_cache=True)
            ev1 = clock.mark()
            clock.span("verify", ev0, ev1)
            output_ids[:, start + 1] = kernels.sample(out.logits, temperature)[:, 0]
            got = readback.fetch([(output_ids[0, start:], 2)])
            acceptance_lengths.append(1)
            start += 1
            ev2 = clock.mark()
            clock.span("commit", ev1, ev2)
            round_ends.append(ev2)
            if stop_ids is not None and any(t in stop_ids for t in got[0]):
                break
        ev_end = clock.mark()
    output_ids = output_ids[:, :max_length]
    output_ids = output_ids[:, output_ids[0] != mask_token_id]
    if stop_ids is not None:
        for i, t in enumerate(output_ids[0, num_input_tokens:].tolist()):
            if t in stop_ids:
                output_ids = output_ids[:, : num_input_tokens + i + 1]
                break
    num_output_tokens = output_ids.shape[1] - num_input_tokens
    clock.resolve(stage_times)
    total = EventClock.seconds(ev_decode, ev_end)
    return SimpleNamespace(
        output_ids=output_ids.cpu(), num_input_tokens=num_input_tokens, num_output_tokens=num_output_tokens,
        time_to_first_token=EventClock.seconds(ev_prefill, ev_first),
        time_per_output_token=total / max(num_output_tokens, 1), acceptance_lengths=acceptance_lengths,
        decode_rounds=len(acceptance_lengths), stage_times=stage_times,
        round_timestamps=[EventClock.seconds(ev_decode, e) for e in round_ends])
