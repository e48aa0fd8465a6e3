"""The verify-attention boundary: an attention function with the HF
``AttentionInterface`` signature (the one ``sdpa_attention_forward`` has in
transformers/integrations/sdpa_attention.py) that runs the tcgen05
tree-attention kernel.

The reference verifies a tree by passing a 4-D additive mask to the target
(ddtree.py:523-531, eagle3.py:213-220); every attention layer then runs
SDPA with K/V repeated for GQA.  Here each layer calls
``ddt_tree_attention`` with the mask reduced once per forward to a packed
ancestor bitmask of its last ``q_len`` columns (the prefix before them must
be fully visible, as in the reference's masks).  Causal prefill / decode
calls (no mask) use the causal bitmask.

Sliding-window layers of hybrid models (the attention function gets
``sliding_window`` and the reference's ``sliding_attention`` mask,
ddtree.py:258-287) run ``ddt_tree_attention_window``: each row's first
visible prefix key comes from the mask (``ddtree_key_lo`` attached by
``ddtree.compile_ddtree_tree``, else counted from the mask's prefix
columns, which must hide a leading block of keys per row), or from the row's
position for causal calls.

Register with ``register()`` and load the target with
``attn_implementation="ddtree_b200"``.
"""
from __future__ import annotations

import torch

from . import kernels

ATTN_NAME = "ddtree_b200"

_bits_cache: dict = {}
_causal_cache: dict = {}


def causal_bits(n: int, device: torch.device, window: int | None = None) -> torch.Tensor:
    """Packed causal mask of n new rows; with a sliding window shorter than
    n, row t sees only rows t - window + 1 .. t of them."""
    if window is not None and window >= n:
        window = None
    key = (n, device, window)
    b = _causal_cache.get(key)
    if b is None:
        vis = torch.ones((n, n), dtype=torch.bool, device=device).tril_()
        if window is not None:
            vis &= ~torch.ones((n, n), dtype=torch.bool, device=device).tril_(-int(window))
        b = kernels.mask_to_bits(vis, 0, n)
        _causal_cache[key] = b
    return b


def _mask_bits(mask: torch.Tensor, q_len: int, kv_len: int):
    """Packed bits of the tree block and the prefix length for a dense mask."""
    bits = getattr(mask, "ddtree_bits", None)
    if bits is not None and bits.shape[0] == q_len and getattr(mask, "ddtree_past", None) == kv_len - q_len:
        return bits, kv_len - q_len
    key = (mask.data_ptr(), tuple(mask.shape), mask.stride(), mask._version, q_len, kv_len)
    hit = _bits_cache.get("last")
    if hit is not None and hit[0] == key:
        return hit[1], kv_len - q_len
    m2 = mask.reshape(-1, mask.shape[-2], mask.shape[-1])[0]
    if m2.shape[-1] < kv_len:
        raise ValueError("attention mask is narrower than the key length")
    past = kv_len - q_len
    bits = kernels.mask_to_bits(m2[:q_len], past, q_len)
    _bits_cache["last"] = (key, bits)
    return bits, past


def _mask_key_lo(mask: torch.Tensor, q_len: int, kv_len: int) -> torch.Tensor:
    """First visible prefix key of each row of a sliding-window mask."""
    past = kv_len - q_len
    lo = getattr(mask, "ddtree_key_lo", None)
    if lo is not None and lo.shape[0] == q_len and getattr(mask, "ddtree_past", None) == past:
        return lo
    key = (mask.data_ptr(), tuple(mask.shape), mask.stride(), mask._version, q_len, kv_len)
    hit = _bits_cache.get("last_key_lo")
    if hit is not None and hit[0] == key:
        return hit[1]
    m2 = mask.reshape(-1, mask.shape[-2], mask.shape[-1])[0][:q_len, :past]
    visible = m2 if m2.dtype == torch.bool else m2 > torch.finfo(m2.dtype).min / 2
    lo = (~visible).sum(dim=1, dtype=torch.int64)
    leading = torch.arange(past, device=m2.device).unsqueeze(0) >= lo.unsqueeze(1)
    if not torch.equal(visible, leading):
        raise ValueError("sliding-window mask: each row must hide a leading block of prefix keys")
    _bits_cache["last_key_lo"] = (key, lo)
    return lo


def tree_verify_attention(module, query: torch.Tensor, key: torch.Tensor, value: torch.Tensor,
                          attention_mask: torch.Tensor | None, dropout: float = 0.0, scaling: float | None = None,
                          is_causal: bool | None = None, **kwargs):
    """query [1, Hq, T, D], key / value [1, Hkv, S, D] -> ([1, T, Hq, D], None)."""
    if query.shape[0] != 1:
        raise NotImplementedError("the tree-verify attention runs batch 1 (as the reference does)")
    window = kwargs.get("sliding_window")
    if dropout and module.training:
        raise NotImplementedError("dropout is not supported")
    _, hq, T, d = query.shape
    S = key.shape[-2]
    scale = float(scaling) if scaling is not None else d ** -0.5
    past_dev = getattr(attention_mask, "ddtree_past_dev", None) if attention_mask is not None else None
    if past_dev is not None:
        # a captured verify forward: the cache returns its whole buffers and
        # the prefix length lives on the device (TreeMask.static)
        q = query[0].transpose(0, 1)
        out = torch.empty((1, T, hq, d), dtype=query.dtype, device=query.device)
        kernels.tree_attention(q, key[0], value[0], attention_mask.ddtree_past_max, attention_mask.ddtree_bits, scale,
                               out=out[0], key_lo=getattr(attention_mask, "ddtree_key_lo", None), past_dev=past_dev,
                               workspace=attention_mask.ddtree_workspace)
        return out, None
    if attention_mask is None:
        bits, past = causal_bits(T, query.device, window), S - T
    else:
        bits, past = _mask_bits(attention_mask, T, S)
    key_lo = None
    if window is not None:
        if attention_mask is None:   # causal: row t sits at position past + t
            key_lo = torch.arange(past - int(window) + 1, past - int(window) + 1 + T, dtype=torch.int64,
                                  device=query.device)
        else:
            key_lo = _mask_key_lo(attention_mask, T, S)
    q = query[0].transpose(0, 1)            # [T, Hq, D]
    out = torch.empty((1, T, hq, d), dtype=query.dtype, device=query.device)
    kernels.tree_attention(q, key[0], value[0], past, bits, scale, out=out[0], key_lo=key_lo)
    return out, None


def register() -> str:
    """Register the kernel under ``ATTN_NAME`` in the HF attention registry."""
    from transformers import AttentionInterface
    AttentionInterface.register(ATTN_NAME, tree_verify_attention)
    try:
        from transformers.masking_utils import ALL_MASK_ATTENTION_FUNCTIONS, sdpa_mask
        ALL_MASK_ATTENTION_FUNCTIONS.register(ATTN_NAME, sdpa_mask)
    except Exception:  # older transformers: the sdpa mask path is picked by name
        pass
    return ATTN_NAME
