"""A preallocated KV cache with an in-place append for the verify boundary.

``transformers``' ``DynamicCache`` appends each round's tree rows with
``torch.cat`` (its ``DynamicLayer.update``), which reallocates and copies a
layer's whole K and V every round.  ``TreeAppendCache`` keeps the same
``Cache`` interface but each layer owns one ``[batch, heads, capacity, dim]``
buffer per kind: ``update`` copies the new rows into place and returns views
of the filled length, and ``crop`` only shortens the views.  The views carry
the buffer's strides, so ``ddtree.compact_dynamic_cache`` compacts every layer
of the cache in one kernel launch exactly as it does for a ``DynamicCache``
(ddtree.py:323-369), and the tree attention kernel reads them in place.

Static mode (``set_static``) is for forwards captured once and replayed
every round: the append lands at a row offset read from a device int32
scalar (``ddt_kv_append``) and ``update`` returns views of the whole
buffer, so the addresses and shapes a captured forward sees never change;
the attention reads the prefix length from the same scalar.  Buffers are
zero-filled when allocated, so rows past the written ones always hold finite
values.

A buffer that would overflow in host mode grows to twice the needed length
(one copy); size ``capacity`` to the prompt plus the new tokens plus one
tree to avoid it.  Static mode never grows.
"""
from __future__ import annotations

import torch
from transformers.cache_utils import Cache, CacheLayerMixin

from . import kernels

__all__ = ["TreeAppendLayer", "TreeAppendCache"]


class TreeAppendLayer(CacheLayerMixin):
    """One layer's preallocated K/V buffers; ``keys`` / ``values`` are views
    of the first ``length`` rows (host mode) or of the whole buffer (static
    mode)."""

    is_sliding = False

    def __init__(self, capacity: int = 0):
        super().__init__()
        self.capacity = int(capacity)
        self._k = None
        self._v = None
        self.offset_dev = None     # static mode: int32 device row offset of the next append

    def lazy_initialization(self, key_states: torch.Tensor, value_states: torch.Tensor) -> None:
        self.dtype, self.device = key_states.dtype, key_states.device
        shape = list(key_states.shape)
        shape[-2] = max(self.capacity, key_states.shape[-2])
        self._k = torch.zeros(shape, dtype=key_states.dtype, device=key_states.device)
        self._v = torch.zeros(shape[:-1] + [value_states.shape[-1]], dtype=value_states.dtype,
                              device=value_states.device)
        self.keys = self._k[..., :0, :]
        self.values = self._v[..., :0, :]
        self.is_initialized = True

    def _grow(self, needed: int) -> None:
        n = self.keys.shape[-2]
        new_cap = max(needed, 2 * self._k.shape[-2])
        k = torch.zeros(list(self._k.shape[:-2]) + [new_cap, self._k.shape[-1]], dtype=self._k.dtype,
                        device=self._k.device)
        v = torch.zeros(list(self._v.shape[:-2]) + [new_cap, self._v.shape[-1]], dtype=self._v.dtype,
                        device=self._v.device)
        k[..., :n, :].copy_(self.keys)
        v[..., :n, :].copy_(self.values)
        self._k, self._v = k, v

    def update(self, key_states: torch.Tensor, value_states: torch.Tensor, *args, **kwargs):
        """Append the new rows in place; returns the filled K and V views
        (the whole buffers in static mode)."""
        if not self.is_initialized:
            self.lazy_initialization(key_states, value_states)
        if self.offset_dev is not None:
            return self.update_at(key_states, value_states, self.offset_dev)
        n0 = self.keys.shape[-2]
        n1 = n0 + key_states.shape[-2]
        if n1 > self._k.shape[-2]:
            self._grow(n1)
        self._k[..., n0:n1, :].copy_(key_states)
        self._v[..., n0:n1, :].copy_(value_states)
        self.keys = self._k[..., :n1, :]
        self.values = self._v[..., :n1, :]
        return self.keys, self.values

    def update_at(self, key_states: torch.Tensor, value_states: torch.Tensor, offset_dev: torch.Tensor,
                  rows_dev: torch.Tensor | None = None):
        """Static-mode append: rows [0, rows) of the new K/V (fewer when
        ``rows_dev`` holds a smaller count) at row ``offset_dev`` of the
        buffers, both read on the device.  Returns the whole buffers."""
        if not self.is_initialized:
            self.lazy_initialization(key_states, value_states)
        kernels.kv_append(key_states, value_states, self._k, self._v, offset_dev, rows_dev)
        self.keys, self.values = self._k, self._v
        return self._k, self._v

    def get_mask_sizes(self, query_length: int) -> tuple[int, int]:
        return self.get_seq_length() + query_length, 0

    def get_seq_length(self) -> int:
        if not self.is_initialized:
            return 0
        return self.keys.shape[-2]

    def get_max_cache_shape(self) -> int:
        return -1

    def crop(self, max_length: int) -> None:
        if not self.is_initialized or self.offset_dev is not None:
            return
        if max_length < 0:
            max_length = self.get_seq_length() - abs(max_length)
        if self.get_seq_length() <= max_length:
            return
        self.keys = self._k[..., :max_length, :]
        self.values = self._v[..., :max_length, :]

    def reset(self) -> None:
        if self.is_initialized:
            self.keys = self._k[..., :0, :]
            self.values = self._v[..., :0, :]

    def batch_repeat_interleave(self, repeats: int) -> None:
        if self.get_seq_length() > 0:
            n = self.keys.shape[-2]
            self._k = self._k.repeat_interleave(repeats, dim=0)
            self._v = self._v.repeat_interleave(repeats, dim=0)
            self.keys, self.values = self._k[..., :n, :], self._v[..., :n, :]

    def batch_select_indices(self, indices: torch.Tensor) -> None:
        if self.get_seq_length() > 0:
            n = self.keys.shape[-2]
            self._k = self._k[indices, ...].contiguous()
            self._v = self._v[indices, ...].contiguous()
            self.keys, self.values = self._k[..., :n, :], self._v[..., :n, :]


class TreeAppendCache(Cache):
    """``Cache`` of ``TreeAppendLayer`` s: pass it as ``past_key_values`` in
    place of a ``DynamicCache``.  ``capacity`` rows are preallocated per layer
    at the first update (``num_layers`` from ``config.num_hidden_layers`` when
    given; otherwise layers are added as the model reaches them)."""

    def __init__(self, capacity: int, config=None, num_layers: int | None = None):
        if num_layers is None and config is not None:
            text = config.get_text_config(decoder=True) if hasattr(config, "get_text_config") else config
            num_layers = getattr(text, "num_hidden_layers", None)
        self.capacity = int(capacity)
        self.offset_dev = None
        if num_layers is not None:
            super().__init__(layers=[TreeAppendLayer(capacity) for _ in range(int(num_layers))])
        else:
            super().__init__(layer_class_to_replicate=TreeAppendLayer)

    def update(self, key_states, value_states, layer_idx: int, *args, **kwargs):
        # layers added on demand get this cache's capacity
        while len(self.layers) <= layer_idx:
            layer = TreeAppendLayer(self.capacity)
            layer.offset_dev = self.offset_dev
            self.layers.append(layer)
        return self.layers[layer_idx].update(key_states, value_states, *args, **kwargs)

    def update_at(self, key_states, value_states, layer_idx: int, offset_dev, rows_dev=None):
        """Static-mode append of one layer at a device-side row offset."""
        while len(self.layers) <= layer_idx:
            self.layers.append(TreeAppendLayer(self.capacity))
        return self.layers[layer_idx].update_at(key_states, value_states, offset_dev, rows_dev)

    def set_static(self, offset_dev: torch.Tensor | None) -> None:
        """Enter static mode (appends at ``offset_dev``, an int32 device
        scalar, and whole-buffer views) or leave it with None."""
        self.offset_dev = offset_dev
        for layer in self.layers:
            layer.offset_dev = offset_dev
            if layer.is_initialized and offset_dev is not None:
                layer.keys, layer.values = layer._k, layer._v
