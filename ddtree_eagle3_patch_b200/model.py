"""The DFlash block-diffusion draft model and the model-side helpers that the
decode loop calls (the reference's ``model`` package: model/dflash.py,
model/utils.py of kimwin2/ddtree_eagle3_patch).

The draft is not part of the accelerated path: it produces the draft logits
that the tree build consumes.  It is here so the decode loop can run where
the reference cannot be imported, and its parameter names, config keys and
``forward`` signature are the reference's, so a DFlash checkpoint loads
into it unchanged (``DFlashDraftModel.from_pretrained``) and ``ddtree_generate``
accepts either class.

What it computes (model/dflash.py:28-197): each layer attends from the
block's noise rows (queries) to [context rows ; noise rows] (keys/values),
non-causally; the context rows are the target's hidden features projected
by ``fc`` and normalised by ``hidden_norm``; K gets ``k_norm`` before the
rotary embedding and Q takes the last ``q_len`` rotary positions.  The
attention itself runs on the tree-attention kernel with every key visible,
over the draft cache's rows in place.
"""
from __future__ import annotations

import os
from typing import Optional

import numpy as np
import torch
import torch.nn.functional as F
from torch import nn
from transformers.models.qwen3.modeling_qwen3 import (
    Qwen3Config,
    Qwen3MLP,
    Qwen3PreTrainedModel,
    Qwen3RMSNorm,
    Qwen3RotaryEmbedding,
    rotate_half,
)

from . import kernels

__all__ = [
    "DFlashDraftModel",
    "build_target_layer_ids",
    "extract_context_feature",
    "sample",
    "get_final_logit_softcapping",
    "apply_final_logit_softcapping",
]


def build_target_layer_ids(num_target_layers: int, num_draft_layers: int) -> list[int]:
    """Target layers whose hidden states feed the draft (model/utils.py:5-15):
    the middle layer for a 1-layer draft, else evenly spaced from layer 1 to
    layer num_target_layers - 3."""
    if num_draft_layers == 1:
        return [num_target_layers // 2]
    lo, hi = 1, num_target_layers - 3
    return [int(round(lo + i * (hi - lo) / (num_draft_layers - 1))) for i in range(num_draft_layers)]


def extract_context_feature(hidden_states, layer_ids) -> torch.Tensor:
    """Concatenate the target's hidden states after each listed layer
    (index + 1 into HF's ``hidden_states``, whose entry 0 is the embedding
    output; model/utils.py:17-26)."""
    return torch.cat([hidden_states[i + 1] for i in layer_ids], dim=-1)


def sample(logits: torch.Tensor, temperature: float = 0.0) -> torch.Tensor:
    """``model.utils.sample`` (model/utils.py:28-35) on the device kernels:
    row argmax below temperature 1e-5, else a draw from softmax(logits / T)."""
    return kernels.sample(logits, temperature)


def get_final_logit_softcapping(config) -> Optional[float]:
    """``dflash_config['final_logit_softcapping']``, else the config attribute
    (model/utils.py:37-42)."""
    dflash_config = getattr(config, "dflash_config", None) or {}
    value = dflash_config.get("final_logit_softcapping", getattr(config, "final_logit_softcapping", None))
    return None if value is None else float(value)


def apply_final_logit_softcapping(logits: torch.Tensor, final_logit_softcapping: Optional[float]) -> torch.Tensor:
    """cap * tanh(logits / cap), or the logits unchanged (model/utils.py:44-50)."""
    if final_logit_softcapping is None:
        return logits
    return torch.tanh(logits / final_logit_softcapping) * final_logit_softcapping


_ALL_VISIBLE: dict = {}


def _all_visible_bits(n: int, device: torch.device) -> torch.Tensor:
    """Packed mask of n rows that see all n new keys (non-causal)."""
    key = (n, device)
    b = _ALL_VISIBLE.get(key)
    if b is None:
        words = np.zeros((n, (n + 31) // 32), np.uint32)
        full, rem = divmod(n, 32)
        words[:, :full] = 0xFFFFFFFF
        if rem:
            words[:, full] = (1 << rem) - 1
        b = torch.from_numpy(words.view(np.int32)).to(device)
        _ALL_VISIBLE[key] = b
    return b


class DFlashAttention(nn.Module):
    """Noise-row queries over [context ; noise] keys (model/dflash.py:36-108)."""

    def __init__(self, config: Qwen3Config, layer_idx: int):
        super().__init__()
        self.layer_idx = layer_idx
        self.head_dim = getattr(config, "head_dim", None) or config.hidden_size // config.num_attention_heads
        self.num_heads = config.num_attention_heads
        self.num_kv_heads = config.num_key_value_heads
        self.scaling = self.head_dim ** -0.5
        bias = config.attention_bias
        self.q_proj = nn.Linear(config.hidden_size, self.num_heads * self.head_dim, bias=bias)
        self.k_proj = nn.Linear(config.hidden_size, self.num_kv_heads * self.head_dim, bias=bias)
        self.v_proj = nn.Linear(config.hidden_size, self.num_kv_heads * self.head_dim, bias=bias)
        self.o_proj = nn.Linear(self.num_heads * self.head_dim, config.hidden_size, bias=bias)
        self.q_norm = Qwen3RMSNorm(self.head_dim, eps=config.rms_norm_eps)
        self.k_norm = Qwen3RMSNorm(self.head_dim, eps=config.rms_norm_eps)

    def forward(self, hidden_states: torch.Tensor, target_hidden: torch.Tensor, position_embeddings,
                past_key_values=None) -> torch.Tensor:
        bsz, q_len, _ = hidden_states.shape
        if bsz != 1:
            raise NotImplementedError("the DFlash draft runs batch 1, as the reference's decode loop does")
        ctx_len = target_hidden.shape[1]
        hd = self.head_dim
        q = self.q_norm(self.q_proj(hidden_states).view(1, q_len, self.num_heads, hd))
        # context and noise rows are projected separately, as in the reference,
        # so each row sees the same GEMM shapes as there
        k = torch.cat([self.k_proj(target_hidden), self.k_proj(hidden_states)], dim=1)
        v = torch.cat([self.v_proj(target_hidden), self.v_proj(hidden_states)], dim=1)
        k = self.k_norm(k.view(1, ctx_len + q_len, self.num_kv_heads, hd)).transpose(1, 2)
        v = v.view(1, ctx_len + q_len, self.num_kv_heads, hd).transpose(1, 2)
        cos, sin = position_embeddings
        cos_q, sin_q = cos[:, -q_len:].unsqueeze(2), sin[:, -q_len:].unsqueeze(2)
        q = q * cos_q + rotate_half(q) * sin_q                      # [1, q_len, Hq, D]
        k = k * cos.unsqueeze(1) + rotate_half(k) * sin.unsqueeze(1)  # [1, Hkv, S, D]
        if past_key_values is not None:
            k, v = past_key_values.update(k, v, self.layer_idx)
        kv_len = k.shape[-2]
        bits = _all_visible_bits(q_len, q.device)
        out = kernels.tree_attention(q[0], k[0], v[0], kv_len - q_len, bits, self.scaling)
        return self.o_proj(out.reshape(1, q_len, self.num_heads * hd))

    def forward_static(self, hidden_states, target_hidden, position_embeddings, cache, rs, past_max: int,
                       workspace) -> torch.Tensor:
        """The same attention with every length on the device (a forward
        that can be captured once and replayed each round).  ``rs`` is an
        int32 device vector [start, ctx_offset, ctx_count]: the first
        ctx_count of the context rows go to the draft cache at ctx_offset,
        the block's rows at start, and the block's queries see the cache's
        first start rows and every block row."""
        q_len, ctx_len, hd = hidden_states.shape[1], target_hidden.shape[1], self.head_dim
        q = self.q_norm(self.q_proj(hidden_states).view(1, q_len, self.num_heads, hd))
        k = torch.cat([self.k_proj(target_hidden), self.k_proj(hidden_states)], dim=1)
        v = torch.cat([self.v_proj(target_hidden), self.v_proj(hidden_states)], dim=1)
        k = self.k_norm(k.view(1, ctx_len + q_len, self.num_kv_heads, hd)).transpose(1, 2)
        v = v.view(1, ctx_len + q_len, self.num_kv_heads, hd).transpose(1, 2)
        cos, sin = position_embeddings
        q = q * cos[:, -q_len:].unsqueeze(2) + rotate_half(q) * sin[:, -q_len:].unsqueeze(2)
        k = k * cos.unsqueeze(1) + rotate_half(k) * sin.unsqueeze(1)
        cache.update_at(k[:, :, :ctx_len], v[:, :, :ctx_len], self.layer_idx, rs[1:2], rs[2:3])
        kf, vf = cache.update_at(k[:, :, ctx_len:], v[:, :, ctx_len:], self.layer_idx, rs[0:1])
        bits = _all_visible_bits(q_len, q.device)
        # keys before this round's context rows (at rs[1]) are stable
        out = kernels.tree_attention(q[0], kf[0], vf[0], past_max, bits, self.scaling, past_dev=rs[0:1],
                                     workspace=workspace, stable_dev=rs[1:2])
        return self.o_proj(out.reshape(1, q_len, self.num_heads * hd))


class DFlashDecoderLayer(nn.Module):
    """Pre-norm attention + MLP block (model/dflash.py:110-150)."""

    def __init__(self, config: Qwen3Config, layer_idx: int):
        super().__init__()
        self.self_attn = DFlashAttention(config, layer_idx)
        self.mlp = Qwen3MLP(config)
        self.input_layernorm = Qwen3RMSNorm(config.hidden_size, eps=config.rms_norm_eps)
        self.post_attention_layernorm = Qwen3RMSNorm(config.hidden_size, eps=config.rms_norm_eps)

    def forward(self, hidden_states, target_hidden, position_embeddings, past_key_values=None):
        h = hidden_states + self.self_attn(self.input_layernorm(hidden_states), target_hidden, position_embeddings,
                                           past_key_values)
        return h + self.mlp(self.post_attention_layernorm(h))

    def forward_static(self, hidden_states, target_hidden, position_embeddings, cache, rs, past_max, workspace):
        """The layer with device-side cache lengths.  For the Qwen3-style
        layer (head_dim 128, no biases, SiLU) the elementwise steps run as
        fused kernels: RMSNorm, q/k norm + rotary embedding + both cache
        appends in one launch, SiLU * up; the residual adds fold into the
        o_proj / down_proj GEMMs."""
        from .fused_layers import supported_layer
        if not supported_layer(self) or os.environ.get("DDTREE_FUSED", "1") == "0":
            h = hidden_states + self.self_attn.forward_static(self.input_layernorm(hidden_states), target_hidden,
                                                              position_embeddings, cache, rs, past_max, workspace)
            return h + self.mlp(self.post_attention_layernorm(h))
        from .fused_layers import gate_up_act, linear_rows, packed_weights, residual_linear
        attn, mlp = self.self_attn, self.mlp
        x, c = hidden_states[0], target_hidden[0]
        T = x.shape[0]
        nq, nk = attn.num_heads * attn.head_dim, attn.num_kv_heads * attn.head_dim
        h = kernels.rms_norm(x, self.input_layernorm.weight, self.input_layernorm.variance_epsilon)
        packed = packed_weights(self)
        if packed is not None:
            qkv = linear_rows(h, packed[0], "draft_qkv")
            q, k_n, v_n = qkv[:, :nq], qkv[:, nq: nq + nk], qkv[:, nq + nk:]
            kv = linear_rows(c, packed[0][nq:], "draft_qkv")
            k_c, v_c = kv[:, :nk], kv[:, nk:]
        else:
            q = F.linear(h, attn.q_proj.weight)
            k_c, v_c = F.linear(c, attn.k_proj.weight), F.linear(c, attn.v_proj.weight)
            k_n, v_n = F.linear(h, attn.k_proj.weight), F.linear(h, attn.v_proj.weight)
        layer_cache = cache.layers[attn.layer_idx]
        if not layer_cache.is_initialized:
            empty = torch.empty((1, attn.num_kv_heads, 0, attn.head_dim), dtype=x.dtype, device=x.device)
            layer_cache.lazy_initialization(empty, empty)
        cos, sin = position_embeddings
        qr = kernels.qk_norm_rope_append(q, k_n, v_n, attn.q_norm.weight, attn.k_norm.weight,
                                         attn.q_norm.variance_epsilon, attn.k_norm.variance_epsilon, cos[0], sin[0],
                                         layer_cache._k, layer_cache._v, rs, attn.num_heads, attn.num_kv_heads,
                                         ctx_k=k_c, ctx_v=v_c)
        bits = _all_visible_bits(T, x.device)
        # the append above wrote the context rows at rs[1] and the block at
        # rs[0]: keys before rs[1] are stable
        o = kernels.tree_attention(qr, layer_cache._k[0], layer_cache._v[0], past_max, bits, attn.scaling,
                                   past_dev=rs[0:1], workspace=workspace, stable_dev=rs[1:2])
        x2 = residual_linear(o.view(T, -1), attn.o_proj.weight, x, "o")
        h2 = kernels.rms_norm(x2, self.post_attention_layernorm.weight, self.post_attention_layernorm.variance_epsilon)
        if packed is not None:
            a = gate_up_act(h2, packed[1])
        else:
            a = kernels.silu_mul(F.linear(h2, mlp.gate_proj.weight), F.linear(h2, mlp.up_proj.weight))
        return residual_linear(a, mlp.down_proj.weight, x2, "down").unsqueeze(0)


class DFlashDraftModel(Qwen3PreTrainedModel):
    """The DFlash block draft (model/dflash.py:153-197): same config keys
    (``dflash_config.target_layer_ids`` / ``mask_token_id``, ``block_size``,
    ``num_target_layers``), same parameter names, same ``forward``."""

    config_class = Qwen3Config
    _no_split_modules = ["DFlashDecoderLayer"]

    def __init__(self, config) -> None:
        super().__init__(config)
        self.config = config
        layer_types = getattr(config, "layer_types", None) or []
        if "sliding_attention" in layer_types:
            raise NotImplementedError("sliding-window DFlash draft layers are not supported")
        self.layers = nn.ModuleList([DFlashDecoderLayer(config, i) for i in range(config.num_hidden_layers)])
        dflash_config = getattr(config, "dflash_config", None) or {}
        self.target_layer_ids = dflash_config.get(
            "target_layer_ids", build_target_layer_ids(config.num_target_layers, config.num_hidden_layers))
        self.norm = Qwen3RMSNorm(config.hidden_size, eps=config.rms_norm_eps)
        self.rotary_emb = Qwen3RotaryEmbedding(config)
        self.fc = nn.Linear(len(self.target_layer_ids) * config.hidden_size, config.hidden_size, bias=False)
        self.hidden_norm = Qwen3RMSNorm(config.hidden_size, eps=config.rms_norm_eps)
        self.block_size = config.block_size
        self.mask_token_id = dflash_config.get("mask_token_id", None)
        self.final_logit_softcapping = get_final_logit_softcapping(config)
        self.post_init()

    def forward(self, position_ids: torch.LongTensor, attention_mask: Optional[torch.Tensor] = None,
                noise_embedding: Optional[torch.Tensor] = None, target_hidden: Optional[torch.Tensor] = None,
                past_key_values=None, use_cache: bool = False, **kwargs) -> torch.Tensor:
        """Hidden states of the noise rows, normalised: [1, q_len, hidden]."""
        if attention_mask is not None:
            raise NotImplementedError("the DFlash draft attends to every context and block row (no mask)")
        hidden_states = noise_embedding
        ctx = self.hidden_norm(self.fc(target_hidden))
        position_embeddings = self.rotary_emb(hidden_states, position_ids)
        cache = past_key_values if use_cache else None
        for layer in self.layers:
            hidden_states = layer(hidden_states, ctx, position_embeddings, cache)
        return self.norm(hidden_states)

    def forward_static(self, noise_embedding: torch.Tensor, target_hidden: torch.Tensor, position_ids: torch.Tensor,
                       cache, rs: torch.Tensor, past_max: int, workspace: torch.Tensor) -> torch.Tensor:
        """``forward`` with the cache lengths on the device, for a forward
        captured once and replayed every decode round.  ``cache`` is a
        TreeAppendCache; ``rs`` the int32 device vector [start, ctx_offset,
        ctx_count] (see DFlashAttention.forward_static); ``position_ids``
        cover the context rows then the block rows.  ``past_max`` bounds
        start."""
        from .fused_layers import linear_rows, rms_norm_rows
        fused = os.environ.get("DDTREE_FUSED", "1") != "0"
        norm = (lambda m, x: rms_norm_rows(m, x)) if fused else (lambda m, x: m(x))
        hidden_states = noise_embedding
        if fused and target_hidden.shape[0] == 1 and self.fc.bias is None:   # on the weight-streaming GEMM
            fc_out = linear_rows(target_hidden[0], self.fc.weight, "fc").unsqueeze(0)
        else:
            fc_out = self.fc(target_hidden)
        ctx = norm(self.hidden_norm, fc_out)
        position_embeddings = self.rotary_emb(hidden_states, position_ids)
        for layer in self.layers:
            hidden_states = layer.forward_static(hidden_states, ctx, position_embeddings, cache, rs, past_max, workspace)
        return norm(self.norm, hidden_states)
