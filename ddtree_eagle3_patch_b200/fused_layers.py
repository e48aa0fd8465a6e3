"""Fused forward of a Qwen3-style decoder layer for the captured verify
forward of a decode round.

The stock eager layer (transformers Qwen3DecoderLayer) issues ~50 kernels
per layer at verify time, six of them GEMMs; the rest are small elementwise
steps that dominate a round at batch 1.  ``fused_decoder_layers(target)``
gives each supported layer of the target, for the duration of a decode
call, a forward that keeps the six GEMMs (cuBLAS through torch, the two
residual adds folded into the o_proj and down_proj GEMMs as addmm) and
replaces everything else by four launches of this library:

  rms_norm                 input_layernorm / post_attention_layernorm
  qk_norm_rope_append      q_norm, k_norm, rotary embedding, and the K/V
                           append into the static cache at the device-side
                           prefix length
  tree attention           the verify attention, prefix length on the device
  silu_mul                 the MLP's act_fn(gate) * up

The fused forward runs only where the stock one would run the verify
attention through this library with a static cache (the stand-in mask of
``TreeMask.static``); any other call (the prefill, a host-mode cache)
takes the stock forward, so results outside the decode rounds are
unchanged.  The fused steps follow the stock modules' rounding order; the
addmm folds round the residual sum once instead of twice.
"""
from __future__ import annotations

import os
import types
from contextlib import contextmanager

import torch
import torch.nn.functional as F

from . import kernels


def _is_silu(act) -> bool:
    return isinstance(act, torch.nn.SiLU) or type(act).__name__ in ("SiLUActivation", "SiLU")


def supported_layer(layer) -> bool:
    """Qwen3-style layer: pre-norm attention with q_norm / k_norm, head_dim
    128, SwiGLU MLP with SiLU, no biases."""
    attn, mlp = getattr(layer, "self_attn", None), getattr(layer, "mlp", None)
    if attn is None or mlp is None:
        return False
    names = ("q_proj", "k_proj", "v_proj", "o_proj", "q_norm", "k_norm")
    if not all(hasattr(attn, n) for n in names) or not all(hasattr(mlp, n) for n in ("gate_proj", "up_proj",
                                                                                       "down_proj", "act_fn")):
        return False
    if not hasattr(layer, "input_layernorm") or not hasattr(layer, "post_attention_layernorm"):
        return False
    lin = (attn.q_proj, attn.k_proj, attn.v_proj, attn.o_proj, mlp.gate_proj, mlp.up_proj, mlp.down_proj)
    if any(getattr(m, "bias", None) is not None for m in lin):
        return False
    return getattr(attn, "head_dim", None) == 128 and _is_silu(mlp.act_fn) and getattr(attn, "sliding_window",
                                                                                        None) is None


def packed_weights(layer):
    """``([Wq; Wk; Wv], Wgate/Wup interleaved)`` of a layer: one GEMM for the
    three projections and one for the two MLP inputs instead of five, each
    streaming the same bytes (at a few dozen rows every GEMM is bound by its
    weight bytes plus a fixed latency, so fewer, larger ones are faster).
    The MLP pair is interleaved in blocks of 64 rows
    (``kernels.interleave_gate_up``) so one GEMM also applies act(gate) * up.
    Built once and kept on the layer (outside its state dict) while the
    source weights are unchanged; it costs a second copy of those weights
    (4.7 GB for Qwen3-4B).  ``None`` when DDTREE_PACK=0."""
    if os.environ.get("DDTREE_PACK", "1") == "0":
        return None
    attn, mlp = layer.self_attn, layer.mlp
    src = (attn.q_proj.weight, attn.k_proj.weight, attn.v_proj.weight, mlp.gate_proj.weight, mlp.up_proj.weight)
    if src[3].shape[0] % 64:
        return None
    key = tuple((w.data_ptr(), w._version, tuple(w.shape)) for w in src)
    cached = layer.__dict__.get("_ddtree_packed")
    if cached is None or cached[0] != key:
        with torch.no_grad():
            wqkv = torch.cat([w.detach() for w in src[:3]], 0)
            wgu = kernels.interleave_gate_up(src[3].detach(), src[4].detach())
        cached = (key, wqkv, wgu)
        layer.__dict__["_ddtree_packed"] = cached
    return cached[1], cached[2]


# Projections the weight-streaming GEMM serves by default.  The target's
# packed q/k/v (6144 x 2560 at Qwen3-4B) stays on cuBLAS: in the captured
# decode round it measured 286 tok/s there against 268 on this kernel.
_WGEMM_DEFAULT = {"qkv": "0"}


def _wgemm_on(kind: str) -> bool:
    """The weight-streaming GEMM serves projection ``kind`` (``qkv``,
    ``draft_qkv``, ``o``, ``gate_up``, ``down``, ``head``): DDTREE_WGEMM=0
    turns it off everywhere, DDTREE_WGEMM_<KIND>=0/1 per projection."""
    if os.environ.get("DDTREE_WGEMM", "1") == "0":
        return False
    return os.environ.get(f"DDTREE_WGEMM_{kind.upper()}", _WGEMM_DEFAULT.get(kind, "1")) != "0"


def linear_rows(x: torch.Tensor, w: torch.Tensor, kind: str) -> torch.Tensor:
    """x @ w.T for the few rows of a decode forward: the weight-streaming
    tcgen05 GEMM where it takes the shapes, else cuBLAS."""
    if _wgemm_on(kind) and kernels.wgemm_supported(x, w):
        return kernels.wgemm(x, w)
    return F.linear(x, w)


def gate_up_act(h: torch.Tensor, w_packed: torch.Tensor) -> torch.Tensor:
    """act(h Wg^T) * (h Wu^T) from the interleaved pair: one launch of the
    weight-streaming GEMM with the SiLU product in its epilogue, else cuBLAS
    and the elementwise kernel."""
    if _wgemm_on("gate_up") and kernels.wgemm_supported(h, w_packed):
        return kernels.wgemm_gate_up(h, w_packed)
    T = h.shape[0]
    gu = F.linear(h, w_packed).view(T, -1, 2, 64)
    inter = w_packed.shape[0] // 2
    return kernels.silu_mul(gu[:, :, 0].reshape(T, inter), gu[:, :, 1].reshape(T, inter))


def residual_linear(a: torch.Tensor, w: torch.Tensor, residual: torch.Tensor, kind: str) -> torch.Tensor:
    """residual + a @ w.T, rounded once (``torch.addmm``).  bf16 decode
    shapes run on the weight-streaming tcgen05 GEMM with the residual added
    in its epilogue (the o_proj and down_proj of a layer: at 33 rows it
    streams 21 / 50 MB of weights in 9.4 / 14.1 us against cuBLAS's 10.2 /
    16.7 us on B200); anything else on cuBLAS."""
    if _wgemm_on(kind) and kernels.wgemm_supported(a, w) and residual.dtype == torch.bfloat16 \
            and residual.stride(1) == 1:
        return kernels.wgemm(a, w, residual=residual)
    return torch.addmm(residual, a, w.t())


def head_logits(lm_head, h: torch.Tensor) -> torch.Tensor:
    """``lm_head(h)`` for the draft rows of a round ([1, L, hidden]).  A
    bias-free bf16 head runs on the weight-streaming GEMM (Qwen3-4B's
    151936 x 2560 head at 15 rows: 116 us against cuBLAS's 129 us on
    B200); anything else calls the module.  ``DDTREE_WGEMM=0`` keeps the
    module."""
    w = getattr(lm_head, "weight", None)
    if (_wgemm_on("head") and isinstance(lm_head, torch.nn.Linear)
            and lm_head.bias is None and h.dim() == 3 and h.shape[0] == 1):
        x = h[0]
        if kernels.wgemm_supported(x, w):
            return kernels.wgemm(x, w).unsqueeze(0)
    return lm_head(h)


def _fused_forward(self, hidden_states, attention_mask=None, position_ids=None, past_key_values=None,
                   use_cache=False, position_embeddings=None, **kwargs):
    past_dev = getattr(attention_mask, "ddtree_past_dev", None) if torch.is_tensor(attention_mask) else None
    if past_dev is None or getattr(past_key_values, "offset_dev", None) is None or hidden_states.shape[0] != 1:
        return type(self).forward(self, hidden_states, attention_mask=attention_mask, position_ids=position_ids,
                                  past_key_values=past_key_values, use_cache=use_cache,
                                  position_embeddings=position_embeddings, **kwargs)
    attn, mlp = self.self_attn, self.mlp
    x = hidden_states[0]
    T = x.shape[0]
    hq, hkv = attn.q_proj.weight.shape[0] // 128, attn.k_proj.weight.shape[0] // 128
    h = kernels.rms_norm(x, self.input_layernorm.weight, self.input_layernorm.variance_epsilon)
    packed = packed_weights(self)
    if packed is not None:
        qkv = linear_rows(h, packed[0], "qkv")
        q, k, v = qkv[:, : hq * 128], qkv[:, hq * 128: (hq + hkv) * 128], qkv[:, (hq + hkv) * 128:]
    else:
        q, k, v = F.linear(h, attn.q_proj.weight), F.linear(h, attn.k_proj.weight), F.linear(h, attn.v_proj.weight)
    cos, sin = position_embeddings
    cache = past_key_values.layers[attn.layer_idx]
    qr = kernels.qk_norm_rope_append(q, k, v, attn.q_norm.weight, attn.k_norm.weight, attn.q_norm.variance_epsilon,
                                     attn.k_norm.variance_epsilon, cos[0], sin[0], cache._k, cache._v,
                                     past_key_values.offset_dev, hq, hkv)
    # the tree rows just appended start at the prefix: every key before them is stable
    o = kernels.tree_attention(qr, cache._k[0], cache._v[0], attention_mask.ddtree_past_max,
                               attention_mask.ddtree_bits, attn.scaling, past_dev=past_dev,
                               workspace=attention_mask.ddtree_workspace, stable_dev=past_dev)
    x2 = residual_linear(o.view(T, -1), attn.o_proj.weight, x, "o")
    h2 = kernels.rms_norm(x2, self.post_attention_layernorm.weight, self.post_attention_layernorm.variance_epsilon)
    if packed is not None:
        a = gate_up_act(h2, packed[1])
    else:
        a = kernels.silu_mul(F.linear(h2, mlp.gate_proj.weight), F.linear(h2, mlp.up_proj.weight))
    return residual_linear(a, mlp.down_proj.weight, x2, "down").unsqueeze(0)


def rms_norm_rows(norm, x: torch.Tensor) -> torch.Tensor:
    """``norm(x)`` for a Qwen3RMSNorm over the last dimension: one launch of
    the fused RMSNorm kernel (the stock module's rounding order) for a CUDA
    tensor with contiguous rows in the weight's dtype, else the module's own
    forward."""
    if not x.is_cuda or x.stride(-1) != 1 or x.dtype != norm.weight.dtype \
            or x.dtype not in (torch.bfloat16, torch.float16, torch.float32):
        return type(norm).forward(norm, x)
    rows = x.reshape(-1, x.shape[-1])
    return kernels.rms_norm(rows, norm.weight, norm.variance_epsilon).view(x.shape)


def _norm_forward(self, hidden_states):
    return rms_norm_rows(self, hidden_states)


def _decoder_layers(model):
    inner = getattr(model, "model", model)
    layers = getattr(inner, "layers", None)
    return list(layers) if layers is not None else []


@contextmanager
def fused_decoder_layers(target):
    """Give every supported decoder layer of ``target`` the fused forward for
    the duration of the block (an instance attribute, removed afterwards)."""
    patched = []
    try:
        for layer in _decoder_layers(target):
            if supported_layer(layer) and "forward" not in layer.__dict__:
                layer.forward = types.MethodType(_fused_forward, layer)
                patched.append(layer)
        # the final norm before the lm_head, as one launch
        norm = getattr(getattr(target, "model", target), "norm", None)
        if patched and norm is not None and hasattr(norm, "variance_epsilon") and "forward" not in norm.__dict__:
            norm.forward = types.MethodType(_norm_forward, norm)
            patched.append(norm)
        yield len(patched)
    finally:
        for module in patched:
            module.__dict__.pop("forward", None)
