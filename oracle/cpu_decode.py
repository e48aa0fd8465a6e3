"""CPU port of the reference's DDTree decode loop, used as the timed CPU
baseline of the end-to-end decode benchmark.

TEST / MEASUREMENT INFRASTRUCTURE ONLY (bench.py's CPU-baseline leg and
``--impl reference``).  The reference's loop (ddtree.py:372-587) is pure
Python on top of torch and transformers; this port makes the same library
calls on the host, in the same order:

  prefill       HF target forward with output_hidden_states, logits_to_keep=1
  draft         embed_tokens -> DFlash draft (SDPA, non-causal) -> lm_head
                (ddtree.py:476-486; model/dflash.py:36-197)
  tree build    torch.topk + torch.logsumexp, heapq expansion, numpy
                visibility (ddtree.py:114-196; cpu_reference.build_tree)
  compile       dense additive mask rows (ddtree.py:199-253)
  verify        HF target forward with the 4-D mask, DynamicCache.update
                (torch.cat), SDPA with repeat_kv (ddtree.py:523-531)
  commit        argmax, .tolist() walk, index_select, per-layer
                index_select + copy_ compaction and crop (ddtree.py:534-548)

The DFlash draft here is a restatement of model/dflash.py with the same
parameter names, computed with torch SDPA.
"""
from __future__ import annotations

import time

import numpy as np
import torch
from torch import nn

from . import cpu_reference as R


def _rotate_half(x):
    h = x.shape[-1] // 2
    return torch.cat((-x[..., h:], x[..., :h]), dim=-1)


class _RMSNorm(nn.Module):
    def __init__(self, n, eps):
        super().__init__()
        self.weight = nn.Parameter(torch.ones(n))
        self.eps = eps

    def forward(self, x):
        dt = x.dtype
        x = x.float()
        x = x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + self.eps)
        return self.weight * x.to(dt)


class _MLP(nn.Module):
    def __init__(self, h, i):
        super().__init__()
        self.gate_proj = nn.Linear(h, i, bias=False)
        self.up_proj = nn.Linear(h, i, bias=False)
        self.down_proj = nn.Linear(i, h, bias=False)

    def forward(self, x):
        return self.down_proj(nn.functional.silu(self.gate_proj(x)) * self.up_proj(x))


class _Attn(nn.Module):
    def __init__(self, cfg, idx):
        super().__init__()
        self.idx = idx
        self.hd = cfg.head_dim
        self.hq, self.hkv = cfg.num_attention_heads, cfg.num_key_value_heads
        h = cfg.hidden_size
        self.q_proj = nn.Linear(h, self.hq * self.hd, bias=False)
        self.k_proj = nn.Linear(h, self.hkv * self.hd, bias=False)
        self.v_proj = nn.Linear(h, self.hkv * self.hd, bias=False)
        self.o_proj = nn.Linear(self.hq * self.hd, h, bias=False)
        self.q_norm = _RMSNorm(self.hd, cfg.rms_norm_eps)
        self.k_norm = _RMSNorm(self.hd, cfg.rms_norm_eps)

    def forward(self, x, ctx, cos, sin, cache):
        b, q_len, _ = x.shape
        c_len = ctx.shape[1]
        q = self.q_norm(self.q_proj(x).view(b, q_len, -1, self.hd)).transpose(1, 2)
        k = torch.cat([self.k_proj(ctx), self.k_proj(x)], 1).view(b, c_len + q_len, -1, self.hd)
        v = torch.cat([self.v_proj(ctx), self.v_proj(x)], 1).view(b, c_len + q_len, -1, self.hd)
        k = self.k_norm(k).transpose(1, 2)
        v = v.transpose(1, 2)
        c, s = cos.unsqueeze(1), sin.unsqueeze(1)
        q = q * c[..., -q_len:, :] + _rotate_half(q) * s[..., -q_len:, :]
        k = k * c + _rotate_half(k) * s
        k, v = cache.update(k, v, self.idx)
        g = self.hq // self.hkv
        k = k.repeat_interleave(g, dim=1)
        v = v.repeat_interleave(g, dim=1)
        o = nn.functional.scaled_dot_product_attention(q, k, v, is_causal=False, scale=self.hd ** -0.5)
        return self.o_proj(o.transpose(1, 2).reshape(b, q_len, -1))


class _Layer(nn.Module):
    def __init__(self, cfg, idx):
        super().__init__()
        self.self_attn = _Attn(cfg, idx)
        self.mlp = _MLP(cfg.hidden_size, cfg.intermediate_size)
        self.input_layernorm = _RMSNorm(cfg.hidden_size, cfg.rms_norm_eps)
        self.post_attention_layernorm = _RMSNorm(cfg.hidden_size, cfg.rms_norm_eps)

    def forward(self, x, ctx, cos, sin, cache):
        x = x + self.self_attn(self.input_layernorm(x), ctx, cos, sin, cache)
        return x + self.mlp(self.post_attention_layernorm(x))


class CpuDFlashDraft(nn.Module):
    """model/dflash.py:153-197 restated (parameter names kept)."""

    def __init__(self, cfg):
        super().__init__()
        self.layers = nn.ModuleList([_Layer(cfg, i) for i in range(cfg.num_hidden_layers)])
        self.target_layer_ids = list(cfg.dflash_config["target_layer_ids"])
        self.mask_token_id = cfg.dflash_config["mask_token_id"]
        self.block_size = cfg.block_size
        self.norm = _RMSNorm(cfg.hidden_size, cfg.rms_norm_eps)
        self.fc = nn.Linear(len(self.target_layer_ids) * cfg.hidden_size, cfg.hidden_size, bias=False)
        self.hidden_norm = _RMSNorm(cfg.hidden_size, cfg.rms_norm_eps)
        rope = getattr(cfg, "rope_parameters", None) or {}
        base = rope.get("rope_theta", getattr(cfg, "rope_theta", 10000.0))
        self.register_buffer("inv_freq", 1.0 / (base ** (torch.arange(0, cfg.head_dim, 2).float() / cfg.head_dim)),
                             persistent=False)

    def forward(self, position_ids, noise_embedding, target_hidden, past_key_values):
        x = noise_embedding
        ctx = self.hidden_norm(self.fc(target_hidden))
        f = position_ids[0].float()[:, None] * self.inv_freq[None, :]
        emb = torch.cat([f, f], -1)
        cos, sin = emb.cos().to(x.dtype)[None], emb.sin().to(x.dtype)[None]
        for layer in self.layers:
            x = layer(x, ctx, cos, sin, past_key_values)
        return self.norm(x)


def _features(hidden_states, layer_ids):
    return torch.cat([hidden_states[i + 1] for i in layer_ids], dim=-1)


class CpuDecode:
    """The reference loop on the host, split so that a benchmark can time
    the prefill and a bounded number of rounds.  ``target`` is an HF causal
    LM on the CPU (loaded with SDPA attention, as the reference requires);
    ``draft`` a CpuDFlashDraft."""

    def __init__(self, draft, target, input_ids, max_new_tokens, block_size, budget):
        from transformers import DynamicCache
        self.draft, self.target = draft, target
        self.P = input_ids.shape[1]
        self.max_length = self.P + max_new_tokens
        self.block = block_size
        self.budget = budget
        self.mask_id = draft.mask_token_id
        N = 1 + budget
        self.output_ids = torch.full((1, self.max_length + N), self.mask_id, dtype=torch.long)
        self.pos = torch.arange(self.output_ids.shape[1]).unsqueeze(0)
        self.tcache, self.dcache = DynamicCache(), DynamicCache()
        self.mask_buf = torch.zeros((1, 1, N, self.max_length + N), dtype=target.dtype)
        self.input_ids = input_ids
        self.prev = (0, 0)
        self.acceptance = []

    @torch.inference_mode()
    def prefill(self) -> float:
        t0 = time.perf_counter()
        out = self.target(self.input_ids, position_ids=self.pos[:, : self.P], past_key_values=self.tcache,
                          use_cache=True, logits_to_keep=1, output_hidden_states=True)
        self.output_ids[:, : self.P] = self.input_ids
        self.output_ids[:, self.P: self.P + 1] = torch.argmax(out.logits, dim=-1)
        self.hidden = _features(out.hidden_states, self.draft.target_layer_ids)
        self.start = self.P
        return time.perf_counter() - t0

    @torch.inference_mode()
    def round(self) -> dict:
        t = {}
        t0 = time.perf_counter()
        start, block = self.start, self.block
        ids = self.output_ids[:, start: start + block].clone()
        noise = self.target.model.embed_tokens(ids)
        h = self.draft(self.pos[:, self.dcache.get_seq_length(): start + block], noise, self.hidden, self.dcache)
        logits = self.target.lm_head(h[:, -(block - 1):, :])
        self.dcache.crop(start)
        t1 = time.perf_counter()
        toks, deps, parents, child_maps, vis = R.build_tree(logits[0], self.budget)
        t2 = time.perf_counter()
        N = 1 + len(toks)
        vid = torch.empty((1, N), dtype=torch.long)
        vid[0, 0] = ids[0, 0]
        vid[0, 1:] = torch.from_numpy(toks)
        vpos = (torch.from_numpy(np.concatenate([[0], deps])) + start).unsqueeze(0)
        ps, pl = self.prev
        if pl > 0:
            self.mask_buf[0, 0, :pl, ps: ps + pl] = 0
        blk = self.mask_buf[0, 0, :N, start: start + N]
        blk.fill_(torch.finfo(self.target.dtype).min)
        blk.masked_fill_(torch.from_numpy(vis), 0)
        self.prev = (start, N)
        mask = self.mask_buf[:, :, :N, : start + N]
        t3 = time.perf_counter()
        out = self.target(vid, position_ids=vpos, attention_mask=mask, past_key_values=self.tcache, use_cache=True,
                          output_hidden_states=True)
        t4 = time.perf_counter()
        post = torch.argmax(out.logits, dim=-1)
        acc, nxt = R.follow(child_maps, post)
        acc_t = torch.tensor(acc, dtype=torch.long)
        self.output_ids[:, start: start + len(acc)] = vid.index_select(1, acc_t)
        self.output_ids[:, start + len(acc)] = nxt
        tensors = []
        for layer in self.tcache.layers:
            tensors += [layer.keys, layer.values]
        R.compact(tensors, start, acc)
        self.tcache.crop(start + len(acc))
        self.hidden = _features(out.hidden_states, self.draft.target_layer_ids).index_select(1, acc_t)
        self.start = start + len(acc)
        self.acceptance.append(len(acc))
        t5 = time.perf_counter()
        t.update(draft=t1 - t0, tree_build=t2 - t1, tree_compile=t3 - t2, verify=t4 - t3, commit=t5 - t4,
                 total=t5 - t0, accepted=len(acc))
        return t


def build_cpu_models(target_cfg, draft_cfg, dtype=torch.bfloat16, seed: int = 0):
    """Random-init CPU target (HF, SDPA) and CpuDFlashDraft in ``dtype``."""
    from transformers import Qwen3ForCausalLM
    old = torch.get_default_dtype()
    torch.manual_seed(seed)
    try:
        torch.set_default_dtype(dtype)
        target_cfg._attn_implementation = "sdpa"
        target = Qwen3ForCausalLM(target_cfg).eval()
        draft = CpuDFlashDraft(draft_cfg).eval()
        with torch.no_grad():
            for name, p in draft.named_parameters():
                if not name.endswith("norm.weight"):
                    p.normal_(0.0, 0.02)
    finally:
        torch.set_default_dtype(old)
    return target.to(dtype), draft.to(dtype)
