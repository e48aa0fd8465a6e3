"""CPU port of the reference's per-step hot path, used as the timed CPU baseline.

TEST / MEASUREMENT INFRASTRUCTURE ONLY (bench.py's CPU-baseline leg and
``--impl reference``).  The reference is pure Python on top of torch, so the
port makes the same library calls it makes, on the host:

  tree build    torch.topk + torch.logsumexp in fp32, heapq best-first
                expansion, numpy visibility           (ddtree.py:132-189)
  compile       dense additive mask rows in the target dtype (ddtree.py:247-251)
  verify attn   HF sdpa_attention_forward math: repeat_kv, then
                torch.nn.functional.scaled_dot_product_attention with the
                float mask, bf16                       (transformers
                integrations/sdpa_attention.py, called via ddtree.py:523-531)
  accept        torch.argmax + .tolist() + dict walk   (model/utils.py:28-30,
                ddtree.py:290-301)
  compaction    index_select + copy_ per layer K and V (ddtree.py:61-88, 304-320)
"""
from __future__ import annotations

import heapq
import time

import numpy as np
import torch


def build_tree(draft_logits: torch.Tensor, budget: int):
    topk = min(budget, draft_logits.shape[-1])
    depth_limit = int(draft_logits.shape[0])
    logits = draft_logits.float()
    top_logits, top_ids = torch.topk(logits, k=topk, dim=-1)
    log_z = torch.logsumexp(logits, dim=-1, keepdim=True)
    lp = (top_logits - log_z).numpy()
    ids = top_ids.numpy()
    first = float(lp[0, 0])
    heap = [(-first, (0,), 0, 1, 0, first)]
    toks = np.empty(budget, np.int64)
    deps = np.empty(budget, np.int64)
    parents = np.empty(budget + 1, np.int32)
    parents[0] = -1
    child_maps = [dict()]
    n = 0
    while heap and n < budget:
        _, ranks, parent, depth, rank, logw = heapq.heappop(heap)
        tok = int(ids[depth - 1, rank])
        cur = n + 1
        toks[n] = tok
        deps[n] = depth
        parents[cur] = parent
        child_maps.append(dict())
        child_maps[parent][tok] = cur
        n += 1
        if rank + 1 < topk:
            s = logw - float(lp[depth - 1, rank]) + float(lp[depth - 1, rank + 1])
            heapq.heappush(heap, (-s, ranks[:-1] + (rank + 1,), parent, depth, rank + 1, s))
        if depth < depth_limit:
            c = logw + float(lp[depth, 0])
            heapq.heappush(heap, (-c, ranks + (0,), cur, depth + 1, 0, c))
    N = n + 1
    vis = np.zeros((N, N), np.bool_)
    vis[0, 0] = True
    for i in range(1, N):
        vis[i, :i] = vis[parents[i], :i]
        vis[i, i] = True
    return toks[:n], deps[:n], parents[:N].tolist(), child_maps, vis


def dense_mask(vis: np.ndarray, past: int, dtype=torch.bfloat16) -> torch.Tensor:
    N = vis.shape[0]
    m = torch.zeros((1, 1, N, past + N), dtype=dtype)
    blk = m[0, 0, :, past:]
    blk.fill_(torch.finfo(dtype).min)
    blk.masked_fill_(torch.from_numpy(vis), 0)
    return m


def verify_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, mask: torch.Tensor, scale: float):
    """q [1, Hq, N, D]; k, v [1, Hkv, S, D]; HF sdpa path with repeat_kv."""
    g = q.shape[1] // k.shape[1]
    k = k[:, :, None].expand(-1, -1, g, -1, -1).reshape(1, -1, k.shape[2], k.shape[3])
    v = v[:, :, None].expand(-1, -1, g, -1, -1).reshape(1, -1, v.shape[2], v.shape[3])
    o = torch.nn.functional.scaled_dot_product_attention(q, k, v, attn_mask=mask, scale=scale)
    return o.transpose(1, 2).contiguous()


def follow(child_maps, posterior: torch.Tensor):
    post = posterior[0].tolist()
    acc = [0]
    cur = 0
    nxt = int(post[0])
    while nxt in child_maps[cur]:
        cur = child_maps[cur][nxt]
        acc.append(cur)
        nxt = int(post[cur])
    return acc, nxt


def compact(tensors, past: int, keep):
    keep_t = torch.tensor(keep, dtype=torch.long)
    for t in tensors:
        cur = t.shape[-2] - past
        if cur <= 0 or len(keep) == cur:
            continue
        kept = t.narrow(-2, past, cur).index_select(-2, keep_t)
        t.narrow(-2, past, len(keep)).copy_(kept)


class CpuStep:
    """One hot-path step on the host; ``attn_layers`` bounds how many of the
    target's layers are attended per call (the timing is scaled to all of
    them by the caller)."""

    def __init__(self, draft_logits, verify_logits, qs, ks, vs, past: int, budget: int, scale: float,
                 layers: int):
        self.draft_logits = draft_logits
        self.verify_logits = verify_logits
        self.qs, self.ks, self.vs = qs, ks, vs
        self.past = past
        self.budget = budget
        self.scale = scale
        self.layers = layers

    def run(self, attn_layers: int):
        t0 = time.perf_counter()
        toks, deps, parents, child_maps, vis = build_tree(self.draft_logits, self.budget)
        mask = dense_mask(vis, self.past)
        t1 = time.perf_counter()
        for layer in range(attn_layers):
            verify_attention(self.qs[layer], self.ks[layer], self.vs[layer], mask, self.scale)
        t2 = time.perf_counter()
        posterior = torch.argmax(self.verify_logits, dim=-1)
        acc, nxt = follow(child_maps, posterior)
        compact([t for pair in zip(self.ks, self.vs) for t in pair], self.past, acc)
        t3 = time.perf_counter()
        return {"build": t1 - t0, "attention": t2 - t1, "accept_compact": t3 - t2, "accepted": len(acc),
                "attn_layers": attn_layers}
