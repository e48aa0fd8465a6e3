"""Generate golden fixtures by running the reference implementation itself.

Run in the build container (where the reference is importable):

    python tests/golden/gen_golden.py <reference checkout>

It imports the reference's ``ddtree``, ``eagle3`` and ``model.utils`` modules
in-process (with ``dflash.cuda_time`` pointed at ``time.perf_counter`` so the
CPU path runs), feeds them seeded synthetic inputs and writes the inputs and
outputs to ``tests/golden/*.npz``.  Large inputs are not stored: they are
regenerated from the recorded torch seed and checked against a stored
SHA-256 of their bytes.

The fixtures pin ``oracle/`` (tests/test_oracle.py) and, through it, the CUDA
path.  Nothing at test time reads the reference.
"""
from __future__ import annotations

import hashlib
import sys
import time
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent.parent))

from ddtree_eagle3_patch_b200.synthetic import (  # noqa: E402
    cfg1_logits, deep_logits, posterior_for_tree, tree_attention_inputs, V_QWEN3)


def _import_reference(ref_root: str):
    sys.path.insert(0, ref_root)
    import dflash  # noqa: F401
    dflash.cuda_time = time.perf_counter
    import ddtree
    ddtree.cuda_time = time.perf_counter
    import eagle3
    eagle3.cuda_time = time.perf_counter
    from model import utils as mutils
    return ddtree, eagle3, mutils


def sha(t: torch.Tensor) -> str:
    return hashlib.sha256(t.contiguous().numpy().tobytes()).hexdigest()


def ref_lp_ids(logits: torch.Tensor, budget: int):
    """The reference's own top-k / log-normaliser arithmetic (ddtree.py:132-140)."""
    topk = min(budget, logits.shape[-1])
    x = logits.float()
    top_logits, top_ids = torch.topk(x, k=topk, dim=-1)
    log_z = torch.logsumexp(x, dim=-1, keepdim=True)
    return (top_logits - log_z).to(torch.float32).numpy(), top_ids.numpy().astype(np.int64), \
        log_z[:, 0].numpy(), top_logits.numpy()


def tree_record(ddtree, logits: torch.Tensor, budget: int, prefix: str, out: dict, store_input: bool):
    ids, depths, parents, child_maps, vis, _ = ddtree.build_ddtree_tree(logits, budget)
    if logits.shape[0] > 0 and budget > 0:
        lp, tids, logz, tvals = ref_lp_ids(logits, budget)
        out[prefix + "lp"] = lp
        out[prefix + "ids"] = tids
        out[prefix + "logz"] = logz
        out[prefix + "top_vals"] = tvals
    out[prefix + "budget"] = np.int64(budget)
    out[prefix + "node_token_ids"] = ids.numpy().astype(np.int64)
    out[prefix + "node_depths"] = depths.numpy().astype(np.int64)
    out[prefix + "parents"] = np.asarray(parents, np.int32)
    out[prefix + "visibility"] = vis.numpy().astype(bool)
    if store_input:
        out[prefix + "logits"] = logits.numpy()
    else:
        out[prefix + "logits_sha256"] = np.array(sha(logits))
        out[prefix + "logits_shape"] = np.array(list(logits.shape), np.int64)
    return ids, depths, parents, child_maps, vis


def gen_tree_cases(ddtree, mutils, out: dict):
    # configuration 1: seed 0, [15, 151936] fp32 N(0,1) + 8 peak, budgets 32 / 64
    for budget in (32, 64):
        logits = cfg1_logits(seed=0)
        p = f"cfg1_b{budget}_"
        ids, depths, parents, child_maps, vis = tree_record(ddtree, logits, budget, p, out, store_input=False)
        posterior = posterior_for_tree(ids.numpy(), depths.numpy(), out[p + "ids"], V_QWEN3, seed=budget)
        acc, nxt = ddtree.follow_verified_tree(child_maps, torch.from_numpy(posterior)[None])
        out[p + "posterior"] = posterior
        out[p + "accepted"] = np.asarray(acc, np.int64)
        out[p + "next_token"] = np.int64(nxt)
    # deep trees (+16 peaks make the top-1 chain dominate)
    for budget in (64, 128):
        logits = deep_logits(seed=1, peak=16.0)
        p = f"deep_b{budget}_"
        ids, depths, parents, child_maps, vis = tree_record(ddtree, logits, budget, p, out, store_input=False)
        posterior = posterior_for_tree(ids.numpy(), depths.numpy(), out[p + "ids"], V_QWEN3, seed=7 + budget,
                                       p_top1=0.9)
        acc, nxt = ddtree.follow_verified_tree(child_maps, torch.from_numpy(posterior)[None])
        out[p + "posterior"] = posterior
        out[p + "accepted"] = np.asarray(acc, np.int64)
        out[p + "next_token"] = np.int64(nxt)
    # small shapes, budgets around V (topk = min(budget, V)) and zero budget
    g = torch.Generator().manual_seed(3)
    for i, (L, V, budget) in enumerate([(4, 50, 1), (4, 50, 3), (4, 50, 8), (4, 50, 20), (3, 7, 12),
                                        (6, 300, 40), (1, 30, 5), (15, 1000, 64), (4, 50, 0), (0, 50, 5)]):
        logits = torch.randn(L, V, generator=g) * 2.0
        tree_record(ddtree, logits, budget, f"small{i}_", out, store_input=True)
    # exact ties in the float64 path scores: log-probs on a coarse dyadic grid
    for i, (L, V, budget) in enumerate([(5, 16, 24), (8, 8, 40), (3, 64, 64)]):
        gg = torch.Generator().manual_seed(100 + i)
        logits = torch.randint(-3, 1, (L, V), generator=gg).float()
        tree_record(ddtree, logits, budget, f"ties{i}_", out, store_input=True)
    # bf16-valued logits (value ties in the top-k)
    gg = torch.Generator().manual_seed(11)
    logits = (torch.randn(15, 4096, generator=gg) * 3).to(torch.bfloat16).float()
    tree_record(ddtree, logits, 32, "bf16_", out, store_input=True)


def gen_compile_cases(ddtree, out: dict):
    g = torch.Generator().manual_seed(5)
    logits = torch.randn(6, 200, generator=g) * 2
    ids, depths, parents, child_maps, vis, _ = ddtree.build_ddtree_tree(logits, 12)
    N = 1 + ids.numel()
    max_len, past, start = 64, 20, 20
    dtype = torch.bfloat16
    vi = torch.empty((1, 1 + 12), dtype=torch.long)
    vp = torch.empty((1, 1 + 12), dtype=torch.long)
    am = torch.zeros((1, 1, 1 + 12, max_len + 1 + 12), dtype=dtype)
    tv = torch.empty((1 + 12, 1 + 12), dtype=torch.bool)
    # a previous tree at [10, 10+7) to be cleared first
    am[0, 0, :7, 10:17] = torch.finfo(dtype).min
    r = ddtree.compile_ddtree_tree(torch.tensor(777), start, ids, depths, vis, past, dtype, torch.device("cpu"),
                                   vi, vp, am, tv, 10, 7)
    out["compile_node_token_ids"] = ids.numpy()
    out["compile_node_depths"] = depths.numpy()
    out["compile_visibility"] = vis.numpy()
    out["compile_ids"] = r[0].numpy()
    out["compile_pos"] = r[1].numpy()
    out["compile_mask"] = r[2].float().numpy()
    out["compile_full_buffer"] = am.float().numpy()
    out["compile_past"] = np.int64(r[3])
    out["compile_len"] = np.int64(r[4])
    # sliding-window hybrid mask
    am2 = torch.zeros_like(am)
    sm = torch.zeros_like(am)
    r2 = ddtree.compile_ddtree_tree(torch.tensor(777), start, ids, depths, vis, past, dtype, torch.device("cpu"),
                                    vi, vp, am2, tv, 0, 0, sliding_window=8, sliding_attention_mask_buffer=sm)
    out["compile_sw_full"] = r2[2]["full_attention"].float().numpy()
    out["compile_sw_sliding"] = r2[2]["sliding_attention"].float().numpy()


def gen_compact_cases(ddtree, out: dict):
    from transformers import DynamicCache
    g = torch.Generator().manual_seed(9)
    cache = DynamicCache()
    n_layers, H, past, cur, D = 3, 2, 11, 9, 16
    ks, vs = [], []
    for layer in range(n_layers):
        k = torch.randn(1, H, past + cur, D, generator=g).to(torch.bfloat16)
        v = torch.randn(1, H, past + cur, D, generator=g).to(torch.bfloat16)
        cache.update(k.clone(), v.clone(), layer)
        ks.append(k)
        vs.append(v)
    keep = [0, 2, 3, 7]
    ddtree.compact_dynamic_cache(cache, past, keep)
    out["compact_keys_in"] = torch.stack(ks).float().numpy()
    out["compact_values_in"] = torch.stack(vs).float().numpy()
    out["compact_keep"] = np.asarray(keep, np.int64)
    out["compact_past"] = np.int64(past)
    out["compact_keys_out"] = torch.stack([layer.keys for layer in cache.layers]).float().numpy()
    out["compact_values_out"] = torch.stack([layer.values for layer in cache.layers]).float().numpy()


def gen_eagle3_cases(eagle3, out: dict):
    g = torch.Generator().manual_seed(21)
    T, V = 9, 60
    # a small tree: root 0; 1,2 children of 0; 3,4 of 1; 5 of 2; 6 of 3; 7 of 6; 8 of 5
    parent = [-1, 0, 0, 1, 1, 2, 3, 6, 5]
    leaves = [i for i in range(T) if i not in parent]
    depth = [0] * T
    for i in range(1, T):
        depth[i] = depth[parent[i]] + 1
    W = max(depth) + 1
    retrieve = -np.ones((len(leaves), W), np.int64)
    for r, leaf in enumerate(leaves):
        cur = leaf
        for d in range(depth[leaf], -1, -1):
            retrieve[r, d] = cur
            cur = parent[cur]
    cases = []
    for c in range(6):
        draft = torch.randint(0, V, (1, T), generator=g)
        logits = torch.randn(1, T, V, generator=g)
        post = logits.argmax(-1)[0]
        # make some paths accepted: set posterior of parent to the child's token
        for i in range(1, T):
            if torch.rand(1, generator=g).item() < 0.6:
                logits[0, parent[i], draft[0, i]] += 50.0
        tm = torch.zeros(1, 1, T, T)
        for i in range(T):
            cur = i
            while cur >= 0:
                tm[0, 0, i, cur] = 1
                cur = parent[cur]
        best, alen, samp, cands, acc = eagle3.evaluate_eagle3_posterior(logits, draft, torch.from_numpy(retrieve),
                                                                         0.0)
        mask = eagle3.compile_eagle3_attention_mask(tm, past_length=5, dtype=torch.bfloat16,
                                                    device=torch.device("cpu"))
        cases.append(dict(logits=logits.numpy(), draft=draft.numpy(), best=best, alen=alen,
                          sample=int(samp.reshape(-1)[0]), cands=cands.numpy(), acc=np.asarray(acc),
                          mask=mask.float().numpy(), tree_mask=tm.numpy()))
        del post
    out["eagle3_retrieve"] = retrieve
    out["eagle3_parent"] = np.asarray(parent, np.int64)
    for i, c in enumerate(cases):
        for k, v in c.items():
            out[f"eagle3_{i}_{k}"] = np.asarray(v)


def gen_attention_cases(out: dict):
    """HF sdpa attention with the reference's dense tree mask (transformers
    integrations/sdpa_attention.py), small shapes, float32."""
    from transformers.integrations.sdpa_attention import sdpa_attention_forward

    class _M(torch.nn.Module):
        is_causal = False
        num_key_value_groups = 4

    for i, (past, n, hq, hkv, d) in enumerate([(37, 9, 8, 2, 128), (130, 33, 4, 1, 128), (0, 5, 4, 1, 128)]):
        q, k, v, vis, scale = tree_attention_inputs(seed=40 + i, past=past, n=n, hq=hq, hkv=hkv, d=d)
        mod = _M()
        mod.num_key_value_groups = hq // hkv
        mask = torch.zeros(1, 1, n, past + n)
        blk = torch.full((n, n), torch.finfo(torch.float32).min)
        blk.masked_fill_(torch.from_numpy(vis), 0)
        mask[0, 0, :, past:] = blk
        o, _ = sdpa_attention_forward(mod, torch.from_numpy(q).permute(1, 0, 2)[None],
                                      torch.from_numpy(k)[None], torch.from_numpy(v)[None], mask, dropout=0.0,
                                      scaling=scale)
        p = f"attn{i}_"
        out[p + "q"] = q
        out[p + "k"] = k
        out[p + "v"] = v
        out[p + "vis"] = vis
        out[p + "past"] = np.int64(past)
        out[p + "scale"] = np.float64(scale)
        out[p + "out"] = o[0].numpy()   # [N, Hq, D]


def main():
    ref_root = sys.argv[1] if len(sys.argv) > 1 else "/root/reference"
    ddtree, eagle3, mutils = _import_reference(ref_root)
    torch.set_num_threads(8)
    trees: dict = {}
    gen_tree_cases(ddtree, mutils, trees)
    np.savez_compressed(HERE / "trees.npz", **trees)
    misc: dict = {}
    gen_compile_cases(ddtree, misc)
    gen_compact_cases(ddtree, misc)
    gen_eagle3_cases(eagle3, misc)
    np.savez_compressed(HERE / "misc.npz", **misc)
    attn: dict = {}
    gen_attention_cases(attn)
    np.savez_compressed(HERE / "attention.npz", **attn)
    for f in ("trees.npz", "misc.npz", "attention.npz"):
        print(f, (HERE / f).stat().st_size, "bytes")


if __name__ == "__main__":
    main()
