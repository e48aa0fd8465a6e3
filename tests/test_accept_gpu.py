"""Kernel (3): greedy acceptance, EAGLE3 path acceptance and KV compaction."""
import numpy as np
import pytest
import torch

from oracle import oracle as O
from tests.golden_cases import regenerate_logits

pytestmark = pytest.mark.gpu


def _k():
    from ddtree_eagle3_patch_b200 import kernels
    return kernels


def _bf16_bits(x: torch.Tensor) -> np.ndarray:
    return x.contiguous().view(torch.int16).numpy().view(np.uint16)


@pytest.mark.parametrize("rows,V", [(65, 151936), (33, 151936), (1, 151936), (5, 1000), (3, 7), (130, 20000)])
def test_argmax_matches_oracle_with_ties_and_nan(rows, V):
    K = _k()
    g = torch.Generator().manual_seed(rows + V)
    x = torch.randn(rows, V, generator=g).to(torch.bfloat16)   # bf16 -> many ties
    if V > 10:
        x[0, 3] = 100.0
        x[0, V - 2] = 100.0                      # tie: first index wins
        if rows > 2:
            x[2, 7] = float("nan")               # NaN is the max
            x[2, 1] = float("nan")
            x[1, :] = -0.0
            x[1, 5] = 0.0                        # -0 == +0: first index wins
        if rows > 4:
            x[3, V // 2] = float("inf")          # +inf is the max
            x[3, V - 1] = float("inf")
            x[4, :] = float("-inf")              # all -inf: first index
    got = K.argmax_rows(x.cuda()).cpu().numpy()
    ref = O.argmax_rows(_bf16_bits(x))
    assert np.array_equal(got, ref)
    assert np.array_equal(got, torch.argmax(x.float(), dim=-1).numpy())


def test_argmax_fp32_and_fp16():
    K = _k()
    x = torch.randn(17, 50000)
    for dt in (torch.float32, torch.float16):
        xx = x.to(dt)
        assert torch.equal(K.argmax_rows(xx.cuda()).cpu(), torch.argmax(xx.float(), dim=-1))


def test_tree_accept_matches_reference_walk(golden_trees):
    """posterior fixture -> verify logits with that argmax -> fused accept =
    the reference's follow_verified_tree result."""
    from ddtree_eagle3_patch_b200.synthetic import verify_logits_for_posterior
    K = _k()
    z = golden_trees
    for p in ("cfg1_b32_", "cfg1_b64_", "deep_b64_", "deep_b128_"):
        x = torch.from_numpy(regenerate_logits(z, p)).cuda()
        tree = K.tree_build(x, int(z[p + "budget"]))
        logits = verify_logits_for_posterior(z[p + "posterior"], 151936, seed=3).cuda()
        acc, info, post = K.tree_accept(logits, tree.parents, tree.node_token_ids, tree.info)
        count = int(info[0])
        assert acc[:count].cpu().tolist() == z[p + "accepted"].tolist(), p
        assert int(info[1]) == int(z[p + "next_token"]), p
        assert np.array_equal(post.cpu().numpy(), z[p + "posterior"])


def test_tree_walk_and_dropin_follow(golden_trees):
    from ddtree_eagle3_patch_b200.ddtree import build_ddtree_tree, follow_verified_tree
    z = golden_trees
    for p in ("cfg1_b64_", "deep_b128_"):
        x = torch.from_numpy(regenerate_logits(z, p)).cuda()
        ids, depths, parents, child_maps, vis, _ = build_ddtree_tree(x, int(z[p + "budget"]))
        post = torch.from_numpy(z[p + "posterior"]).cuda()[None]
        acc, nxt = follow_verified_tree(child_maps, post)
        assert acc == z[p + "accepted"].tolist() and nxt == int(z[p + "next_token"])
        # plain list-of-dict child maps (no device tree attached)
        acc2, nxt2 = follow_verified_tree([dict(m) for m in child_maps], post)
        assert acc2 == acc and nxt2 == nxt


def test_random_trees_walk_vs_oracle():
    K = _k()
    rs = np.random.RandomState(0)
    for trial in range(20):
        x = torch.from_numpy((rs.randn(15, 3000) * 3).astype(np.float32))
        x[np.arange(15), rs.randint(0, 3000, 15)] += 15
        budget = int(rs.choice([8, 32, 64, 200]))
        tree = K.tree_build(x.cuda(), budget)
        n = int(tree.info[0])
        toks = tree.node_token_ids[:n].cpu().numpy()
        par = tree.parents[: n + 1].cpu().numpy()
        depth = np.concatenate([[0], tree.node_depths[:n].cpu().numpy()])
        top = tree.top_ids.cpu().numpy()
        post = np.where(rs.rand(n + 1) < 0.8, top[np.minimum(depth, 14), 0], rs.randint(0, 3000, n + 1))
        acc_o, nxt_o = O.follow(par, toks, post)
        acc, info = K.tree_walk(torch.from_numpy(post).cuda(), tree.parents, tree.node_token_ids, tree.info)
        assert acc[: int(info[0])].cpu().tolist() == acc_o and int(info[1]) == nxt_o


def test_eagle3_accept_matches_reference(golden_misc):
    from ddtree_eagle3_patch_b200.eagle3 import evaluate_eagle3_posterior
    z = golden_misc
    r = torch.from_numpy(z["eagle3_retrieve"])
    i = 0
    while f"eagle3_{i}_logits" in z.files:
        logits = torch.from_numpy(z[f"eagle3_{i}_logits"]).cuda()
        draft = torch.from_numpy(z[f"eagle3_{i}_draft"]).cuda()
        best, alen, samp, cands, acc = evaluate_eagle3_posterior(logits, draft, r, 0.0)
        assert best == int(z[f"eagle3_{i}_best"]) and alen == int(z[f"eagle3_{i}_alen"]), i
        assert int(samp.reshape(-1)[0]) == int(z[f"eagle3_{i}_sample"]), i
        assert samp.shape == (1, 1)
        assert acc == z[f"eagle3_{i}_acc"].tolist(), i
        assert np.array_equal(cands.cpu().numpy(), z[f"eagle3_{i}_cands"]), i
        i += 1


def test_eagle3_mask_matches_reference(golden_misc):
    from ddtree_eagle3_patch_b200.eagle3 import compile_eagle3_attention_mask
    z = golden_misc
    tm = torch.from_numpy(z["eagle3_0_tree_mask"])
    m = compile_eagle3_attention_mask(tm, 5, torch.bfloat16, torch.device("cuda"))
    assert np.array_equal(m.float().cpu().numpy(), z["eagle3_0_mask"])


def test_kv_compact_dynamic_cache_matches_reference(golden_misc):
    from transformers import DynamicCache

    from ddtree_eagle3_patch_b200.ddtree import compact_dynamic_cache
    z = golden_misc
    past = int(z["compact_past"])
    keep = z["compact_keep"].tolist()
    cache = DynamicCache()
    kin = torch.from_numpy(z["compact_keys_in"]).to(torch.bfloat16)
    vin = torch.from_numpy(z["compact_values_in"]).to(torch.bfloat16)
    for layer in range(kin.shape[0]):
        cache.update(kin[layer].cuda().clone(), vin[layer].cuda().clone(), layer)
    compact_dynamic_cache(cache, past, keep)
    kout = torch.stack([layer.keys for layer in cache.layers]).float().cpu().numpy()
    vout = torch.stack([layer.values for layer in cache.layers]).float().cpu().numpy()
    assert np.array_equal(kout, z["compact_keys_out"])
    assert np.array_equal(vout, z["compact_values_out"])


@pytest.mark.parametrize("keep", [[0, 3, 4, 9], [0], [0, 1, 2], list(range(12)), [5, 2, 7], [0, 11], [3, 3, 1]])
def test_compact_tail_inplace_vs_oracle(keep):
    from ddtree_eagle3_patch_b200.ddtree import compact_tail_inplace
    x = torch.randn(1, 8, 40 + 12, 128).to(torch.bfloat16)
    ref = O.compact_tail(x.float().numpy(), 40, keep)
    y = x.cuda()
    compact_tail_inplace(y, 40, torch.tensor(keep, dtype=torch.long, device="cuda"))
    assert np.array_equal(y.float().cpu().numpy(), ref)


def test_compact_tail_inplace_errors():
    from ddtree_eagle3_patch_b200.ddtree import compact_tail_inplace
    x = torch.randn(1, 2, 10, 16, device="cuda")
    with pytest.raises(RuntimeError, match="keep_count exceeds"):
        compact_tail_inplace(x, 8, torch.arange(5, device="cuda"))
    with pytest.raises(RuntimeError, match="past_length exceeds"):
        compact_tail_inplace(x, 11, torch.arange(1, device="cuda"))
    with pytest.raises(RuntimeError, match="dtype torch.long"):
        compact_tail_inplace(x, 4, torch.arange(2, device="cuda", dtype=torch.int32))


def test_kv_compact_many_layers_from_device_count():
    """The fused decode path: keep indices and count produced on the device
    by the accept kernel drive one compaction launch over 72 tensors."""
    K = _k()
    past, cur, L = 300, 65, 36
    ts = [torch.randn(8, past + cur, 128, device="cuda").to(torch.bfloat16) for _ in range(2 * L)]
    ref = [t.clone() for t in ts]
    keep = torch.tensor([0, 4, 17, 40, 41], device="cuda")
    count = torch.tensor([5], device="cuda")
    K.kv_compact(ts, past, cur, keep, count, 16)
    for t, r in zip(ts, ref):
        exp = r.clone()
        exp[:, past:past + 5] = r[:, past + keep.cpu()]
        assert torch.equal(t, exp)


def test_workspace_reuse_across_shapes():
    """Calls of different shapes share one workspace; counters must stay valid."""
    K = _k()
    for rows, V in [(3, 7), (130, 20000), (65, 151936), (2, 9), (4097, 300), (65, 151936)]:
        x = torch.randn(rows, V).to(torch.bfloat16)
        got = K.argmax_rows(x.cuda()).cpu()
        assert torch.equal(got, torch.argmax(x.float(), dim=-1)), (rows, V)


@pytest.mark.parametrize("width,dtype", [(5 * 2560, torch.bfloat16), (37, torch.bfloat16), (64, torch.float32)])
def test_commit_matches_oracle(width, dtype):
    """The commit step after a walk: tokens and bonus into output_ids, the
    accepted hidden rows, with the count read on the device (ddtree.py:534-548)."""
    K = _k()
    g = torch.Generator().manual_seed(width)
    x = torch.randn(15, 4096, generator=g)
    x[torch.arange(15), torch.randint(0, 4096, (15,), generator=g)] += 8
    tree = K.tree_build(x.cuda(), 32)
    n = int(tree.info[0])
    N = n + 1
    ids = tree.verify_ids[:N].clone()
    # a posterior that follows the tree for a few steps, then leaves it
    post = np.random.RandomState(width).randint(0, 4096, N).astype(np.int64)
    toks = tree.node_token_ids[:n].cpu().numpy()
    par = tree.parents[: n + 1].cpu().numpy()
    cur = 0
    for _ in range(3):
        kids = [i for i in range(1, n + 1) if par[i] == cur]
        if not kids:
            break
        post[cur] = toks[kids[0] - 1]
        cur = kids[0]
    acc, info = K.tree_walk(torch.from_numpy(post).cuda(), tree.parents, tree.node_token_ids, tree.info,
                            max_accept=N)
    count, nxt = int(info[0]), int(info[1])
    hidden = torch.randn(1, N, width, generator=g).to(dtype).cuda()
    out_ids = torch.full((1, 64), -1, dtype=torch.int64, device="cuda")
    sel = K.tree_commit(ids, acc, info, out_ids, 7, hidden)
    o_ids, o_sel = O.commit(ids.cpu().numpy(), acc[:count].cpu().numpy(), nxt, np.full((1, 64), -1, np.int64), 7,
                            hidden[0].float().cpu().numpy())
    assert np.array_equal(out_ids.cpu().numpy(), o_ids)
    assert torch.equal(sel[:count].float().cpu(), torch.from_numpy(o_sel))
    assert count >= 2
    # without hidden features, and with the output ending right after the tokens
    short = torch.full((7 + count,), -5, dtype=torch.int64, device="cuda")
    assert K.tree_commit(ids, acc, info, short, 7) is None
    assert short[7:].cpu().tolist() == o_ids[0, 7:7 + count].tolist()   # the bonus slot is past the end
