"""Kernel (1), tree build, against the oracle and the reference's own outputs."""
import numpy as np
import pytest
import torch

from oracle import oracle as O
from tests.golden_cases import regenerate_logits, tree_prefixes

pytestmark = pytest.mark.gpu


def _kernels():
    from ddtree_eagle3_patch_b200 import kernels
    return kernels


def _tree_np(tree):
    n = int(tree.info[0].item())
    return dict(
        n=n,
        node_token_ids=tree.node_token_ids[:n].cpu().numpy(),
        node_depths=tree.node_depths[:n].cpu().numpy(),
        parents=tree.parents[: n + 1].cpu().numpy(),
        bits=tree.visibility[: n + 1].cpu().numpy().view(np.uint32),
        verify_ids=tree.verify_ids[: n + 1].cpu().numpy(),
        verify_pos=tree.verify_pos[: n + 1].cpu().numpy(),
        info=tree.info.cpu().numpy(),
    )


def _assert_tree_equal(got, ref_tokens, ref_depths, ref_parents, ref_vis, msg=""):
    n = len(ref_tokens)
    assert got["n"] == n, msg
    assert np.array_equal(got["node_token_ids"], ref_tokens), msg
    assert np.array_equal(got["node_depths"], ref_depths), msg
    assert np.array_equal(got["parents"], np.asarray(ref_parents, np.int32)), msg
    W = got["bits"].shape[1]
    assert np.array_equal(got["bits"], O.pack_visibility(np.asarray(ref_vis, bool), W)), msg


def test_expansion_from_reference_log_probs_is_bit_exact(golden_trees):
    """Same (lp, ids) in -> the reference's tree out, for every fixture."""
    K = _kernels()
    z = golden_trees
    for p in tree_prefixes(z):
        b = int(z[p + "budget"])
        if p + "lp" not in z.files:
            continue
        lp = torch.from_numpy(z[p + "lp"]).cuda()
        ids = torch.from_numpy(z[p + "ids"]).cuda()
        root = torch.tensor([12345], dtype=torch.int64, device="cuda")
        t = K.tree_from_log_probs(lp, ids, b, root_token=root, start=100)
        g = _tree_np(t)
        _assert_tree_equal(g, z[p + "node_token_ids"], z[p + "node_depths"], z[p + "parents"], z[p + "visibility"], p)
        assert g["verify_ids"][0] == 12345
        assert np.array_equal(g["verify_ids"][1:], z[p + "node_token_ids"])
        assert np.array_equal(g["verify_pos"], np.concatenate([[100], 100 + z[p + "node_depths"]]))


def test_full_build_matches_oracle_and_reference(golden_trees):
    """Logits in: top-k ids equal the oracle's (value desc, id asc), log-probs
    within 1 ulp, tree bit-exact to the oracle fed the kernel's own lp/ids and
    to the reference wherever torch's top-k order is defined (no value ties)."""
    K = _kernels()
    z = golden_trees
    for p in tree_prefixes(z):
        b = int(z[p + "budget"])
        x = regenerate_logits(z, p) if (p + "logits" in z.files or p + "logits_sha256" in z.files) else None
        if x is None or b <= 0 or x.shape[0] == 0:
            continue
        t = K.tree_build(torch.from_numpy(np.ascontiguousarray(x)).cuda(), b)
        g = _tree_np(t)
        k = min(b, x.shape[1])
        ids_g = t.top_ids[:, :k].cpu().numpy()
        lp_g = t.top_lp[:, :k].cpu().numpy()
        o_ids, o_vals, o_logz = O.topk_logz(x, k)
        assert np.array_equal(ids_g, o_ids), p
        o_lp = O.log_probs(o_vals, o_logz)
        # lp = top - log_z: the kernel's log-normaliser may differ from the
        # float64-accumulated one by an ulp of log_z (torch's own does too)
        tol = 2 * np.spacing(np.abs(o_logz))[:, None] + np.spacing(np.abs(o_lp))
        assert np.all(np.abs(lp_g - o_lp) <= tol), (p, np.abs(lp_g - o_lp).max())
        o = O.tree_from_lp(lp_g, ids_g, b)
        _assert_tree_equal(g, o["node_token_ids"], o["node_depths"], o["parents"], o["visibility"], p)
        if np.array_equal(ids_g, z[p + "ids"]) and np.array_equal(lp_g, z[p + "lp"]):
            _assert_tree_equal(g, z[p + "node_token_ids"], z[p + "node_depths"], z[p + "parents"],
                               z[p + "visibility"], p)


def test_configuration_1_trees_equal_reference(golden_trees):
    K = _kernels()
    z = golden_trees
    for p in ("cfg1_b32_", "cfg1_b64_", "deep_b64_", "deep_b128_"):
        x = torch.from_numpy(regenerate_logits(z, p)).cuda()
        t = K.tree_build(x, int(z[p + "budget"]))
        g = _tree_np(t)
        _assert_tree_equal(g, z[p + "node_token_ids"], z[p + "node_depths"], z[p + "parents"], z[p + "visibility"], p)
        assert g["info"][2] == 0


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_half_precision_logits(dtype):
    K = _kernels()
    g = torch.Generator().manual_seed(7)
    x = (torch.randn(15, 151936, generator=g) * 3).to(dtype)
    t = K.tree_build(x.cuda(), 64)
    xf = x.float().numpy()
    o = O.build_tree(xf, 64)
    gt = _tree_np(t)
    assert np.array_equal(t.top_ids.cpu().numpy(), o["ids"])
    lp = t.top_lp.cpu().numpy()
    o2 = O.tree_from_lp(lp, o["ids"], 64)
    _assert_tree_equal(gt, o2["node_token_ids"], o2["node_depths"], o2["parents"], o2["visibility"])


@pytest.mark.parametrize("L,V,budget", [(15, 151936, 1), (15, 151936, 256), (15, 151936, 1024), (1, 151936, 64),
                                        (32, 50000, 128), (4, 5, 40), (2, 3, 10), (15, 2049, 64), (7, 16384, 300)])
def test_shapes_and_budgets(L, V, budget):
    K = _kernels()
    g = torch.Generator().manual_seed(L * 1000 + budget)
    x = torch.randn(L, V, generator=g) * 2
    if L > 2:
        x[torch.arange(L), torch.randint(0, V, (L,), generator=g)] += 12
    t = K.tree_build(x.cuda(), budget)
    gt = _tree_np(t)
    o = O.build_tree(x.numpy(), budget)
    k = min(budget, V)
    assert np.array_equal(t.top_ids[:, :k].cpu().numpy(), o["ids"])
    o2 = O.tree_from_lp(t.top_lp[:, :k].cpu().numpy(), o["ids"], budget)
    _assert_tree_equal(gt, o2["node_token_ids"], o2["node_depths"], o2["parents"], o2["visibility"], (L, V, budget))


def _frontier_before_last_pop(o, rows, topk):
    """Frontier size when the last node is popped: each popped node adds its
    next sibling (rank + 1 < topk) and its first child (depth < rows) and
    leaves itself."""
    f = 1
    for d, r in zip(o["node_depths"][:-1], o["node_ranks"][:-1]):
        f += int(r + 1 < topk) + int(d < rows) - 1
    return f


@pytest.mark.parametrize("budget", [32, 64, 96, 128])
def test_register_frontier_full_at_last_pop(budget):
    """Flat draft logits make a broad tree in which every pop but the last
    grows the frontier by one, so the frontier holds exactly ``budget`` entries
    (every register slot) when the last node is popped."""
    K = _kernels()
    L, V = 32, 4096
    g = torch.Generator().manual_seed(7 + budget)
    x = torch.randn(L, V, generator=g) * 0.05
    t = K.tree_build(x.cuda(), budget)
    o = O.build_tree(x.numpy(), budget)
    assert _frontier_before_last_pop(o, L, min(budget, V)) == budget
    assert np.array_equal(t.top_ids[:, :budget].cpu().numpy(), o["ids"])
    o2 = O.tree_from_lp(t.top_lp[:, :budget].cpu().numpy(), o["ids"], budget)
    _assert_tree_equal(_tree_np(t), o2["node_token_ids"], o2["node_depths"], o2["parents"], o2["visibility"],
                       budget)


def test_value_ties_break_by_lowest_token_id():
    K = _kernels()
    x = torch.zeros(3, 5000)
    x[:, ::7] = 1.0           # many equal maxima
    x[1, 4999] = 2.0
    t = K.tree_build(x.cuda(), 16)
    ids = t.top_ids.cpu().numpy()
    assert ids[0].tolist() == list(range(0, 7 * 16, 7))
    assert ids[1, 0] == 4999 and ids[1, 1:].tolist() == list(range(0, 7 * 15, 7))


def test_root_only_tree():
    K = _kernels()
    root = torch.tensor([42], dtype=torch.int64, device="cuda")
    t = K.tree_build(torch.randn(15, 100, device="cuda"), 0, root_token=root, start=9)
    assert int(t.info[0]) == 0
    assert int(t.parents[0]) == -1
    assert int(t.verify_ids[0]) == 42 and int(t.verify_pos[0]) == 9
    assert int(t.visibility[0, 0]) == 1


def test_nonfinite_logits_are_flagged():
    K = _kernels()
    x = torch.randn(4, 1000)
    x[2, 5] = float("nan")
    t = K.tree_build(x.cuda(), 8)
    assert int(t.info[2]) & 1
    # the flag is per call: a clean call afterwards reports nothing
    t2 = K.tree_build(torch.randn(4, 1000).cuda(), 8)
    assert int(t2.info[2]) == 0


def test_repeated_calls_reuse_workspace():
    K = _kernels()
    x = torch.from_numpy(O.np.random.RandomState(0).randn(15, 151936).astype(np.float32)).cuda()
    a = _tree_np(K.tree_build(x, 64))
    for _ in range(3):
        b = _tree_np(K.tree_build(x, 64))
        assert np.array_equal(a["parents"], b["parents"]) and np.array_equal(a["node_token_ids"], b["node_token_ids"])


def test_dropin_build_ddtree_tree_matches_reference(golden_trees):
    from ddtree_eagle3_patch_b200.ddtree import build_ddtree_tree
    z = golden_trees
    for p in ("cfg1_b32_", "cfg1_b64_", "deep_b64_"):
        x = torch.from_numpy(regenerate_logits(z, p)).cuda()
        ids, depths, parents, child_maps, vis, sub = build_ddtree_tree(x, int(z[p + "budget"]))
        assert ids.device.type == "cpu" and ids.dtype == torch.long
        assert np.array_equal(ids.numpy(), z[p + "node_token_ids"])
        assert np.array_equal(depths.numpy(), z[p + "node_depths"])
        assert parents == z[p + "parents"].tolist()
        assert np.array_equal(vis.numpy(), z[p + "visibility"])
        assert isinstance(child_maps, list) and len(child_maps) == len(parents)
        for i in range(1, len(parents)):
            assert child_maps[parents[i]][int(ids[i - 1])] == i
        assert set(sub) == {"tree_build_copy", "tree_build_heap", "tree_build_visibility"}
    out = build_ddtree_tree(torch.randn(15, 100, device="cuda"), 0)
    assert out[2] == [-1] and out[4].shape == (1, 1)


def test_candidate_overflow_rows_match_oracle():
    """Rows built to defeat the chunk pre-filter, so each of the kernel's
    candidate paths runs (9 chunks of 16888 at this width, 512 threads x
    16-byte vectors; thread t of warp t // 32 holds chunk-local positions
    with (position // 4) % 512 == t):
    - rows 0-2: warp 15's slots at -100 and large values in thread 0's
      slots, so the lower bound falls to -100 and most of the chunk is a
      candidate (the radix select over the whole chunk);
    - rows 3-6: warp 15's slots scaled down, so about 8 % of the chunk is a
      candidate (the radix select over the candidates);
    - rows 7-9: large values in thread 0's slots over a normal base (the
      ranked candidates);
    - rows 10-11: exact ties; rows 12-14: a fifth of the entries at the max."""
    K = _kernels()
    L, V, budget = 15, 151936, 64
    rs = np.random.RandomState(11)
    x = rs.randn(L, V).astype(np.float32)
    local = np.arange(V) % 16888
    thread = (local // 4) % 512
    first = thread == 0
    x[0:3] = np.where(first, 8.0 + rs.rand(3, V), np.where(thread >= 480, -100.0, x[0:3]))
    x[3:7] = np.where(thread >= 480, 0.6 * x[3:7], x[3:7])
    x[7:10] = np.where(first, 8.0 + rs.rand(3, V), x[7:10])
    x[10:12] = 0.5
    x[10:12, rs.randint(0, V, 40)] = 3.0
    for r in range(12, 15):
        x[r, rs.rand(V) < 0.2] = x[r].max()
    x = x.astype(np.float32)
    t = K.tree_build(torch.from_numpy(x).cuda(), budget)
    g = _tree_np(t)
    k = min(budget, V)
    ids_g = t.top_ids[:, :k].cpu().numpy()
    lp_g = t.top_lp[:, :k].cpu().numpy()
    o_ids, o_vals, o_logz = O.topk_logz(x, k)
    assert np.array_equal(ids_g, o_ids)
    o_lp = O.log_probs(o_vals, o_logz)
    tol = 2 * np.spacing(np.abs(o_logz))[:, None] + np.spacing(np.abs(o_lp))
    assert np.all(np.abs(lp_g - o_lp) <= tol), np.abs(lp_g - o_lp).max()
    o = O.tree_from_lp(lp_g, ids_g, budget)
    _assert_tree_equal(g, o["node_token_ids"], o["node_depths"], o["parents"], o["visibility"], "overflow")


def _random_table(rng, kind, L, V):
    if kind == 0:      # continuous values
        return rng.standard_normal((L, V)).astype(np.float32)
    if kind == 1:      # values on a coarse grid: many exact ties
        return (np.round(rng.standard_normal((L, V)) * 8) / 8).astype(np.float32)
    if kind == 2:      # one confident token per row
        x = rng.standard_normal((L, V)).astype(np.float32)
        x[np.arange(L), rng.integers(0, V, L)] += rng.uniform(2, 20)
        return x
    return rng.integers(0, 3, (L, V)).astype(np.float32)   # three values only


@pytest.mark.parametrize("kind", [0, 1, 2, 3])
def test_expansion_random_tables_match_oracle(kind):
    """The expansion (parallel for budget <= 64 and <= 16 rows, else the
    serial loop, which also takes over when a check fails) on random
    log-prob tables: continuous, tied on a coarse grid, peaked, and
    three-valued, at random depths, budgets and widths."""
    K = _kernels()
    rng = np.random.default_rng(100 + kind)
    for trial in range(50):
        L = int(rng.integers(1, 17))
        B = int(rng.integers(1, 80))
        V = int(rng.integers(2, 3000))
        k = min(B, V)
        ids, vals, logz = O.topk_logz(_random_table(rng, kind, L, V), k)
        lp = O.log_probs(vals, logz)
        ref = O.tree_from_lp(lp, ids, B)
        tree = K.tree_from_log_probs(torch.from_numpy(lp).cuda(), torch.from_numpy(ids).cuda(), B)
        got = _tree_np(tree)
        _assert_tree_equal(got, ref["node_token_ids"], ref["node_depths"], ref["parents"], ref["visibility"],
                           msg=(kind, trial, L, B, V))


def test_full_build_bf16_ties_match_oracle():
    """bf16 draft logits at the vocabulary width (many exact value ties in
    every row's top-k) through the whole kernel, budgets 8 / 32 / 64."""
    K = _kernels()
    g = torch.Generator().manual_seed(7)
    for budget in (8, 32, 64):
        for peak in (0.0, 6.0, 16.0):
            x = torch.randn(15, 151936, generator=g)
            x[torch.arange(15), torch.randint(0, 151936, (15,), generator=g)] += peak
            x = x.to(torch.bfloat16)
            ref = O.build_tree(x.float().numpy(), budget)
            got = _tree_np(K.tree_build(x.cuda(), budget))
            _assert_tree_equal(got, ref["node_token_ids"], ref["node_depths"], ref["parents"], ref["visibility"],
                               msg=(budget, peak))
