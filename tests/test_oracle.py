"""The CPU oracle against the reference's own outputs (golden fixtures)."""
import numpy as np
import pytest

from oracle import oracle as O
from tests.golden_cases import regenerate_logits, same_up_to_value_ties, tree_prefixes


def test_heap_matches_reference_on_reference_log_probs(golden_trees):
    """Best-first expansion from the reference's own (lp, ids) is bit-exact."""
    z = golden_trees
    for p in tree_prefixes(z):
        b = int(z[p + "budget"])
        if p + "lp" in z.files:
            t = O.tree_from_lp(z[p + "lp"], z[p + "ids"], b)
        else:
            t = O.tree_from_lp(np.zeros((0, 1), np.float32), np.zeros((0, 1), np.int64), b)
        assert np.array_equal(t["node_token_ids"], z[p + "node_token_ids"]), p
        assert np.array_equal(t["node_depths"], z[p + "node_depths"]), p
        assert np.array_equal(t["parents"], z[p + "parents"]), p
        assert np.array_equal(t["visibility"], z[p + "visibility"]), p


def test_topk_and_log_probs_match_reference(golden_trees):
    """Top-k ids equal (up to the order of equal values, which torch leaves
    undefined) and log-probs within 2 ulp of torch's fp32 logsumexp."""
    z = golden_trees
    for p in tree_prefixes(z):
        b = int(z[p + "budget"])
        if p + "lp" not in z.files:
            continue
        x = regenerate_logits(z, p)
        o = O.build_tree(x, b)
        assert same_up_to_value_ties(o["top_vals"], o["ids"], z[p + "top_vals"], z[p + "ids"]), p
        ulp = np.abs(o["logz"].view(np.int32).astype(np.int64) - z[p + "logz"].view(np.int32).astype(np.int64))
        assert ulp.max() <= 2, (p, ulp.max())
        if np.array_equal(o["ids"], z[p + "ids"]) and np.array_equal(o["lp"], z[p + "lp"]):
            assert np.array_equal(o["node_token_ids"], z[p + "node_token_ids"]), p
            assert np.array_equal(o["parents"], z[p + "parents"]), p


def test_full_size_trees_match_reference(golden_trees):
    """Configuration-1 and deep-tree inputs: the whole build from logits gives
    the reference's tree."""
    z = golden_trees
    for p in ("cfg1_b32_", "cfg1_b64_", "deep_b64_", "deep_b128_"):
        x = regenerate_logits(z, p)
        o = O.build_tree(x, int(z[p + "budget"]))
        assert np.array_equal(o["ids"], z[p + "ids"]), p
        assert np.array_equal(o["node_token_ids"], z[p + "node_token_ids"]), p
        assert np.array_equal(o["node_depths"], z[p + "node_depths"]), p
        assert np.array_equal(o["parents"], z[p + "parents"]), p


def test_follow_matches_reference(golden_trees):
    z = golden_trees
    for p in ("cfg1_b32_", "cfg1_b64_", "deep_b64_", "deep_b128_"):
        acc, nxt = O.follow(z[p + "parents"], z[p + "node_token_ids"], z[p + "posterior"])
        assert acc == z[p + "accepted"].tolist(), p
        assert nxt == int(z[p + "next_token"]), p


def test_deep_trees_are_deep(golden_trees):
    z = golden_trees
    assert z["deep_b64_node_depths"].max() == 15
    assert len(z["deep_b128_accepted"]) > 3


def test_compile_matches_reference(golden_misc):
    z = golden_misc
    ids, pos, mask = O.compile_tree(777, 20, z["compile_node_token_ids"], z["compile_node_depths"],
                                    z["compile_visibility"], int(z["compile_past"]), -3.3895313892515355e38)
    assert np.array_equal(ids, z["compile_ids"][0])
    assert np.array_equal(pos, z["compile_pos"][0])
    assert np.array_equal(mask, z["compile_mask"][0, 0])


def test_compact_matches_reference(golden_misc):
    z = golden_misc
    past = int(z["compact_past"])
    keep = z["compact_keep"]
    for name in ("keys", "values"):
        got = O.compact_tail(z[f"compact_{name}_in"], past, keep)[..., : past + len(keep), :]
        assert np.array_equal(got, z[f"compact_{name}_out"]), name


def test_eagle3_posterior_matches_reference(golden_misc):
    z = golden_misc
    r = z["eagle3_retrieve"]
    i = 0
    while f"eagle3_{i}_logits" in z.files:
        logits = z[f"eagle3_{i}_logits"][0]
        post = O.argmax_rows(logits)
        best, alen, samp, acc = O.eagle3_posterior(post, z[f"eagle3_{i}_draft"], r)
        assert best == int(z[f"eagle3_{i}_best"]), i
        assert alen == int(z[f"eagle3_{i}_alen"]), i
        assert samp == int(z[f"eagle3_{i}_sample"]), i
        assert acc == z[f"eagle3_{i}_acc"].tolist(), i
        i += 1
    assert i >= 6


def test_attention_reference_matches_hf_sdpa(golden_attention):
    z = golden_attention
    for i in range(3):
        p = f"attn{i}_"
        o = O.tree_attention_ref(z[p + "q"], z[p + "k"], z[p + "v"], int(z[p + "past"]), z[p + "vis"],
                                 float(z[p + "scale"]))
        np.testing.assert_allclose(o, z[p + "out"], rtol=1e-5, atol=1e-5)


def test_pack_unpack_visibility_roundtrip():
    rs = np.random.RandomState(0)
    for n in (1, 5, 32, 33, 65, 130):
        vis = rs.rand(n, n) < 0.3
        assert np.array_equal(O.unpack_visibility(O.pack_visibility(vis), n), vis)


def test_argmax_first_max_and_nan():
    x = np.array([[1.0, 3.0, 3.0, 2.0], [np.nan, 5.0, np.nan, 1.0], [0.0, 0.0, 0.0, 0.0]], np.float32)
    assert O.argmax_rows(x).tolist() == [1, 0, 0]
    b = (x.view(np.uint32) >> 16).astype(np.uint16)
    assert O.argmax_rows(b).tolist() == [1, 0, 0]


@pytest.mark.parametrize("budget", [0, 1, 7])
def test_small_budgets_root_only_or_chain(budget):
    x = np.random.RandomState(1).randn(4, 20).astype(np.float32)
    o = O.build_tree(x, budget)
    assert len(o["node_token_ids"]) == max(budget, 0)
    assert o["parents"][0] == -1
