"""The draft head fused with the tree build's first step (ddt_wgemm_head +
ddt_tree_build_head) against the head GEMM and the tree build on the
logits: same logits, exact block statistics, same top-k and tree."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _kernels():
    from ddtree_eagle3_patch_b200 import kernels
    return kernels


def _ord_keys(vals: np.ndarray, ids: np.ndarray) -> np.ndarray:
    """The library's top-k keys: ordered fp32 bits, then ~id (larger key =
    larger value, then lower id)."""
    u = vals.astype(np.float32).view(np.uint32).astype(np.uint64)
    neg = (u & 0x80000000) != 0
    o = np.where(neg, (~u) & 0xFFFFFFFF, u | 0x80000000)
    return (o << np.uint64(32)) | (np.uint64(0xFFFFFFFF) - ids.astype(np.uint64))


def _designed(values: torch.Tensor, K: int = 64):
    """x, w with x @ w.T == values exactly: x[t] = e_t, w[:, t] = values[t]
    (bf16 values, one nonzero product per output)."""
    T, V = values.shape
    assert T <= K
    x = torch.zeros((T, K), dtype=torch.bfloat16, device="cuda")
    x[torch.arange(T), torch.arange(T)] = 1
    w = torch.zeros((V, K), dtype=torch.bfloat16, device="cuda")
    w[:, :T] = values.t().to(torch.bfloat16)
    return x, w


def _split_stats(stats: torch.Tensor, T: int, V: int):
    nblk = V // 128
    n = T * nblk
    s_off = (4 * n + 255) // 256 * 256
    k_off = s_off + (4 * n + 255) // 256 * 256
    raw = stats.cpu().numpy()
    m = raw[:4 * n].view(np.float32).reshape(T, nblk)
    s = raw[s_off:s_off + 4 * n].view(np.float32).reshape(T, nblk)
    keys = raw[k_off:k_off + 8 * n].view(np.uint64).reshape(T, nblk)
    return m, s, keys


@pytest.mark.parametrize("T,V,K", [(15, 151936, 2560), (16, 4096, 256), (1, 1024, 64), (33, 2048, 128)])
def test_head_logits_and_block_statistics(T, V, K):
    kern = _kernels()
    g = torch.Generator(device="cuda").manual_seed(T * 7 + V)
    x = torch.randn((T, K), device="cuda", generator=g).to(torch.bfloat16)
    w = (torch.randn((V, K), device="cuda", generator=g) * 0.05).to(torch.bfloat16)
    stats = kern.head_stats_buffer(T, V, x.device)
    y = kern.wgemm_head(x, w, stats)
    torch.cuda.synchronize()
    assert torch.equal(y, kern.wgemm(x, w, splits=1)), "logits differ from the plain GEMM"
    m, s, keys = _split_stats(stats, T, V)
    yb = y.float().cpu().numpy().reshape(T, V // 128, 128)
    assert np.array_equal(m, yb.max(axis=2))
    ref_s = np.exp(yb.astype(np.float64) - yb.max(axis=2, keepdims=True)).sum(axis=2)
    np.testing.assert_allclose(s, ref_s, rtol=2e-6)
    ids = np.arange(V, dtype=np.int64).reshape(V // 128, 128)
    all_keys = _ord_keys(yb, np.broadcast_to(ids, yb.shape))
    assert np.array_equal(keys, all_keys.max(axis=2))


def _build_both(values: torch.Tensor, budget: int):
    kern = _kernels()
    T, V = values.shape
    x, w = _designed(values)
    stats = kern.head_stats_buffer(T, V, x.device)
    logits = kern.wgemm_head(x, w, stats)
    assert torch.equal(logits, values.to(torch.bfloat16))
    root = torch.tensor([7], dtype=torch.int64, device="cuda")
    plain = kern.tree_build(logits, budget, root_token=root, start=100)
    plain_ids, plain_info = plain.top_ids.clone(), plain.info.clone()
    fused = kern.tree_build(logits, budget, root_token=root, start=100, head_stats=stats)
    # the expansion alone on the fused path's own top-k: the same tree
    again = kern.tree_from_log_probs(fused.top_lp, fused.top_ids, budget, root_token=root, start=100)
    torch.cuda.synchronize()
    return logits, (plain_ids, plain_info), fused, again


def _check_same(logits, plain, fused, again):
    """Top-k ids equal to the tree build on the logits; lp within 2 ulp of
    v - log-sum-exp computed in float64 (the tolerance of the tree build's
    own tests); the tree is the expansion of that top-k."""
    plain_ids, plain_info = plain
    assert torch.equal(plain_ids, fused.top_ids), "top-k ids differ"
    v = logits.float().cpu().numpy().astype(np.float64)
    mx = v.max(axis=1, keepdims=True)
    logz = (mx + np.log(np.exp(v - mx).sum(axis=1, keepdims=True))).astype(np.float32)
    ids = fused.top_ids.cpu().numpy()
    top_v = np.take_along_axis(v, ids, axis=1).astype(np.float32)
    lp_ref = top_v - logz
    lp = fused.top_lp.cpu().numpy()
    assert np.all(np.abs(lp - lp_ref) <= 2 * np.spacing(np.abs(logz) + np.abs(lp_ref))), "lp off by > 2 ulp"
    n = int(fused.info[0].item())
    assert n == int(again.info[0].item()) == int(plain_info[0].item())
    assert torch.equal(fused.node_token_ids[:n], again.node_token_ids[:n])
    assert torch.equal(fused.parents[: n + 1], again.parents[: n + 1])
    assert torch.equal(fused.visibility[: n + 1], again.visibility[: n + 1])
    assert torch.equal(fused.verify_ids[: n + 1], again.verify_ids[: n + 1])
    assert int(fused.info[2].item()) == int(plain_info[2].item()) == 0


@pytest.mark.parametrize("budget", [32, 64])
def test_random_logits_same_top_k_and_tree(budget):
    g = torch.Generator(device="cuda").manual_seed(budget)
    values = (torch.randn((15, 151936), device="cuda", generator=g) * 3).to(torch.bfloat16)
    _check_same(*_build_both(values, budget))


def test_top_values_clustered_in_one_block():
    # every row's 64 largest logits sit in one 128-row block: its listed
    # 8 keys all rank, so the block is read again from the logits
    g = torch.Generator(device="cuda").manual_seed(3)
    values = torch.randn((15, 151936), device="cuda", generator=g)
    for t in range(15):
        b = 37 * (t + 1)
        values[t, b * 128: b * 128 + 64] = 10 + torch.rand(64, device="cuda", generator=g)
    _check_same(*_build_both(values.to(torch.bfloat16), 64))


def test_equal_logits_break_ties_by_lowest_id():
    values = torch.zeros((4, 8192), device="cuda", dtype=torch.bfloat16)
    _check_same(*_build_both(values, 32))


@pytest.mark.parametrize("V,budget", [(1024, 64), (128, 32), (2048, 80), (151936, 80)])
def test_small_vocabularies_and_wide_budgets(V, budget):
    g = torch.Generator(device="cuda").manual_seed(V + budget)
    values = torch.randn((15, V), device="cuda", generator=g).to(torch.bfloat16)
    _check_same(*_build_both(values, budget))


def test_budgets_beyond_the_limit_are_rejected():
    kern = _kernels()
    from ddtree_eagle3_patch_b200._lib import DDTreeError
    values = torch.zeros((15, 151936), device="cuda", dtype=torch.bfloat16)
    x, w = _designed(values)
    stats = kern.head_stats_buffer(15, 151936, x.device)
    logits = kern.wgemm_head(x, w, stats)
    with pytest.raises(DDTreeError):
        kern.tree_build(logits, 96, head_stats=stats)


def test_repeated_calls_reuse_the_statistics_buffer():
    kern = _kernels()
    g = torch.Generator(device="cuda").manual_seed(9)
    for _ in range(3):
        values = torch.randn((15, 16384), device="cuda", generator=g).to(torch.bfloat16)
        _check_same(*_build_both(values, 32))
    assert kern.wgemm_status(torch.device("cuda")) == 0
