"""Sliding-window layers (the reference's ``sliding_attention`` mask of hybrid
models, ddtree.py:258-287): row t sees prefix key j only if
j >= position_t - window + 1, and the tree keys through the tree mask.

CPU: the oracle's per-row lower bound reproduces the reference's own sliding
mask (golden fixture), and the oracle attention with it equals attention with
that dense mask.  GPU: ``ddt_tree_attention_window`` against the oracle on
every kernel path (key splits with the transposed tail, the unsplit kernel,
several waves of splits), within the attention tests' bf16 tolerance."""
import numpy as np
import pytest
import torch

from oracle import oracle as O
from tests.test_attention_gpu import assert_close_bf16


def _dense_mask_attention(q, k, v, allowed, scale):
    q, k, v = (np.asarray(x, np.float64) for x in (q, k, v))
    N, Hq, D = q.shape
    g = Hq // k.shape[0]
    out = np.zeros((N, Hq, D))
    for h in range(Hq):
        s = q[:, h] @ k[h // g].T * scale
        s = np.where(allowed, s, -np.inf)
        p = np.exp(s - s.max(axis=1, keepdims=True))
        out[:, h] = (p / p.sum(axis=1, keepdims=True)) @ v[h // g]
    return out


def test_key_lo_reproduces_reference_sliding_mask(golden_misc):
    z = golden_misc
    past = int(z["compile_past"])
    sliding = z["compile_sw_sliding"][0, 0]
    lo = O.sliding_key_lo(z["compile_pos"].reshape(-1), 8)
    visible = sliding[:, :past] == 0
    assert past > 8 and (~visible).any() and visible.any()
    assert np.array_equal(visible, np.arange(past)[None, :] >= lo[:, None])
    # the tree block is the full-attention mask's
    assert np.array_equal(sliding[:, past:], z["compile_sw_full"][0, 0][:, past:])


def test_oracle_key_lo_equals_reference_dense_mask(golden_misc):
    z = golden_misc
    past = int(z["compile_past"])
    sliding = z["compile_sw_sliding"][0, 0]
    N = sliding.shape[0]
    rng = np.random.default_rng(4)
    q = rng.standard_normal((N, 4, 16))
    k = rng.standard_normal((2, past + N, 16))
    v = rng.standard_normal((2, past + N, 16))
    vis = z["compile_visibility"].astype(bool)
    lo = O.sliding_key_lo(z["compile_pos"].reshape(-1), 8)
    got = O.tree_attention_ref(q, k, v, past, vis, 0.25, key_lo=lo)
    ref = _dense_mask_attention(q, k, v, sliding == 0, 0.25)
    assert np.allclose(got, ref, rtol=1e-12, atol=1e-12)


def test_wrapper_bounds_from_reference_mask(golden_misc):
    """The HF attention function's bounds, counted from the reference's own
    sliding mask, are the clamped position - window + 1; a mask whose hidden
    prefix keys are not a leading block is refused."""
    from ddtree_eagle3_patch_b200.attention import _mask_key_lo
    z = golden_misc
    past = int(z["compile_past"])
    mask = torch.from_numpy(z["compile_sw_sliding"]).to(torch.bfloat16)
    N = mask.shape[-2]
    lo = _mask_key_lo(mask, N, past + N).numpy()
    expect = np.clip(O.sliding_key_lo(z["compile_pos"].reshape(-1), 8), 0, past)
    assert np.array_equal(lo, expect)
    holed = mask.clone()
    row = int(np.argmax(expect > 1))
    holed[0, 0, row, 0] = 0.0      # key 0 visible again, after hidden keys
    with pytest.raises(ValueError):
        _mask_key_lo(holed, N, past + N)


def _inputs(past, n, hq, hkv, seed):
    from ddtree_eagle3_patch_b200.synthetic import tree_attention_inputs
    q, k, v, vis, scale = tree_attention_inputs(seed=seed, past=past, n=n, hq=hq, hkv=hkv, d=128)
    depth = vis.sum(axis=1).astype(np.int64) - 1      # a row sees itself and its ancestors
    return q, k, v, vis, scale, past + depth


def _run_window(q, k, v, past, vis, scale, key_lo):
    from ddtree_eagle3_patch_b200 import kernels as K
    bits = torch.from_numpy(O.pack_visibility(vis).view(np.int32)).cuda()
    qb = torch.from_numpy(q).to(torch.bfloat16).cuda()
    kb = torch.from_numpy(k).to(torch.bfloat16).cuda()
    vb = torch.from_numpy(v).to(torch.bfloat16).cuda()
    lo = torch.from_numpy(np.asarray(key_lo, np.int64)).cuda()
    out = K.tree_attention(qb, kb, vb, past, bits, scale, key_lo=lo)
    torch.cuda.synchronize()
    assert K.attention_status(qb.device) == 0
    ref = O.tree_attention_ref(qb.float().cpu().numpy(), kb.float().cpu().numpy(), vb.float().cpu().numpy(), past,
                               vis, scale, key_lo=key_lo)
    return out.float().cpu().numpy(), ref


@pytest.mark.gpu
@pytest.mark.parametrize("past,n,hq,hkv,window", [
    (4096, 65, 32, 8, 1000),    # verify shape: key splits, 4-row transposed tail
    (4096, 65, 32, 8, 8),       # window inside the tree depth: almost no prefix
    (4096, 65, 32, 8, 4200),    # window wider than the sequence: no restriction
    (4096, 4, 32, 8, 2000),     # tail pass only
    (900, 97, 32, 8, 450),      # M-tile pair, then one M tile + tail
    (1000, 9, 32, 2, 300),      # group 16: one M tile + 16-row tail
    (20000, 65, 32, 8, 5000),   # several waves of key splits
    (64, 600, 32, 8, 40),       # many M tiles: unsplit kernel
    (100, 131, 8, 8, 30),       # no GQA: 3-row tail
])
def test_window_vs_float64(past, n, hq, hkv, window):
    q, k, v, vis, scale, pos = _inputs(past, n, hq, hkv, seed=past + n + window)
    out, ref = _run_window(q, k, v, past, vis, scale, O.sliding_key_lo(pos, window))
    assert np.isfinite(out).all()
    assert_close_bf16(out, ref, (past, n, hq, hkv, window))


@pytest.mark.gpu
@pytest.mark.parametrize("past,n", [(4096, 65), (64, 600), (1000, 9)])
def test_window_per_row_bounds_and_clamping(past, n):
    """Arbitrary per-row bounds: below 0, above past (no prefix at all), and
    on 32- and 128-key boundaries."""
    hkv = 2 if n == 9 else 8
    q, k, v, vis, scale, _ = _inputs(past, n, 32, hkv, seed=11 + n)
    rng = np.random.default_rng(n)
    lo = rng.integers(-300, past + 300, size=n)
    lo[:: 5] = (lo[:: 5] // 128) * 128
    lo[1:: 7] = (lo[1:: 7] // 32) * 32
    lo[2] = past + 10
    lo[3] = -5
    out, ref = _run_window(q, k, v, past, vis, scale, lo)
    assert np.isfinite(out).all()
    assert_close_bf16(out, ref, (past, n))


@pytest.mark.gpu
def test_hf_sliding_layer_through_attention_function():
    """A sliding-window layer through the AttentionInterface function, with the
    mask from ``ddtree.compile_ddtree_tree`` (bounds attached) and with the
    same mask as a plain tensor (bounds counted from it), against fp32 SDPA
    with the dense mask."""
    from ddtree_eagle3_patch_b200 import ddtree
    from ddtree_eagle3_patch_b200.attention import tree_verify_attention
    from ddtree_eagle3_patch_b200.synthetic import tree_attention_inputs
    past, n, hq, hkv, window, start = 1500, 33, 32, 8, 700, 1500
    q, k, v, vis, scale = tree_attention_inputs(seed=8, past=past, n=n, hq=hq, hkv=hkv, d=128)
    depths = torch.from_numpy(vis.sum(axis=1)[1:].astype(np.int64) - 1)
    dev = torch.device("cuda")
    cap = past + n + 8
    bufs = (torch.zeros(1, cap, dtype=torch.long, device=dev), torch.zeros(1, cap, dtype=torch.long, device=dev),
            torch.zeros(1, 1, cap, cap, dtype=torch.bfloat16, device=dev),
            torch.zeros(cap, cap, dtype=torch.bool, device=dev))
    smask_buf = torch.zeros(1, 1, cap, cap, dtype=torch.bfloat16, device=dev)
    node_ids = torch.arange(1, n, dtype=torch.long)
    _, pos, masks, _, _ = ddtree.compile_ddtree_tree(
        5, start, node_ids.to(dev), depths.to(dev), torch.from_numpy(vis), past, torch.bfloat16, dev, *bufs, 0, 0,
        sliding_window=window, sliding_attention_mask_buffer=smask_buf)
    smask = masks["sliding_attention"]
    query = torch.from_numpy(q).to(torch.bfloat16).cuda().permute(1, 0, 2)[None]
    key = torch.from_numpy(k).to(torch.bfloat16).cuda()[None]
    value = torch.from_numpy(v).to(torch.bfloat16).cuda()[None]

    class M:
        training = False
        num_key_value_groups = hq // hkv
    ref = torch.nn.functional.scaled_dot_product_attention(
        query.float(), key.float().repeat_interleave(hq // hkv, 1), value.float().repeat_interleave(hq // hkv, 1),
        attn_mask=smask.float(), scale=scale).transpose(1, 2)
    assert (smask[0, 0, :, :past] != 0).any()     # the window hides some prefix keys
    for m in (smask, smask.clone()):
        out, _ = tree_verify_attention(M(), query, key, value, m, scaling=scale, sliding_window=window)
        assert_close_bf16(out.float().cpu().numpy(), ref.cpu().numpy())
    # causal call of a sliding layer (no mask): row t at position past + t
    qp = torch.randn(1, hq, 70, 128, device=dev).to(torch.bfloat16)
    kp = torch.randn(1, hkv, 300, 128, device=dev).to(torch.bfloat16)
    vp = torch.randn(1, hkv, 300, 128, device=dev).to(torch.bfloat16)
    o2, _ = tree_verify_attention(M(), qp, kp, vp, None, scaling=scale, sliding_window=64)
    qi = torch.arange(230, 300, device=dev)[:, None]
    kj = torch.arange(300, device=dev)[None, :]
    allowed = (kj <= qi) & (kj >= qi - 63)
    ref2 = torch.nn.functional.scaled_dot_product_attention(
        qp.float(), kp.float().repeat_interleave(hq // hkv, 1), vp.float().repeat_interleave(hq // hkv, 1),
        attn_mask=allowed, scale=scale).transpose(1, 2)
    assert_close_bf16(o2.float().cpu().numpy(), ref2.cpu().numpy())
