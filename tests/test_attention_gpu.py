"""Kernel (2), tree-masked verify attention, against float64 / fp32 references.

Tolerance (bf16 inputs and output): max |out - ref| <= 2e-2 * max |ref| and
elementwise |out - ref| <= 2e-2 * |ref| + 2e-2 * rms(ref)."""
import numpy as np
import pytest
import torch

from oracle import oracle as O

pytestmark = pytest.mark.gpu

RTOL = 2e-2


def _k():
    from ddtree_eagle3_patch_b200 import kernels
    return kernels


def assert_close_bf16(out, ref, msg=""):
    out = np.asarray(out, np.float64)
    ref = np.asarray(ref, np.float64)
    scale = np.abs(ref).max()
    rms = np.sqrt((ref ** 2).mean())
    err = np.abs(out - ref)
    assert err.max() <= RTOL * scale + 1e-6, (msg, err.max(), scale)
    assert np.all(err <= RTOL * np.abs(ref) + RTOL * rms), (msg, (err - RTOL * np.abs(ref)).max(), rms)


def _run(q, k, v, past, vis, scale):
    K = _k()
    bits = torch.from_numpy(O.pack_visibility(vis).view(np.int32)).cuda()
    qb = torch.from_numpy(q).to(torch.bfloat16).cuda()
    kb = torch.from_numpy(k).to(torch.bfloat16).cuda()
    vb = torch.from_numpy(v).to(torch.bfloat16).cuda()
    out = K.tree_attention(qb, kb, vb, past, bits, scale)
    torch.cuda.synchronize()
    assert K.attention_status(qb.device) == 0
    ref = O.tree_attention_ref(qb.float().cpu().numpy(), kb.float().cpu().numpy(), vb.float().cpu().numpy(), past,
                               vis, scale)
    return out.float().cpu().numpy(), ref


def test_matches_hf_sdpa_fixtures(golden_attention):
    z = golden_attention
    for i in range(3):
        p = f"attn{i}_"
        out, ref = _run(z[p + "q"], z[p + "k"], z[p + "v"], int(z[p + "past"]), z[p + "vis"], float(z[p + "scale"]))
        assert_close_bf16(out, ref, p)
        assert_close_bf16(out, z[p + "out"], p + "hf")


@pytest.mark.parametrize("past,n,hq,hkv", [
    (4096, 65, 32, 8),      # verify attention at Qwen3-4B shape
    (4096, 33, 32, 8),
    (1536, 33, 32, 8),
    (0, 1, 32, 8),
    (1, 1, 32, 8),
    (127, 2, 32, 8),
    (128, 65, 32, 8),
    (300, 129, 32, 8),
    (50, 17, 8, 8),         # no GQA
    (50, 17, 16, 2),        # group 8
    (700, 40, 4, 2),        # group 2
    (2500, 65, 32, 8),
    (4096, 4, 32, 8),       # 16 rows: tail pass only
    (4096, 5, 32, 8),       # 20 rows: one padded M tile
    (900, 97, 32, 8),       # 388 rows: an M-tile pair, then one M tile + tail
    (1000, 9, 32, 2),       # group 16: one M tile + 16-row tail
    (20000, 65, 32, 8),     # long context: several waves of key splits
    (64, 600, 32, 8),       # many M tiles: unsplit kernel
    (100, 131, 8, 8),       # no GQA: 3-row tail (three tokens)
    (200, 65, 16, 8),       # group 2: 2-row tail
])
def test_random_trees_vs_float64(past, n, hq, hkv):
    from ddtree_eagle3_patch_b200.synthetic import tree_attention_inputs
    q, k, v, vis, scale = tree_attention_inputs(seed=past + n, past=past, n=n, hq=hq, hkv=hkv, d=128)
    out, ref = _run(q, k, v, past, vis, scale)
    assert_close_bf16(out, ref, (past, n, hq, hkv))


def test_strided_hf_layouts():
    """q as the transposed view HF passes ([T, Hq, D] out of [Hq, T, D]) and K/V
    inside a larger preallocated cache (kv_rows > past + n)."""
    from ddtree_eagle3_patch_b200.synthetic import tree_attention_inputs
    K = _k()
    past, n, hq, hkv = 1000, 65, 32, 8
    q, k, v, vis, scale = tree_attention_inputs(seed=5, past=past, n=n, hq=hq, hkv=hkv, d=128)
    q_hf = torch.from_numpy(q).to(torch.bfloat16).cuda().transpose(0, 1).contiguous().transpose(0, 1)  # strided
    cap = past + n + 300
    kc = torch.zeros(hkv, cap, 128, dtype=torch.bfloat16, device="cuda")
    vc = torch.zeros_like(kc)
    kc[:, : past + n] = torch.from_numpy(k).to(torch.bfloat16).cuda()
    vc[:, : past + n] = torch.from_numpy(v).to(torch.bfloat16).cuda()
    kc[:, past + n:] = 50.0    # rows past the tree must not be read
    vc[:, past + n:] = float("nan")
    bits = torch.from_numpy(O.pack_visibility(vis).view(np.int32)).cuda()
    out = K.tree_attention(q_hf, kc, vc, past, bits, scale)
    ref = O.tree_attention_ref(q_hf.float().cpu().numpy(), kc[:, : past + n].float().cpu().numpy(),
                               vc[:, : past + n].float().cpu().numpy(), past, vis, scale)
    assert_close_bf16(out.float().cpu().numpy(), ref)


def test_against_torch_sdpa_fp32_reference_path():
    """The reference's own math path (repeat_kv + SDPA with the additive
    float mask) in fp32 on the GPU, at the verify-attention shape."""
    from ddtree_eagle3_patch_b200.synthetic import tree_attention_inputs
    K = _k()
    past, n, hq, hkv = 4096, 65, 32, 8
    q, k, v, vis, scale = tree_attention_inputs(seed=11, past=past, n=n, hq=hq, hkv=hkv, d=128)
    qb = torch.from_numpy(q).to(torch.bfloat16).cuda()
    kb = torch.from_numpy(k).to(torch.bfloat16).cuda()
    vb = torch.from_numpy(v).to(torch.bfloat16).cuda()
    mask = torch.zeros(n, past + n, device="cuda")
    blk = torch.full((n, n), torch.finfo(torch.float32).min, device="cuda")
    blk.masked_fill_(torch.from_numpy(vis).cuda(), 0)
    mask[:, past:] = blk
    g = hq // hkv
    ref = torch.nn.functional.scaled_dot_product_attention(
        qb.float().transpose(0, 1)[None], kb.float().repeat_interleave(g, 0)[None],
        vb.float().repeat_interleave(g, 0)[None], attn_mask=mask[None, None], scale=scale)[0].transpose(0, 1)
    bits = torch.from_numpy(O.pack_visibility(vis).view(np.int32)).cuda()
    out = K.tree_attention(qb, kb, vb, past, bits, scale)
    assert_close_bf16(out.float().cpu().numpy(), ref.cpu().numpy())


def test_hf_attention_function_with_dense_mask():
    """The AttentionInterface function reduces the reference's dense mask to bits."""
    from ddtree_eagle3_patch_b200.attention import tree_verify_attention
    from ddtree_eagle3_patch_b200.synthetic import tree_attention_inputs
    past, n, hq, hkv = 777, 33, 32, 8
    q, k, v, vis, scale = tree_attention_inputs(seed=3, past=past, n=n, hq=hq, hkv=hkv, d=128)
    mask = torch.zeros(1, 1, n, past + n, dtype=torch.bfloat16)
    blk = torch.full((n, n), torch.finfo(torch.bfloat16).min, dtype=torch.bfloat16)
    blk.masked_fill_(torch.from_numpy(vis), 0)
    mask[0, 0, :, past:] = blk
    query = torch.from_numpy(q).to(torch.bfloat16).cuda().permute(1, 0, 2)[None]
    key = torch.from_numpy(k).to(torch.bfloat16).cuda()[None]
    value = torch.from_numpy(v).to(torch.bfloat16).cuda()[None]

    class M:
        training = False
        num_key_value_groups = hq // hkv
    out, w = tree_verify_attention(M(), query, key, value, mask.cuda(), scaling=scale)
    assert w is None and out.shape == (1, n, hq, 128)
    ref = O.tree_attention_ref(query[0].transpose(0, 1).float().cpu().numpy(), key[0].float().cpu().numpy(),
                               value[0].float().cpu().numpy(), past, vis, scale)
    assert_close_bf16(out[0].float().cpu().numpy(), ref)
    # causal (no mask): prefill of 70 tokens
    qp = torch.randn(1, hq, 70, 128, device="cuda").to(torch.bfloat16)
    kp = torch.randn(1, hkv, 70, 128, device="cuda").to(torch.bfloat16)
    vp = torch.randn(1, hkv, 70, 128, device="cuda").to(torch.bfloat16)
    o2, _ = tree_verify_attention(M(), qp, kp, vp, None, scaling=scale)
    ref2 = torch.nn.functional.scaled_dot_product_attention(qp.float(), kp.float().repeat_interleave(4, 1),
                                                            vp.float().repeat_interleave(4, 1), is_causal=True,
                                                            scale=scale).transpose(1, 2)
    assert_close_bf16(o2.float().cpu().numpy(), ref2.cpu().numpy())


def test_fully_masked_split_rows_are_finite():
    """A key split can hold only tree keys a row does not see; its partial
    must carry zero weight (no NaN)."""
    from ddtree_eagle3_patch_b200.synthetic import tree_attention_inputs
    past, n = 4200, 129   # tree spans key tiles 32 and 33
    q, k, v, vis, scale = tree_attention_inputs(seed=1, past=past, n=n, hq=32, hkv=8, d=128)
    out, ref = _run(q, k, v, past, vis, scale)
    assert np.isfinite(out).all()
    assert_close_bf16(out, ref)


@pytest.mark.parametrize("past,n", [(4096, 65), (64, 600)])
def test_row_max_jump_between_key_tiles(past, n):
    """One key in a second key tile scores far above everything before it, for
    the rows of one query head per KV group only: those rows' running max
    grows by more than 2^8 and O is rescaled, while the other rows of the
    same warps keep theirs (split kernel, then the unsplit kernel)."""
    from ddtree_eagle3_patch_b200.synthetic import tree_attention_inputs
    hq, hkv = 32, 8
    q, k, v, vis, scale = tree_attention_inputs(seed=21 + n, past=past, n=n, hq=hq, hkv=hkv, d=128)
    key = 150                       # key tile 1 of the first split
    k[:, key, :] = 0.0
    k[:, key, 0] = 16.0
    q[:, :, 0] = 0.0
    q[:, ::hq // hkv, 0] = 10.0     # head 0 of each group: score 160 * scale on that key
    out, ref = _run(q, k, v, past, vis, scale)
    assert np.isfinite(out).all()
    assert_close_bf16(out, ref, (past, n))
