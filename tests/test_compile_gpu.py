"""GPU parity of compile_ddtree_tree against the reference's own recorded
outputs (tests/golden/misc.npz, written by gen_golden.py's compile case).

The reference (ddtree.py:199-287) writes the verify ids, the positions
start + depth and the additive mask into caller buffers, after clearing the
previous tree's block (ddtree.py:230-231).  Here the mask rows come from the
mask-fill kernel (ddt_tree_mask_fill); every byte of the whole buffer is
compared, so the clear of the previous tree at [10, 17) is checked too.
"""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda", 0)


def _inputs(z):
    ids = torch.from_numpy(z["compile_node_token_ids"])
    depths = torch.from_numpy(z["compile_node_depths"])
    vis = torch.from_numpy(z["compile_visibility"])
    return ids, depths, vis


def _buffers(max_len=64, budget=12, dtype=torch.bfloat16):
    vi = torch.empty((1, 1 + budget), dtype=torch.long, device=DEV)
    vp = torch.empty((1, 1 + budget), dtype=torch.long, device=DEV)
    am = torch.zeros((1, 1, 1 + budget, max_len + 1 + budget), dtype=dtype, device=DEV)
    tv = torch.empty((1 + budget, 1 + budget), dtype=torch.bool, device=DEV)
    return vi, vp, am, tv


def test_compile_matches_reference_buffers(golden_misc):
    from ddtree_eagle3_patch_b200 import ddtree as D
    z = golden_misc
    ids, depths, vis = _inputs(z)
    vi, vp, am, tv = _buffers()
    # the reference's previous tree at [10, 17), rows 0..6, to be cleared first
    am[0, 0, :7, 10:17] = torch.finfo(torch.bfloat16).min
    r = D.compile_ddtree_tree(torch.tensor(777), 20, ids, depths, vis, 20, torch.bfloat16, DEV, vi, vp, am, tv, 10, 7)
    torch.cuda.synchronize()
    assert np.array_equal(r[0].cpu().numpy(), z["compile_ids"])
    assert np.array_equal(r[1].cpu().numpy(), z["compile_pos"])
    assert np.array_equal(r[2].float().cpu().numpy(), z["compile_mask"])
    assert np.array_equal(am.float().cpu().numpy(), z["compile_full_buffer"])
    assert r[3] == int(z["compile_past"]) and r[4] == int(z["compile_len"])
    # the packed bits the attention kernel reads agree with the dense mask
    bits = r[2].ddtree_bits.cpu().numpy().view(np.uint32)
    n = int(z["compile_len"])
    cols = np.arange(n)
    unpacked = ((bits[:, cols // 32] >> (cols % 32).astype(np.uint32)) & 1).astype(bool)
    assert np.array_equal(unpacked, z["compile_visibility"])


def test_compile_sliding_window_matches_reference(golden_misc):
    from ddtree_eagle3_patch_b200 import ddtree as D
    z = golden_misc
    ids, depths, vis = _inputs(z)
    vi, vp, am, tv = _buffers()
    sm = torch.zeros_like(am)
    r = D.compile_ddtree_tree(torch.tensor(777), 20, ids, depths, vis, 20, torch.bfloat16, DEV, vi, vp, am, tv, 0, 0,
                              sliding_window=8, sliding_attention_mask_buffer=sm)
    torch.cuda.synchronize()
    assert np.array_equal(r[2]["full_attention"].float().cpu().numpy(), z["compile_sw_full"])
    assert np.array_equal(r[2]["sliding_attention"].float().cpu().numpy(), z["compile_sw_sliding"])


def test_compile_repeated_rounds_clear_previous_tree(golden_misc):
    """Two rounds into one buffer: the second tree starts later and is
    smaller, so the first tree's block must be cleared (ddtree.py:230-231)
    and nothing else may change."""
    from ddtree_eagle3_patch_b200 import ddtree as D
    z = golden_misc
    ids, depths, vis = _inputs(z)
    vi, vp, am, tv = _buffers()
    r1 = D.compile_ddtree_tree(torch.tensor(5), 20, ids, depths, vis, 20, torch.bfloat16, DEV, vi, vp, am, tv, 0, 0)
    n1 = r1[4]
    keep = 5
    ids2, depths2 = ids[:keep], depths[:keep]
    vis2 = vis[: keep + 1, : keep + 1].clone()
    r2 = D.compile_ddtree_tree(torch.tensor(6), 23, ids2, depths2, vis2, 23, torch.bfloat16, DEV, vi, vp, am, tv,
                               20, n1)
    torch.cuda.synchronize()
    exp = torch.zeros_like(am, device="cpu", dtype=torch.float32)
    fmin = float(torch.finfo(torch.bfloat16).min)
    blk = np.where(vis2.numpy(), 0.0, fmin).astype(np.float32)
    exp[0, 0, : keep + 1, 23: 23 + keep + 1] = torch.from_numpy(blk)
    assert torch.equal(am.float().cpu(), exp)
    assert r2[1].cpu().tolist() == [[23] + (23 + depths2).tolist()]
