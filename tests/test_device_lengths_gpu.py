"""Kernels that read their lengths from device memory, so that one captured
launch serves every decode round: the tree attention with a run-time prefix
(ddt_tree_attention_dev) and the KV append at a device-side row offset
(ddt_kv_append)."""
import numpy as np
import pytest
import torch

from oracle import oracle as O

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda", 0)


def _k():
    from ddtree_eagle3_patch_b200 import kernels
    return kernels


def _inputs(seed, cap, n, hq, hkv):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(n, hq, 128, generator=g).to(torch.bfloat16).to(DEV)
    k = (torch.randn(hkv, cap, 128, generator=g) / np.sqrt(128)).to(torch.bfloat16).to(DEV)
    v = torch.randn(hkv, cap, 128, generator=g).to(torch.bfloat16).to(DEV)
    from ddtree_eagle3_patch_b200.synthetic import random_tree
    _, _, vis = random_tree(n - 1, max_depth=16, seed=seed)
    bits = torch.from_numpy(O.pack_visibility(vis).view(np.int32)).to(DEV)
    return q, k, v, vis, bits


@pytest.mark.parametrize("n,hq,hkv", [(33, 32, 8), (16, 32, 8), (65, 32, 8), (17, 8, 2)])
def test_device_past_equals_host_past(n, hq, hkv):
    """Same bytes as the host-length call for run-time prefixes across the
    planned range, including ones that leave most split CTAs idle; the K/V
    rows past the tree hold finite data that must not leak in."""
    K = _k()
    past_max = 1536
    cap = past_max + n
    q, k, v, vis, bits = _inputs(7, cap, n, hq, hkv)
    ws = K.attention_workspace(n, hq, hkv, past_max, DEV)
    pd = torch.zeros((1,), dtype=torch.int32, device=DEV)
    for past in (0, 1, 127, 128, 513, 1000, past_max):
        # the tree's K/V rows sit at [past, past + n) of the same buffers
        kk = k.clone()
        vv = v.clone()
        pd.fill_(past)
        dev_out = K.tree_attention(q, kk, vv, past_max, bits, 128 ** -0.5, past_dev=pd, workspace=ws)
        host_out = K.tree_attention(q, kk[:, : past + n], vv[:, : past + n], past, bits, 128 ** -0.5)
        torch.cuda.synchronize()
        assert K.attention_status(DEV, ws) == 0
        if not torch.equal(dev_out, host_out):
            ref = O.tree_attention_ref(q.float().cpu().numpy(), kk[:, : past + n].float().cpu().numpy(),
                                       vv[:, : past + n].float().cpu().numpy(), past, vis, 128 ** -0.5)
            err = np.abs(dev_out.float().cpu().numpy() - ref).max()
            assert err <= 2e-2 * np.abs(ref).max(), (past, err)


def test_device_past_captured_once_replayed_for_many_prefixes():
    K = _k()
    n, hq, hkv, past_max = 33, 32, 8, 1200
    cap = past_max + n
    q, k, v, vis, bits = _inputs(11, cap, n, hq, hkv)
    ws = K.attention_workspace(n, hq, hkv, past_max, DEV)
    pd = torch.full((1,), 600, dtype=torch.int32, device=DEV)
    out = torch.empty((n, hq, 128), dtype=torch.bfloat16, device=DEV)
    K.tree_attention(q, k, v, past_max, bits, 128 ** -0.5, out=out, past_dev=pd, workspace=ws)   # warm
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        K.tree_attention(q, k, v, past_max, bits, 128 ** -0.5, out=out, past_dev=pd, workspace=ws)
    for past in (5, 300, 1199, 1200):
        pd.fill_(past)
        g.replay()
        ref = K.tree_attention(q, k[:, : past + n], v[:, : past + n], past, bits, 128 ** -0.5)
        torch.cuda.synchronize()
        exp = O.tree_attention_ref(q.float().cpu().numpy(), k[:, : past + n].float().cpu().numpy(),
                                   v[:, : past + n].float().cpu().numpy(), past, vis, 128 ** -0.5)
        err = np.abs(out.float().cpu().numpy() - exp).max()
        assert err <= 2e-2 * np.abs(exp).max(), (past, err)
        assert torch.equal(out, ref) or np.abs(out.float().cpu().numpy() - ref.float().cpu().numpy()).max() \
            <= 2e-2 * np.abs(exp).max()
    assert K.attention_status(DEV, ws) == 0
    del g


def test_device_past_rejects_shapes_beyond_the_split_kernel():
    from ddtree_eagle3_patch_b200._lib import DDTreeError
    K = _k()
    n, hq, hkv = 2048, 32, 8   # 64 M tiles x 8 KV heads: the unsplit kernel's shape
    q = torch.zeros((n, hq, 128), dtype=torch.bfloat16, device=DEV)
    k = torch.zeros((hkv, n + 64, 128), dtype=torch.bfloat16, device=DEV)
    bits = torch.zeros((n, n // 32), dtype=torch.int32, device=DEV)
    pd = torch.zeros((1,), dtype=torch.int32, device=DEV)
    with pytest.raises(DDTreeError, match="split kernel"):
        K.tree_attention(q, k, k, 64, bits, 0.1, past_dev=pd, workspace=K.attention_workspace(n, hq, hkv, 64, DEV))


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_kv_append_at_device_offset(dtype):
    K = _k()
    hkv, cap, rows = 8, 300, 33
    dst_k = torch.zeros((1, hkv, cap, 128), dtype=dtype, device=DEV)
    dst_v = torch.zeros_like(dst_k)
    src = torch.randn((1, hkv, rows + 7, 128), dtype=torch.float32, device=DEV).to(dtype)
    src_k, src_v = src[:, :, :rows], src[:, :, 7:]            # strided row windows of one tensor
    off = torch.tensor([123], dtype=torch.int32, device=DEV)
    K.kv_append(src_k, src_v, dst_k, dst_v, off)
    exp_k = torch.zeros_like(dst_k)
    exp_v = torch.zeros_like(dst_v)
    exp_k[:, :, 123:123 + rows] = src_k
    exp_v[:, :, 123:123 + rows] = src_v
    assert torch.equal(dst_k, exp_k) and torch.equal(dst_v, exp_v)
    # a device row count shorter than the source, and an offset near the end
    # whose overflow rows are skipped
    cnt = torch.tensor([5], dtype=torch.int32, device=DEV)
    off.fill_(cap - 3)
    K.kv_append(src_k, src_v, dst_k, dst_v, off, cnt)
    exp_k[:, :, cap - 3:] = src_k[:, :, :3]
    exp_v[:, :, cap - 3:] = src_v[:, :, :3]
    assert torch.equal(dst_k, exp_k) and torch.equal(dst_v, exp_v)
    off.fill_(-10)   # wholly outside: nothing written
    K.kv_append(src_k, src_v, dst_k, dst_v, off, cnt)
    assert torch.equal(dst_k, exp_k)
