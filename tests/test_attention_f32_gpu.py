"""Float32 tree attention (ddt_tree_attention_f32) against the float64 oracle.

Tolerance (float32 in and out): max |out - ref| <= 1e-5 * max |ref|, the
float32 bound of the verify attention's contract."""
import numpy as np
import pytest
import torch

from oracle import oracle as O

pytestmark = pytest.mark.gpu

RTOL = 1e-5


def _k():
    from ddtree_eagle3_patch_b200 import kernels
    return kernels


def _close(out, ref, msg=""):
    err = np.abs(np.asarray(out, np.float64) - ref).max()
    assert err <= RTOL * np.abs(ref).max(), (msg, err, np.abs(ref).max())


def _run(seed, past, n, hq, hkv, key_lo=None, strided=False):
    from ddtree_eagle3_patch_b200.synthetic import tree_attention_inputs
    q, k, v, vis, scale = tree_attention_inputs(seed=seed, past=past, n=n, hq=hq, hkv=hkv, d=128)
    K = _k()
    dev = torch.device("cuda", 0)
    bits = torch.from_numpy(O.pack_visibility(vis).view(np.int32)).to(dev)
    qt = torch.from_numpy(q).to(dev)
    if strided:   # HF layout: q is the [T, Hq, D] transpose of [Hq, T, D]; K/V rows of a larger cache
        qt = qt.transpose(0, 1).contiguous().transpose(0, 1)
        kc = torch.zeros((hkv, past + n + 40, 128), dtype=torch.float32, device=dev)
        vc = torch.zeros_like(kc)
        kc[:, : past + n] = torch.from_numpy(k).to(dev)
        vc[:, : past + n] = torch.from_numpy(v).to(dev)
        kt, vt = kc, vc
    else:
        kt, vt = torch.from_numpy(k).to(dev), torch.from_numpy(v).to(dev)
    lo_t = None if key_lo is None else torch.from_numpy(np.asarray(key_lo, np.int64)).to(dev)
    out = K.tree_attention(qt, kt, vt, past, bits, scale, key_lo=lo_t)
    ref = O.tree_attention_ref(q.astype(np.float64), k.astype(np.float64), v.astype(np.float64), past, vis, scale,
                               key_lo=key_lo)
    return out.cpu().numpy(), ref


@pytest.mark.parametrize("past,n,hq,hkv", [
    (4096, 65, 32, 8),
    (1536, 33, 32, 8),
    (0, 1, 32, 8),
    (1, 1, 4, 2),
    (127, 2, 32, 8),
    (300, 17, 8, 2),
    (0, 96, 4, 2),       # prefill-like: no prefix, many rows
    (513, 33, 16, 16),   # no grouping
    (200, 9, 32, 2),     # group 16
])
def test_f32_matches_float64_oracle(past, n, hq, hkv):
    out, ref = _run(seed=past + n, past=past, n=n, hq=hq, hkv=hkv)
    _close(out, ref, (past, n, hq, hkv))


def test_f32_strided_cache_and_queries():
    out, ref = _run(seed=3, past=777, n=33, hq=32, hkv=8, strided=True)
    _close(out, ref)


def test_f32_sliding_window_bounds():
    past, n = 400, 33
    rng = np.random.default_rng(0)
    key_lo = rng.integers(-50, past + 50, size=n)
    out, ref = _run(seed=5, past=past, n=n, hq=8, hkv=2, key_lo=key_lo)
    _close(out, ref)


def test_f32_device_past_length():
    """A run-time prefix length read from the device gives the same output as
    the host value, and values past the bound are clamped to it."""
    from ddtree_eagle3_patch_b200.synthetic import tree_attention_inputs
    K = _k()
    dev = torch.device("cuda", 0)
    past, n = 250, 17
    q, k, v, vis, scale = tree_attention_inputs(seed=9, past=past, n=n, hq=8, hkv=2, d=128)
    bits = torch.from_numpy(O.pack_visibility(vis).view(np.int32)).to(dev)
    qt, kt, vt = (torch.from_numpy(x).to(dev) for x in (q, k, v))
    host = K.tree_attention_f32(qt, kt, vt, past, bits, scale)
    pd = torch.tensor([past], dtype=torch.int32, device=dev)
    devp = K.tree_attention_f32(qt, kt, vt, past, bits, scale, past_dev=pd)
    assert torch.equal(host, devp)
    # a smaller run-time prefix over the same buffers equals the host call with it
    pd.fill_(100)
    small = K.tree_attention_f32(qt, kt, vt, past, bits, scale, past_dev=pd)
    ref_small = K.tree_attention_f32(qt, kt, vt, 100, bits, scale)
    assert torch.equal(small, ref_small)
    pd.fill_(10 ** 6)   # clamped to the bound
    assert torch.equal(K.tree_attention_f32(qt, kt, vt, past, bits, scale, past_dev=pd), host)
