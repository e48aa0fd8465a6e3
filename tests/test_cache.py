"""The preallocated in-place-append cache (a drop-in for DynamicCache at the
verify boundary): the same views as DynamicCache's torch.cat appends, and
compaction through the same kernel path."""
import pytest
import torch
from transformers.cache_utils import DynamicCache

from ddtree_eagle3_patch_b200.cache import TreeAppendCache


def _fill(caches, layers, steps, device, seed=0, crop_after=None, crop_to=None):
    g = torch.Generator().manual_seed(seed)
    for step, T in enumerate(steps):
        for layer in range(layers):
            k = torch.randn(1, 2, T, 8, generator=g).to(device)
            v = torch.randn(1, 2, T, 8, generator=g).to(device)
            outs = [c.update(k, v, layer) for c in caches]
            for kk, vv in outs[1:]:
                assert torch.equal(kk, outs[0][0]) and torch.equal(vv, outs[0][1])
        if crop_after is not None and step == crop_after:
            for c in caches:
                c.crop(crop_to)


def test_append_crop_and_growth_match_dynamic_cache():
    a, d = TreeAppendCache(capacity=8, num_layers=3), DynamicCache()
    _fill([d, a], 3, [5, 3, 6], "cpu", crop_after=1, crop_to=6)   # 12 rows: the buffers grow once
    assert a.get_seq_length() == d.get_seq_length() == 12
    b = TreeAppendCache(capacity=64)            # layers added as they are reached
    _fill([DynamicCache(), b], 2, [4, 4], "cpu")
    assert len(b.layers) == 2 and b.get_seq_length() == 8


@pytest.mark.gpu
def test_compaction_matches_dynamic_cache():
    from ddtree_eagle3_patch_b200.ddtree import compact_dynamic_cache
    a, d = TreeAppendCache(capacity=64, num_layers=4), DynamicCache()
    _fill([d, a], 4, [20, 9], "cuda")           # past 20, then a 9-row tree window
    keep = [0, 3, 4, 8]
    compact_dynamic_cache(d, 20, keep)
    compact_dynamic_cache(a, 20, keep)
    assert a.get_seq_length() == d.get_seq_length() == 24
    for la, ld in zip(a.layers, d.layers):
        assert torch.equal(la.keys, ld.keys) and torch.equal(la.values, ld.values)
    # the next round appends after the compacted rows, in place
    _fill([d, a], 4, [9], "cuda", seed=1)
    assert a.get_seq_length() == 33
