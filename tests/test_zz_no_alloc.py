"""ddt_tree_build_noalloc: the tree build for callers that cannot allocate.

Some callers cannot call cudaMalloc (a plugin handed only its inputs and
outputs, or an application whose device memory belongs to another
allocator).  The
no-alloc entry point runs the tree-build kernel with its scratch in a fixed
array inside the library instead of a caller workspace.  This test calls it
through the C ABI twice in a row and checks every output against the
regular entry point (ddt_tree_build with a workspace); the outputs are
integer trees and float32 log-probs from the same kernel, so they must be
identical.  This file sorts last so that a run stopping at the first failure
has run every other test before it.
"""
import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _outputs(rows, vocab, budget):
    from ddtree_eagle3_patch_b200.kernels import DeviceTree
    return DeviceTree.allocate(rows, vocab, budget, torch.device("cuda"))


def _host(t):
    n = int(t.info[0].item())
    return {
        "info": t.info.cpu().numpy(),
        "top_ids": t.top_ids.cpu().numpy(),
        "top_lp": t.top_lp.cpu().numpy().view(np.int32),
        "tokens": t.node_token_ids[:n].cpu().numpy(),
        "depths": t.node_depths[:n].cpu().numpy(),
        "parents": t.parents[: n + 1].cpu().numpy(),
        "bits": t.visibility[: n + 1].cpu().numpy(),
        "ids": t.verify_ids[: n + 1].cpu().numpy(),
        "pos": t.verify_pos[: n + 1].cpu().numpy(),
    }


def _call_regular(lib, logits, budget, root, start):
    rows, vocab = logits.shape
    out = _outputs(rows, vocab, budget)
    ws = torch.zeros(lib.ddt_tree_build_workspace_size(rows, vocab, budget), dtype=torch.uint8, device="cuda")
    o = out.c_outputs()
    rc = lib.ddt_tree_build(logits.data_ptr(), 0, rows, vocab, logits.stride(0), budget, root.data_ptr(), start,
                            ctypes.byref(o), ws.data_ptr(), ws.numel(), torch.cuda.current_stream().cuda_stream)
    assert rc == 0, lib.ddt_last_error()
    return out


def _call_noalloc(lib, logits, budget, root, start):
    rows, vocab = logits.shape
    out = _outputs(rows, vocab, budget)
    o = out.c_outputs()
    rc = lib.ddt_tree_build_noalloc(logits.data_ptr(), 0, rows, vocab, logits.stride(0), budget, root.data_ptr(),
                                    start, ctypes.byref(o), torch.cuda.current_stream().cuda_stream)
    assert rc == 0, lib.ddt_last_error()
    return out


def test_noalloc_matches_regular_entry_point_twice_in_a_row():
    from ddtree_eagle3_patch_b200 import _lib
    from ddtree_eagle3_patch_b200.synthetic import cfg1_logits
    lib = _lib.load()
    root = torch.tensor([7], dtype=torch.int64, device="cuda")
    cases = [(cfg1_logits(seed=0).cuda(), 64, 4096), (cfg1_logits(seed=5, peak=16.0).cuda(), 32, 100)]
    for logits, budget, start in cases:          # two calls in a row, different inputs
        got = _host(_call_noalloc(lib, logits, budget, root, start))
        torch.cuda.synchronize()
        want = _host(_call_regular(lib, logits, budget, root, start))
        for key in want:
            assert np.array_equal(got[key], want[key]), key
        assert got["info"][0] == budget and got["info"][2] == 0


def test_noalloc_rejects_shapes_beyond_its_scratch():
    from ddtree_eagle3_patch_b200 import _lib
    lib = _lib.load()
    rows, vocab, budget = 15, 151936, 1024
    out = _outputs(rows, vocab, budget)
    o = out.c_outputs()
    logits = torch.zeros((rows, vocab), device="cuda")
    rc = lib.ddt_tree_build_noalloc(logits.data_ptr(), 0, rows, vocab, vocab, budget, None, 0, ctypes.byref(o),
                                    torch.cuda.current_stream().cuda_stream)
    assert rc == 3
    assert b"scratch" in lib.ddt_last_error()
