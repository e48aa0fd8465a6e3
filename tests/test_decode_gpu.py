"""End-to-end decode parity: this package's ``ddtree_generate`` on the GPU
against the reference's own ``ddtree_generate`` run on CPU
(tests/golden/decode.npz, written by gen_decode_golden.py).

The models are the float32 seeded tiny models of ``decode_case``.  The
fixtures were kept only where every decision of the reference run has a
margin of at least 2e-4 (target argmax on the accepted path, draft top-k,
heap order), so the ~1e-6 float32 differences between the CPU reference and
the GPU path cannot change a decision: the emitted ids, the acceptance
length of every round, and every round's tree (parents, tokens, depths)
and accepted indices must be identical.
"""
import sys
from pathlib import Path

import numpy as np
import pytest
import torch

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE / "golden"))

import decode_case as C  # noqa: E402

DEV = torch.device("cuda", 0)


def _models(name, z):
    from transformers import Qwen3ForCausalLM
    from ddtree_eagle3_patch_b200.model import DFlashDraftModel
    _, vocab, block, budget, plen, max_new = next(c for c in C.CASES if c[0] == name)
    p = name + "_"
    seed = int(z[p + "seed"])
    torch.manual_seed(0)
    tgt = Qwen3ForCausalLM(C.target_config(vocab)).eval()
    assert C.seeded_init(tgt, seed) == str(z[p + "sha_target"])
    drf = DFlashDraftModel(C.draft_config(vocab, block, vocab - 1)).eval()
    assert C.seeded_init(drf, seed + 1000) == str(z[p + "sha_draft"])
    return tgt, drf, vocab, block, budget, plen, max_new


@pytest.fixture(scope="module")
def decode_golden():
    return np.load(HERE / "golden" / "decode.npz")


def test_fixture_models_rebuild_on_cpu(decode_golden):
    """The seeded models (weights hashed) and prompts rebuild exactly."""
    for name, vocab, block, budget, plen, max_new in C.CASES:
        _models(name, decode_golden)
        p = name + "_"
        assert np.array_equal(C.prompt(int(decode_golden[p + "seed"]), plen, vocab, vocab - 1).numpy(),
                              decode_golden[p + "prompt"])


MODES = {  # DDTREE_EAGER, DDTREE_FUSED, DDTREE_PACK
    "graphs": ("0", "1", "1"),            # the default: captured forwards, fused layers, packed weights
    "eager": ("1", "1", "1"),             # every round eager
    "graphs_unfused": ("0", "0", "1"),    # captured forwards over the stock layers
    "graphs_unpacked": ("0", "1", "0"),   # fused layers with one GEMM per projection
}


@pytest.mark.gpu
@pytest.mark.parametrize("mode", list(MODES))
@pytest.mark.parametrize("name", [c[0] for c in C.CASES])
def test_ddtree_generate_matches_reference(name, mode, decode_golden, monkeypatch):
    """Every loop form: captured draft/verify forwards replayed from the
    third round (default), every round eager, the stock layers inside the
    graphs, and the fused layers without packed weights."""
    from ddtree_eagle3_patch_b200.ddtree import ddtree_generate
    eager, fused, pack = MODES[mode]
    monkeypatch.setenv("DDTREE_EAGER", eager)
    monkeypatch.setenv("DDTREE_FUSED", fused)
    monkeypatch.setenv("DDTREE_PACK", pack)
    z = decode_golden
    p = name + "_"
    tgt, drf, vocab, block, budget, plen, max_new = _models(name, z)
    tgt, drf = tgt.to(DEV), drf.to(DEV)
    ids = torch.from_numpy(z[p + "prompt"]).to(DEV)
    res = ddtree_generate(drf, tgt, ids, mask_token_id=vocab - 1, max_new_tokens=max_new, block_size=block,
                          stop_token_ids=None, temperature=0.0, tree_budget=budget, save_tree_traces=True)
    assert res.output_ids.tolist() == z[p + "output_ids"].tolist()
    assert res.acceptance_lengths == z[p + "acceptance"].tolist()
    assert res.decode_rounds == len(z[p + "acceptance"])
    assert res.num_input_tokens == plen
    assert res.num_output_tokens == z[p + "output_ids"].shape[1] - plen
    for r, tr in enumerate(res.round_trees):
        n = len(tr["tree"]["node_token_ids"])
        assert tr["tree"]["parents"] == z[p + "round_parents"][r][: n + 1].tolist(), r
        assert tr["tree"]["node_token_ids"] == z[p + "round_tokens"][r][:n].tolist(), r
        assert tr["tree"]["node_depths"] == z[p + "round_depths"][r][:n].tolist(), r
        acc = tr["accepted_indices"]
        assert acc == z[p + "round_accepted"][r][: len(acc)].tolist(), r
        assert z[p + "round_accepted"][r][len(acc):].tolist() == [-2] * (1 + budget - len(acc))
    assert set(res.stage_times) == {"draft", "tree_build", "tree_compile", "verify", "commit", "tree_build_copy",
                                    "tree_build_heap", "tree_build_visibility"}
    assert res.time_to_first_token > 0 and res.time_per_output_token > 0
    assert len(res.round_timestamps) == res.decode_rounds
    if eager == "0":
        assert res.graph_rounds == max(res.decode_rounds - 2, 0)
    else:
        assert res.graph_rounds == 0
    assert res.native_launches > 0
    assert all(b >= a for a, b in zip(res.round_timestamps, res.round_timestamps[1:]))


@pytest.mark.gpu
def test_session_reused_across_calls(decode_golden):
    """A second call on the same models reuses the captured graphs (no new
    capture) and gives the same result; a longer call gets a new session."""
    from ddtree_eagle3_patch_b200.ddtree import ddtree_generate, release_decode_sessions
    z = decode_golden
    name = "v16_b8_t32"
    p = name + "_"
    tgt, drf, vocab, block, budget, plen, max_new = _models(name, z)
    tgt, drf = tgt.to(DEV), drf.to(DEV)
    ids = torch.from_numpy(z[p + "prompt"]).to(DEV)
    kw = dict(mask_token_id=vocab - 1, max_new_tokens=max_new, block_size=block, stop_token_ids=None,
              tree_budget=budget)
    r1 = ddtree_generate(drf, tgt, ids, **kw)
    assert r1.graph_capture_s > 0
    r2 = ddtree_generate(drf, tgt, ids, **kw)
    assert r2.graph_capture_s == 0 and r2.graph_rounds == r2.decode_rounds - 1
    assert r2.output_ids.tolist() == z[p + "output_ids"].tolist() == r1.output_ids.tolist()
    assert r2.acceptance_lengths == r1.acceptance_lengths
    # a different prompt on the same session
    r3 = ddtree_generate(drf, tgt, ids[:, 3:], **kw)
    assert r3.graph_capture_s == 0 and r3.num_input_tokens == plen - 3
    release_decode_sessions(tgt)
    assert "_ddtree_session" not in tgt.__dict__


@pytest.mark.gpu
@pytest.mark.parametrize("name", [c[0] for c in C.CASES])
def test_ddtree_generate_stop_token_matches_reference(name, decode_golden):
    from ddtree_eagle3_patch_b200.ddtree import ddtree_generate
    z = decode_golden
    p = name + "_"
    tgt, drf, vocab, block, budget, plen, max_new = _models(name, z)
    tgt, drf = tgt.to(DEV), drf.to(DEV)
    ids = torch.from_numpy(z[p + "prompt"]).to(DEV)
    res = ddtree_generate(drf, tgt, ids, mask_token_id=vocab - 1, max_new_tokens=max_new, block_size=block,
                          stop_token_ids=[int(z[p + "stop_token"])], temperature=0.0, tree_budget=budget)
    assert res.output_ids.tolist() == z[p + "stop_output_ids"].tolist()
    assert res.acceptance_lengths == z[p + "stop_acceptance"].tolist()
    assert res.round_trees is None


@pytest.mark.gpu
def test_ddtree_generate_is_lossless_in_bf16():
    """bf16 at a Qwen3-like width: the speculative output equals greedy
    decoding of the same target through the same kernels (block size 1 runs
    the target alone), and temperature > 0 runs and emits in-vocabulary ids."""
    from ddtree_eagle3_patch_b200.ddtree import ddtree_generate
    z = np.load(HERE / "golden" / "decode.npz")
    tgt, drf, vocab, block, budget, plen, max_new = _models("v300_b6_t12", z)
    tgt, drf = tgt.to(DEV, torch.bfloat16), drf.to(DEV, torch.bfloat16)
    ids = torch.from_numpy(z["v300_b6_t12_prompt"]).to(DEV)
    # the reference drops generated tokens equal to the mask token from its
    # output (ddtree.py:566); pick a mask token neither run emits, so that
    # positions line up for the comparison
    for mask_id in range(vocab - 1, vocab - 9, -1):
        spec = ddtree_generate(drf, tgt, ids, mask_token_id=mask_id, max_new_tokens=max_new, block_size=block,
                               stop_token_ids=None, tree_budget=budget)
        ar = ddtree_generate(drf, tgt, ids, mask_token_id=mask_id, max_new_tokens=max_new, block_size=1,
                             stop_token_ids=None)
        if spec.num_output_tokens == max_new and ar.num_output_tokens == max_new:
            break
    assert spec.num_output_tokens == max_new and ar.num_output_tokens == max_new
    assert ar.acceptance_lengths == [1] * ar.decode_rounds
    a, b = spec.output_ids[0], ar.output_ids[0]
    assert torch.equal(a[:plen], b[:plen])
    diff = (a != b).nonzero()
    if diff.numel():
        # bf16 GEMMs of different batch shapes may round differently: the
        # first divergence must be a near-tie of the target's own logits
        # (scored here by the target's stock attention on the shared prefix)
        i = int(diff[0])
        with torch.inference_mode():
            row = tgt(a[:i].unsqueeze(0).to(DEV)).logits[0, -1].float()
        gap = abs(float(row[int(a[i])] - row[int(b[i])]))
        assert gap <= 0.05 * float(row.abs().max()), (i, gap)
    torch.manual_seed(3)
    hot = ddtree_generate(drf, tgt, ids, mask_token_id=vocab - 1, max_new_tokens=16, block_size=block,
                          stop_token_ids=None, temperature=0.8, tree_budget=budget)
    out = hot.output_ids[0, plen:]
    assert out.numel() > 0 and int(out.max()) < vocab and int(out.min()) >= 0
    assert sum(hot.acceptance_lengths) >= 16


@pytest.mark.gpu
def test_bf16_decode_identical_across_launch_forms(monkeypatch):
    """A bf16 model whose projections all take the weight-streaming GEMM
    (fused gate/up included): the captured forwards with programmatic
    dependent launches, without them, and every round eager run the same
    kernels on the same data and so emit identical ids and acceptances;
    the cuBLAS projections (DDTREE_WGEMM=0) sum in another order and are
    held to a near-tie at their first divergence."""
    from ddtree_eagle3_patch_b200.ddtree import ddtree_generate
    from ddtree_eagle3_patch_b200.synthetic import build_decode_models, random_prompt
    tgt, drf = build_decode_models("qwen3-small", DEV, torch.bfloat16, seed=4, draft_layers=2, block_size=8)
    ids = random_prompt(40, vocab=1024, seed=2, exclude=drf.mask_token_id).to(DEV)

    def run(**env):
        for k in ("DDTREE_PDL", "DDTREE_EAGER", "DDTREE_WGEMM", "DDTREE_HEAD_TOPK"):
            monkeypatch.delenv(k, raising=False)
        for k, v in env.items():
            monkeypatch.setenv(k, v)
        return ddtree_generate(drf, tgt, ids, mask_token_id=drf.mask_token_id, max_new_tokens=48, block_size=8,
                               stop_token_ids=None, temperature=0.0, tree_budget=16)

    base = run()
    assert base.graph_rounds > 0
    # (DDTREE_HEAD_TOPK=1: the draft head fused with the tree build's top-k)
    for env in ({"DDTREE_PDL": "0"}, {"DDTREE_EAGER": "1"}, {"DDTREE_HEAD_TOPK": "1"}):
        other = run(**env)
        assert other.output_ids.tolist() == base.output_ids.tolist(), env
        assert other.acceptance_lengths == base.acceptance_lengths, env
    from ddtree_eagle3_patch_b200 import kernels
    assert kernels.wgemm_status(DEV) == 0
    cub = run(DDTREE_WGEMM="0")
    a, b = base.output_ids[0], cub.output_ids[0]
    n = min(a.numel(), b.numel())
    diff = (a[:n] != b[:n]).nonzero()
    if diff.numel():
        i = int(diff[0])
        with torch.inference_mode():
            row = tgt(a[:i].unsqueeze(0)).logits[0, -1].float()
        gap = abs(float(row[int(a[i])] - row[int(b[i])]))
        assert gap <= 0.05 * float(row.abs().max()), (i, gap)
