"""End-to-end EAGLE3 decode parity: this package's ``eagle3_generate`` on
the GPU against the reference's own run on CPU (tests/golden/eagle3.npz,
written by gen_eagle3_golden.py).

The EAGLE3 draft head is not part of the accelerated path; its recorded
``topk_generate`` calls are replayed (a call handed ids other than the
recorded ones fails the test, so every round's accepted tokens are checked
as they happen).  The target is the seeded float32 Qwen3 model, run through
the tree-attention kernel, the static cache with its in-place compaction
and the EAGLE3 accept kernel.  The fixture's verify rows all have an argmax
margin of at least 2e-4, so the emitted ids and acceptance lengths must be
identical."""
import sys
from pathlib import Path

import numpy as np
import pytest
import torch

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE / "golden"))

import decode_case as C  # noqa: E402

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda", 0)
CASES = ["e3_v64_t16", "e3_v300_t12", "e3_v16_t24"]


class ReplayDraft:
    """Stands in for the EAGLE3 draft head: returns the reference's recorded
    trees in order and checks the ids it is given."""

    def __init__(self, z, prefix: str, tree: int):
        self.z, self.p = z, prefix
        self.total_tokens = tree - 1
        self.target_layer_ids = [0, 1, 2]
        self.device = DEV
        self.calls = 0

    def reset_kv(self):
        pass

    def topk_generate(self, hidden, input_ids):
        q = f"{self.p}call{self.calls}_"
        expect = self.z[q + "input_ids"]
        got = input_ids.cpu().numpy()
        assert got.tolist() == expect.tolist(), f"call {self.calls}: ids differ from the reference's"
        assert hidden.shape[0] == 1 and hidden.shape[-1] == 3 * 96
        self.calls += 1
        return (torch.from_numpy(self.z[q + "draft_tokens"]).to(DEV), torch.from_numpy(self.z[q + "retrieve"]).to(DEV),
                torch.from_numpy(self.z[q + "tree_mask"]).to(DEV)[None, None].float(),
                torch.from_numpy(self.z[q + "positions"]).to(DEV))


@pytest.fixture(scope="module")
def eagle3_golden():
    return np.load(HERE / "golden" / "eagle3.npz")


@pytest.mark.parametrize("eager", ["0", "1"], ids=["graph", "eager"])
@pytest.mark.parametrize("name", CASES)
def test_eagle3_generate_matches_reference(name, eager, eagle3_golden, monkeypatch):
    from transformers import Qwen3ForCausalLM
    from ddtree_eagle3_patch_b200.eagle3 import eagle3_generate
    monkeypatch.setenv("DDTREE_EAGER", eager)
    z = eagle3_golden
    p = name + "_"
    vocab = {"e3_v64_t16": 64, "e3_v300_t12": 300, "e3_v16_t24": 16}[name]
    tree = {"e3_v64_t16": 16, "e3_v300_t12": 12, "e3_v16_t24": 24}[name]
    max_new = {"e3_v64_t16": 30, "e3_v300_t12": 24, "e3_v16_t24": 30}[name]
    seed = int(z[p + "seed"])
    torch.manual_seed(0)
    tgt = Qwen3ForCausalLM(C.target_config(vocab)).eval()
    assert C.seeded_init(tgt, seed) == str(z[p + "sha_target"])
    tgt = tgt.to(DEV)
    draft = ReplayDraft(z, p, tree)
    ids = torch.from_numpy(z[p + "prompt"]).to(DEV)
    res = eagle3_generate(draft, tgt, ids, max_new_tokens=max_new, stop_token_ids=None, temperature=0.0)
    assert res.output_ids.tolist() == z[p + "output_ids"].tolist()
    assert res.acceptance_lengths == z[p + "acceptance"].tolist()
    assert draft.calls == int(z[p + "n_calls"])
    assert set(res.stage_times) == {"draft", "verify", "commit"}
    if eager == "0" and res.decode_rounds > 3:
        assert res.graph_rounds > 0
