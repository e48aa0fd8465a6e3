"""The CPU port of the reference's decode loop (oracle/cpu_decode.py, the
timed CPU baseline of the decode benchmark) reproduces the reference's own
recorded runs (tests/golden/decode.npz): same emitted ids and acceptance
lengths on the seeded float32 models."""
import sys
from pathlib import Path

import numpy as np
import pytest
import torch

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE / "golden"))

import decode_case as C  # noqa: E402


@pytest.mark.parametrize("name", [c[0] for c in C.CASES])
def test_cpu_port_matches_reference_fixture(name):
    from transformers import Qwen3ForCausalLM
    from oracle.cpu_decode import CpuDecode, CpuDFlashDraft
    z = np.load(HERE / "golden" / "decode.npz")
    _, vocab, block, budget, plen, max_new = next(c for c in C.CASES if c[0] == name)
    p = name + "_"
    seed = int(z[p + "seed"])
    torch.manual_seed(0)
    tcfg = C.target_config(vocab)
    tcfg._attn_implementation = "sdpa"
    tgt = Qwen3ForCausalLM(tcfg).eval()
    assert C.seeded_init(tgt, seed) == str(z[p + "sha_target"])
    drf = CpuDFlashDraft(C.draft_config(vocab, block, vocab - 1)).eval()
    assert C.seeded_init(drf, seed + 1000) == str(z[p + "sha_draft"])
    run = CpuDecode(drf, tgt, torch.from_numpy(z[p + "prompt"]), max_new, block, budget)
    run.prefill()
    while run.start < run.max_length:
        run.round()
    out = run.output_ids[:, : run.max_length]
    out = out[:, out[0] != vocab - 1]
    assert out.tolist() == z[p + "output_ids"].tolist()
    assert run.acceptance == z[p + "acceptance"].tolist()
