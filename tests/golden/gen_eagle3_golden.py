"""Record end-to-end EAGLE3 decode fixtures from the reference's own
``eagle3_generate``.

Run in a container where the reference checkout is importable:

    python tests/golden/gen_eagle3_golden.py <reference checkout>

The target is the seeded float32 Qwen3 model of ``decode_case``; the draft
is the reference's ``Eagle3DraftModel`` with a small seeded head (hidden 96,
tied to the target's embeddings).  The draft model is not part of the
accelerated path, so every call of its ``topk_generate`` is recorded - the
committed ids it receives and the tree it returns (draft tokens, retrieve
indices, tree mask, positions) - and the GPU test replays those calls,
checking that the ids it is handed are the recorded ones.  The emitted ids
and acceptance lengths are recorded too.

A seed is kept only if every verify row's target argmax has a margin above
``MARGIN``, far above the float32 CPU/GPU difference.
Output: tests/golden/eagle3.npz.
"""
from __future__ import annotations

import sys
import time
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent.parent))
sys.path.insert(0, str(HERE))

import decode_case as C  # noqa: E402

MARGIN = 2e-4
# (name, vocab, tree size, depth, top-k, prompt length, max_new_tokens)
CASES = [("e3_v64_t16", 64, 16, 4, 4, 20, 30), ("e3_v300_t12", 300, 12, 3, 5, 17, 24),
         ("e3_v16_t24", 16, 24, 3, 8, 20, 30)]   # a top-k of half the vocabulary: longer accepted paths


def draft_config(vocab: int):
    from transformers import LlamaConfig
    cfg = LlamaConfig(vocab_size=vocab, hidden_size=96, intermediate_size=192, num_attention_heads=4,
                      num_key_value_heads=2, head_dim=24, max_position_embeddings=512, rms_norm_eps=1e-6,
                      hidden_act="silu", pretraining_tp=1)
    cfg.eagle_aux_hidden_state_layer_ids = [0, 1, 2]
    return cfg


def run(ref_root: str):
    sys.path.insert(0, ref_root)
    import dflash
    dflash.cuda_time = time.perf_counter
    import eagle3
    eagle3.cuda_time = time.perf_counter
    from model import Eagle3DraftModel
    from transformers import Qwen3ForCausalLM
    torch.set_num_threads(8)
    out = {}
    for name, vocab, tree, depth, topk, plen, max_new in CASES:
        for seed in range(300, 400):
            torch.manual_seed(0)
            tgt = Qwen3ForCausalLM(C.target_config(vocab)).eval()
            sha_t = C.seeded_init(tgt, seed)
            drf = Eagle3DraftModel(draft_config(vocab), total_tokens=tree, depth=depth, top_k=topk).eval()
            sha_d = C.seeded_init(drf, seed + 2000)
            drf.tie_target_embeddings(tgt.get_input_embeddings())
            drf.init_tree()
            ids = C.prompt(seed, plen, vocab, vocab)
            calls, logits_seen = [], []
            orig_topk, orig_sample = drf.topk_generate, eagle3.sample

            def rec_topk(hidden, input_ids, *a, **k):
                res = orig_topk(hidden, input_ids, *a, **k)
                calls.append((input_ids.clone(), [r.clone() for r in res]))
                return res

            def rec_sample(logits, temperature=0.0):
                logits_seen.append(logits.detach().float().clone())
                return orig_sample(logits, temperature)

            drf.topk_generate, eagle3.sample = rec_topk, rec_sample
            try:
                res = eagle3.eagle3_generate(drf, tgt, ids, max_new_tokens=max_new, stop_token_ids=None,
                                             temperature=0.0)
            finally:
                eagle3.sample = orig_sample
                del drf.topk_generate
            # the verify logits are the [1, T, V] calls of sample (the others are
            # the prefill and the bonus row)
            margin = np.inf
            for lg in logits_seen:
                s = torch.sort(lg.reshape(-1, lg.shape[-1]), dim=-1, descending=True).values
                margin = min(margin, float((s[:, 0] - s[:, 1]).min()))
            print(f"{name} seed {seed}: margin {margin:.2e} acceptance {res.acceptance_lengths}", flush=True)
            if margin < MARGIN:
                continue
            p = name + "_"
            T = tree
            out[p + "seed"] = np.int64(seed)
            out[p + "sha_target"] = np.array(sha_t)
            out[p + "sha_draft"] = np.array(sha_d)
            out[p + "prompt"] = ids.numpy()
            out[p + "output_ids"] = res.output_ids.numpy()
            out[p + "acceptance"] = np.array(res.acceptance_lengths, np.int64)
            out[p + "margin"] = np.float64(margin)
            out[p + "n_calls"] = np.int64(len(calls))
            for i, (inp, (dt, ri, tm, tp)) in enumerate(calls):
                q = f"{p}call{i}_"
                out[q + "input_ids"] = inp.numpy()
                out[q + "draft_tokens"] = dt.numpy()
                out[q + "retrieve"] = ri.numpy()
                out[q + "tree_mask"] = tm.reshape(T, T).to(torch.bool).numpy()
                out[q + "positions"] = tp.numpy()
            break
        else:
            raise RuntimeError(f"no seed with margin above {MARGIN} for {name}")
    np.savez_compressed(HERE / "eagle3.npz", **out)
    print("wrote", HERE / "eagle3.npz")


if __name__ == "__main__":
    run(sys.argv[1] if len(sys.argv) > 1 else "../reference")
