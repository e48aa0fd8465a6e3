"""Record end-to-end decode fixtures from the reference's own ``ddtree_generate``.

Run in a container where the reference checkout is importable:

    python tests/golden/gen_decode_golden.py <reference checkout>

For each case of ``decode_case.CASES`` it builds a float32 Qwen3 target and
the reference's DFlash draft with seeded weights (``decode_case``), runs the
reference's ``ddtree_generate`` on CPU with tree traces on, and records the
emitted ids, the acceptance lengths and every round's tree and accepted
indices.  It also runs the case again with a stop token taken from the
generated text, to pin the stop logic.

A model seed is kept only if every decision of the run has a margin above
``MARGIN`` (absolute, in logit / log-probability units), far above the
~1e-6 float32 difference between the CPU reference and the GPU path:
  * the target's argmax on every verify row the walk reads (and the
    prefill's first token): top-1 minus top-2 logit;
  * the draft's top-k on every depth the tree reaches: the gaps between
    consecutive sorted logits up to one rank past the deepest rank used;
  * the best-first expansion: at every pop, the popped key against the
    next-best key left in the heap.
The chosen seeds and the smallest margins are stored with the fixture.
Output: tests/golden/decode.npz.
"""
from __future__ import annotations

import heapq
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


def _import_reference(ref_root: str):
    sys.path.insert(0, ref_root)
    import dflash
    dflash.cuda_time = time.perf_counter
    import ddtree
    ddtree.cuda_time = time.perf_counter
    from model import DFlashDraftModel
    return ddtree, DFlashDraftModel


def _heap_margin(lp: np.ndarray, budget: int) -> float:
    """Smallest gap between a popped key and the next-best key, replaying
    the reference's heap (ddtree.py:146-177) on its own log-probs."""
    L, k = lp.shape
    heap = [(-float(lp[0, 0]), (0,), 0, 1, 0, float(lp[0, 0]))]
    best = np.inf
    n = 0
    while heap and n < budget:
        neg, ranks, parent, depth, rank, logw = heapq.heappop(heap)
        if heap:
            best = min(best, heap[0][0] - neg)
        n += 1
        idx = n
        if rank + 1 < k:
            sib = logw - float(lp[depth - 1, rank]) + float(lp[depth - 1, rank + 1])
            heapq.heappush(heap, (-sib, ranks[:-1] + (rank + 1,), parent, depth, rank + 1, sib))
        if depth < L:
            ch = logw + float(lp[depth, 0])
            heapq.heappush(heap, (-ch, ranks + (0,), idx, depth + 1, 0, ch))
    return best


def _topk_margin(logits: np.ndarray, depths_used: dict) -> float:
    best = np.inf
    for d, max_rank in depths_used.items():
        row = np.sort(logits[d].astype(np.float64))[::-1]
        upto = min(max_rank + 2, row.size)
        if upto >= 2:
            best = min(best, float(np.min(row[: upto - 1] - row[1:upto])))
    return best


def _argmax_margin(row: np.ndarray) -> float:
    s = np.sort(row.astype(np.float64))[::-1]
    return float(s[0] - s[1])


def run_case(ddtree, DFlashDraftModel, name, vocab, block, budget, plen, max_new, seed):
    from transformers import Qwen3ForCausalLM
    mask_id = vocab - 1
    torch.manual_seed(0)
    tgt = Qwen3ForCausalLM(C.target_config(vocab)).eval()
    sha_t = C.seeded_init(tgt, seed)
    drf = DFlashDraftModel(C.draft_config(vocab, block, mask_id)).eval()
    sha_d = C.seeded_init(drf, seed + 1000)
    ids = C.prompt(seed, plen, vocab, mask_id)

    draft_logits, sampled = [], []
    orig_build, orig_sample = ddtree.build_ddtree_tree, ddtree.sample

    def rec_build(logits, b):
        draft_logits.append(logits.detach().float().numpy().copy())
        return orig_build(logits, b)

    def rec_sample(logits, temperature=0.0):
        sampled.append(logits.detach().float().numpy().copy())
        return orig_sample(logits, temperature)

    ddtree.build_ddtree_tree, ddtree.sample = rec_build, rec_sample
    try:
        res = ddtree.ddtree_generate(drf, tgt, ids, mask_token_id=mask_id, max_new_tokens=max_new, block_size=block,
                                     stop_token_ids=None, temperature=0.0, tree_budget=budget, save_tree_traces=True)
    finally:
        ddtree.build_ddtree_tree, ddtree.sample = orig_build, orig_sample

    margins = {"argmax": _argmax_margin(sampled[0][0, -1]), "topk": np.inf, "heap": np.inf}
    for r, tr in enumerate(res.round_trees):
        logits = sampled[r + 1][0]
        for i in tr["accepted_indices"]:
            margins["argmax"] = min(margins["argmax"], _argmax_margin(logits[i]))
        dl = draft_logits[r]
        k = min(budget, dl.shape[-1])
        x = torch.from_numpy(dl)
        top, _ = torch.topk(x, k=k, dim=-1)
        lp = (top - torch.logsumexp(x, dim=-1, keepdim=True)).numpy()
        margins["heap"] = min(margins["heap"], _heap_margin(lp, budget))
        used: dict = {}
        depths = tr["tree"]["node_depths"]
        parents = tr["tree"]["parents"]
        # rank of each node within its parent's children, by pop order of the
        # reference's heap: recompute from the top-k ids
        top_ids = torch.topk(x, k=k, dim=-1).indices.numpy()
        for tok, d in zip(tr["tree"]["node_token_ids"], depths):
            r_ = int(np.nonzero(top_ids[d - 1] == tok)[0][0])
            used[d - 1] = max(used.get(d - 1, 0), r_)
        margins["topk"] = min(margins["topk"], _topk_margin(dl, used))
        del parents
    return res, margins, sha_t, sha_d, ids, (tgt, drf)


def main(ref_root: str):
    ddtree, DFlashDraftModel = _import_reference(ref_root)
    torch.set_num_threads(8)
    out = {}
    for name, vocab, block, budget, plen, max_new in C.CASES:
        for seed in range(100, 300):
            res, margins, sha_t, sha_d, ids, models = run_case(ddtree, DFlashDraftModel, name, vocab, block, budget,
                                                               plen, max_new, seed)
            m = min(margins.values())
            print(f"{name} seed {seed}: margins {margins} acceptance {res.acceptance_lengths}", flush=True)
            if m < MARGIN:
                continue
            p = name + "_"
            out[p + "seed"] = np.int64(seed)
            out[p + "sha_target"] = np.array(sha_t)
            out[p + "sha_draft"] = np.array(sha_d)
            out[p + "prompt"] = ids.numpy()
            out[p + "output_ids"] = res.output_ids.numpy()
            out[p + "acceptance"] = np.array(res.acceptance_lengths, np.int64)
            out[p + "margins"] = np.array([margins["argmax"], margins["topk"], margins["heap"]])
            trees = res.round_trees
            out[p + "round_parents"] = np.array([np.pad(t["tree"]["parents"], (0, 1 + budget - len(t["tree"]["parents"])),
                                                        constant_values=-2) for t in trees], np.int64)
            out[p + "round_tokens"] = np.array([np.pad(t["tree"]["node_token_ids"],
                                                       (0, budget - len(t["tree"]["node_token_ids"])),
                                                       constant_values=-2) for t in trees], np.int64)
            out[p + "round_depths"] = np.array([np.pad(t["tree"]["node_depths"],
                                                       (0, budget - len(t["tree"]["node_depths"])),
                                                       constant_values=-2) for t in trees], np.int64)
            out[p + "round_accepted"] = np.array([np.pad(t["accepted_indices"], (0, 1 + budget - len(t["accepted_indices"])),
                                                         constant_values=-2) for t in trees], np.int64)
            # the same run stopped at a token it generates
            gen = res.output_ids[0, plen:].tolist()
            stop = gen[len(gen) // 3]
            tgt, drf = models
            res2 = ddtree.ddtree_generate(drf, tgt, ids, mask_token_id=vocab - 1, max_new_tokens=max_new,
                                          block_size=block, stop_token_ids=[stop], temperature=0.0,
                                          tree_budget=budget)
            out[p + "stop_token"] = np.int64(stop)
            out[p + "stop_output_ids"] = res2.output_ids.numpy()
            out[p + "stop_acceptance"] = np.array(res2.acceptance_lengths, np.int64)
            break
        else:
            raise RuntimeError(f"no seed with margins above {MARGIN} for {name}")
    np.savez_compressed(HERE / "decode.npz", **out)
    print("wrote", HERE / "decode.npz")


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else "../reference")
