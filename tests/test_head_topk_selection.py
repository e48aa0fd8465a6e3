"""The block-selection rule of the tree build's head-statistics mode
(ddt_tree_build_head), restated in numpy and checked against a brute-force
top-k on CPU: a chunk's top-kc keys lie in the kc blocks of 128 with the
largest block keys, at or above the kc-th largest block key t0."""
import zlib

import numpy as np
import pytest

BLOCK = 128


def _keys(vals: np.ndarray, ids: np.ndarray) -> np.ndarray:
    """Value order (fp32 bit pattern made monotone), then the lower id."""
    u = vals.astype(np.float32).view(np.uint32).astype(np.uint64)
    neg = (u & 0x80000000) != 0
    o = np.where(neg, (~u) & 0xFFFFFFFF, u | 0x80000000)
    return (o << np.uint64(32)) | (np.uint64(0xFFFFFFFF) - ids.astype(np.uint64))


def _select(chunk_keys: np.ndarray, kc: int) -> np.ndarray:
    """The candidates the kernel gathers: keys >= t0 of the kc blocks with
    the largest block keys (every block when there are at most kc)."""
    blocks = chunk_keys.reshape(-1, BLOCK)
    bkey = blocks.max(axis=1)
    order = np.argsort(bkey)[::-1]
    picked = order[:kc]
    t0 = bkey[order[kc - 1]] if len(bkey) > kc else np.uint64(0)
    cand = blocks[picked].reshape(-1)
    return cand[cand >= t0]


def _top(keys: np.ndarray, kc: int) -> np.ndarray:
    return np.sort(keys)[::-1][:kc]


def _rows(kind: str, rng, n_blocks: int) -> np.ndarray:
    v = n_blocks * BLOCK
    if kind == "normal":
        return rng.standard_normal(v).astype(np.float32)
    if kind == "clustered":            # the best values crowd into one block
        x = rng.standard_normal(v).astype(np.float32)
        b = int(rng.integers(n_blocks))
        x[b * BLOCK: (b + 1) * BLOCK] += 20
        return x
    if kind == "equal":                # every value equal: ids decide
        return np.zeros(v, np.float32)
    if kind == "few_values":           # heavy ties across blocks
        return rng.integers(0, 3, v).astype(np.float32)
    if kind == "bf16":                 # bf16-rounded logits, many near-ties
        x = rng.standard_normal(v).astype(np.float32) * 4
        return (x.view(np.uint32) & 0xFFFF0000).view(np.float32)
    raise ValueError(kind)


@pytest.mark.parametrize("kind", ["normal", "clustered", "equal", "few_values", "bf16"])
@pytest.mark.parametrize("n_blocks,kc", [(132, 32), (132, 64), (8, 32), (1, 16), (64, 80)])
def test_candidates_hold_the_exact_top_k(kind, n_blocks, kc):
    rng = np.random.default_rng(zlib.crc32(f"{kind}/{n_blocks}/{kc}".encode()))
    for trial in range(5):
        vals = _rows(kind, rng, n_blocks)
        c0 = int(rng.integers(0, 1000)) * BLOCK   # chunk offset inside the row
        keys = _keys(vals, np.arange(c0, c0 + vals.size))
        k = min(kc, vals.size)
        cand = _select(keys, k)
        assert np.array_equal(_top(cand, k), _top(keys, k)), (kind, trial)
        # the rule reads at most k blocks
        assert cand.size <= k * BLOCK
