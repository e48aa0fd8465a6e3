"""CPU oracle for the DDTree per-step draft-tree hot path.

TEST INFRASTRUCTURE ONLY.  Nothing in the product package imports this
module; it is the checker that tests/, ``__graft_entry__.smoke()`` and the
CPU-baseline leg of ``bench.py`` compare the CUDA path against.

The arithmetic lives in ``ddtree_oracle.c`` (a restatement of the reference's
``ddtree.py`` / ``eagle3.py`` / ``model/utils.py`` functions, each citing the
lines it follows); this module builds it with gcc, loads it with ctypes and
adds numpy restatements of the pieces that are plain array moves
(``compile_ddtree_tree`` buffers, KV compaction) plus a float32 attention
reference for the verify-attention kernel.

Parity pins: ``tests/golden/*.npz`` hold outputs of the reference itself
(imported in-process in the build container by ``tests/golden/gen_golden.py``)
and ``tests/test_oracle.py`` checks this oracle against every one of them.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np

_HERE = Path(__file__).resolve().parent
_SRC = _HERE / "ddtree_oracle.c"
_LIB_PATH = _HERE / "libddtree_oracle.so"
_lib = None


def build(force: bool = False) -> Path:
    """Compile the C restatement into ``oracle/libddtree_oracle.so``."""
    if force or not _LIB_PATH.exists() or _LIB_PATH.stat().st_mtime < _SRC.stat().st_mtime:
        tmp = _LIB_PATH.with_suffix(f".so.tmp{os.getpid()}")
        cmd = ["gcc", "-O2", "-fPIC", "-shared", "-std=c11", "-fno-fast-math",
               "-ffp-contract=off", str(_SRC), "-o", str(tmp), "-lm"]
        subprocess.run(cmd, check=True)
        os.replace(tmp, _LIB_PATH)
    return _LIB_PATH


def lib():
    global _lib
    if _lib is None:
        path = build()
        L = ctypes.CDLL(str(path))
        i64, p = ctypes.c_int64, ctypes.c_void_p
        L.ora_topk_logz.argtypes = [p, i64, i64, i64, i64, p, p, p]
        L.ora_topk_logz.restype = ctypes.c_int
        L.ora_log_probs.argtypes = [p, p, i64, i64, p]
        L.ora_log_probs.restype = None
        L.ora_tree_from_lp.argtypes = [p, p, i64, i64, i64, p, p, p, p, p, p, p]
        L.ora_tree_from_lp.restype = ctypes.c_int
        L.ora_argmax_bf16.argtypes = [p, i64, i64, i64, p]
        L.ora_argmax_bf16.restype = None
        L.ora_argmax_f32.argtypes = [p, i64, i64, i64, p]
        L.ora_argmax_f32.restype = None
        L.ora_follow.argtypes = [p, p, i64, p, p, i64, p]
        L.ora_follow.restype = i64
        L.ora_eagle3_posterior.argtypes = [p, p, i64, p, i64, i64, p, p, p, p]
        L.ora_eagle3_posterior.restype = None
        _lib = L
    return _lib


def _ptr(a: np.ndarray):
    return a.ctypes.data_as(ctypes.c_void_p)


# ----------------------------------------------------------------------------
# tree build (ddtree.py:114-196)
# ----------------------------------------------------------------------------
def topk_logz(logits: np.ndarray, k: int):
    """Per-row top-k (value desc, token id asc) and fp32 log-normaliser.

    ``logits`` is float32 [L, V] (bf16 inputs are widened exactly first).
    Returns (ids int64 [L,k], top_vals f32 [L,k], logz f32 [L]).
    """
    x = np.ascontiguousarray(logits, dtype=np.float32)
    L, V = x.shape
    ids = np.empty((L, k), np.int64)
    vals = np.empty((L, k), np.float32)
    logz = np.empty((L,), np.float32)
    rc = lib().ora_topk_logz(_ptr(x), L, V, V, k, _ptr(ids), _ptr(vals), _ptr(logz))
    if rc != 0:
        raise ValueError(f"ora_topk_logz failed ({rc})")
    return ids, vals, logz


def log_probs(vals: np.ndarray, logz: np.ndarray) -> np.ndarray:
    vals = np.ascontiguousarray(vals, np.float32)
    logz = np.ascontiguousarray(logz, np.float32)
    L, K = vals.shape
    lp = np.empty_like(vals)
    lib().ora_log_probs(_ptr(vals), _ptr(logz), L, K, _ptr(lp))
    return lp


def tree_from_lp(lp: np.ndarray, ids: np.ndarray, budget: int) -> dict:
    """Best-first expansion (ddtree.py:146-189) from given log-probs and ids."""
    lp = np.ascontiguousarray(lp, np.float32)
    ids = np.ascontiguousarray(ids, np.int64)
    L, K = lp.shape if lp.ndim == 2 else (0, 0)
    cap = max(int(budget), 0)
    toks = np.zeros(max(cap, 1), np.int64)
    deps = np.zeros(max(cap, 1), np.int64)
    ranks = np.zeros(max(cap, 1), np.int32)
    logw = np.zeros(max(cap, 1), np.float64)
    parents = np.zeros(cap + 1, np.int32)
    vis = np.zeros((cap + 1) * (cap + 1), np.uint8)
    n = np.zeros(1, np.int64)
    rc = lib().ora_tree_from_lp(_ptr(lp), _ptr(ids), L, K, int(budget), _ptr(toks), _ptr(deps),
                                _ptr(ranks), _ptr(parents), _ptr(vis), _ptr(logw), _ptr(n))
    if rc != 0:
        raise ValueError(f"ora_tree_from_lp failed ({rc})")
    n = int(n[0])
    N = n + 1
    return {
        "node_token_ids": toks[:n].copy(),
        "node_depths": deps[:n].copy(),
        "node_ranks": ranks[:n].copy(),
        "node_logw": logw[:n].copy(),
        "parents": parents[:N].copy(),
        "visibility": vis[: N * N].reshape(N, N).astype(bool),
    }


def build_tree(draft_logits: np.ndarray, budget: int) -> dict:
    """Whole ``build_ddtree_tree`` restatement from float32 draft logits [L, V]."""
    x = np.asarray(draft_logits, np.float32)
    L = x.shape[0]
    if budget <= 0 or L == 0:
        return tree_from_lp(np.zeros((0, 1), np.float32), np.zeros((0, 1), np.int64), 0) | {
            "ids": np.zeros((L, 0), np.int64), "lp": np.zeros((L, 0), np.float32),
            "logz": np.zeros((L,), np.float32)}
    k = min(int(budget), x.shape[1])
    ids, vals, logz = topk_logz(x, k)
    lp = log_probs(vals, logz)
    out = tree_from_lp(lp, ids, budget)
    out.update(ids=ids, lp=lp, logz=logz, top_vals=vals)
    return out


def pack_visibility(vis: np.ndarray, words: int | None = None) -> np.ndarray:
    """Pack a bool [N, N] ancestor matrix into uint32 words per row (bit j of
    word j//32 = column j), the layout the CUDA kernels use."""
    N = vis.shape[0]
    W = (N + 31) // 32 if words is None else words
    out = np.zeros((N, W), np.uint32)
    for j in range(N):
        out[:, j // 32] |= (vis[:, j].astype(np.uint32) << np.uint32(j % 32))
    return out


def unpack_visibility(words: np.ndarray, N: int) -> np.ndarray:
    w = np.asarray(words, np.uint32)
    cols = np.arange(N)
    return ((w[:N, cols // 32] >> (cols % 32).astype(np.uint32)) & 1).astype(bool)


# ----------------------------------------------------------------------------
# compile (ddtree.py:199-256)
# ----------------------------------------------------------------------------
def sliding_key_lo(positions, window: int) -> np.ndarray:
    """Lower bound of each row's visible prefix keys under a sliding window:
    query position - window + 1 (ddtree.py:276-281)."""
    return np.asarray(positions, np.int64) - (int(window) - 1)


def compile_tree(root_token: int, start: int, node_token_ids, node_depths, visibility, past_length: int,
                 mask_min: float):
    """Verify ids, position ids and the dense additive mask rows [N, past+N]."""
    N = 1 + len(node_token_ids)
    ids = np.empty(N, np.int64)
    ids[0] = root_token
    ids[1:] = node_token_ids
    pos = np.empty(N, np.int64)
    pos[0] = start
    pos[1:] = np.asarray(node_depths, np.int64) + start
    mask = np.zeros((N, past_length + N), np.float32)
    blk = np.full((N, N), mask_min, np.float32)
    blk[np.asarray(visibility, bool)] = 0.0
    mask[:, past_length:] = blk
    return ids, pos, mask


# ----------------------------------------------------------------------------
# acceptance (ddtree.py:290-301, model/utils.py:28-30, eagle3.py:46-79)
# ----------------------------------------------------------------------------
def argmax_rows(logits: np.ndarray) -> np.ndarray:
    """torch.argmax(dim=-1) restatement; bf16 given as uint16 bit patterns."""
    x = np.ascontiguousarray(logits)
    rows, V = x.shape
    out = np.empty(rows, np.int64)
    if x.dtype == np.uint16:
        lib().ora_argmax_bf16(_ptr(x), rows, V, V, _ptr(out))
    else:
        x = np.ascontiguousarray(x, np.float32)
        lib().ora_argmax_f32(_ptr(x), rows, V, V, _ptr(out))
    return out


def follow(parents, node_token_ids, posterior):
    parents = np.ascontiguousarray(parents, np.int32)
    toks = np.ascontiguousarray(node_token_ids, np.int64)
    post = np.ascontiguousarray(posterior, np.int64)
    n = len(toks)
    acc = np.zeros(n + 2, np.int64)
    nxt = np.zeros(1, np.int64)
    na = lib().ora_follow(_ptr(parents), _ptr(toks), n, _ptr(post), _ptr(acc), n + 2, _ptr(nxt))
    return [int(v) for v in acc[:na]], int(nxt[0])


def eagle3_posterior(posterior, draft_tokens, retrieve):
    post = np.ascontiguousarray(posterior, np.int64)
    dt = np.ascontiguousarray(draft_tokens, np.int64).reshape(-1)
    r = np.ascontiguousarray(retrieve, np.int64)
    leaves, W = r.shape
    best = np.zeros(1, np.int64)
    alen = np.zeros(1, np.int64)
    acc = np.zeros(W, np.int64)
    samp = np.zeros(1, np.int64)
    lib().ora_eagle3_posterior(_ptr(post), _ptr(dt), len(dt), _ptr(r), leaves, W, _ptr(best), _ptr(alen),
                               _ptr(acc), _ptr(samp))
    a = int(alen[0])
    return int(best[0]), a, int(samp[0]), [int(v) for v in acc[: a + 1]]


def compact_tail(cache: np.ndarray, past_length: int, keep) -> np.ndarray:
    """``compact_tail_inplace`` restatement (ddtree.py:61-88, 304-320), on a copy."""
    out = np.array(cache, copy=True)
    S = out.shape[-2]
    cur = S - past_length
    keep = np.asarray(keep, np.int64)
    if cur <= 0 or len(keep) == 0 or len(keep) == cur:
        return out
    tail = out[..., past_length:past_length + cur, :]
    kept = tail[..., keep, :].copy()
    out[..., past_length:past_length + len(keep), :] = kept
    return out


def commit(verify_ids, accepted, next_token: int, output_ids: np.ndarray, start: int, hidden=None):
    """The commit step of a round (ddtree.py:534-548), on copies:
    ``output_ids[..., start:start+n] = verify_ids[..., accepted]``, the bonus
    token at ``start + n``, and the accepted rows of the verify hidden
    features (``index_select(1, accepted)``)."""
    acc = np.asarray(accepted, np.int64)
    out = np.array(output_ids, copy=True)
    n = len(acc)
    out[..., start:start + n] = np.asarray(verify_ids)[..., acc]
    out[..., start + n] = next_token
    sel = None if hidden is None else np.asarray(hidden)[..., acc, :].copy()
    return out, sel


# ----------------------------------------------------------------------------
# verify attention reference (HF sdpa path: softmax(QK^T*scale + mask) V)
# ----------------------------------------------------------------------------
def tree_attention_ref(q, k, v, past_length: int, visibility, scale: float, key_lo=None):
    """float32/float64 attention with the reference's tree mask.

    q: [N, Hq, D]; k, v: [Hkv, S, D] with S = past_length + N; visibility: bool [N, N].
    key_lo (optional, [N]): the sliding-window layers' mask (ddtree.py:276-283),
    prefix key j hidden from row t when j < key_lo[t].
    Returns [N, Hq, D] float64.
    """
    q = np.asarray(q, np.float64)
    k = np.asarray(k, np.float64)
    v = np.asarray(v, np.float64)
    N, Hq, D = q.shape
    Hkv, S, _ = k.shape
    g = Hq // Hkv
    allowed = np.ones((N, S), bool)
    allowed[:, past_length:past_length + N] = np.asarray(visibility, bool)
    allowed[:, past_length + N:] = False
    if key_lo is not None:
        allowed[:, :past_length] &= np.arange(past_length)[None, :] >= np.asarray(key_lo, np.int64)[:, None]
    out = np.zeros((N, Hq, D), np.float64)
    for h in range(Hq):
        kh = k[h // g]
        vh = v[h // g]
        s = q[:, h, :] @ kh.T * scale
        s = np.where(allowed, s, -np.inf)
        s = s - s.max(axis=1, keepdims=True)
        p = np.exp(s)
        p /= p.sum(axis=1, keepdims=True)
        out[:, h, :] = p @ vh
    return out
