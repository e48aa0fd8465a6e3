"""Seeded synthetic workloads for the DDTree hot path.

The reference benchmarks on public evaluation sets that are not available
offline; the hot-path workloads are defined on random inputs instead, and
these generators produce them deterministically (torch CPU generator, fixed
seeds) so tests, fixtures and the benchmark see the same bytes on every
machine with the same torch build.

* tree build + acceptance: draft logits [15, 151936] float32 ~ N(0,1) plus a
  +8 peak at one random token per row; node budgets 32 / 64; the target's
  greedy token at each node equals the draft top-1 token of the next depth
  with probability 0.7, else a uniform random token.
* verify attention at Qwen3-4B shape: 32 query / 8 KV heads, head_dim 128,
  bf16, a 4096-token prefix ~ N(0,1) (keys scaled by 1/sqrt(128)) and a
  64-node tree whose parents are uniform over earlier nodes (depth <= 16),
  36 layers, batch 1.
"""
from __future__ import annotations

import numpy as np
import torch

V_QWEN3 = 151936
DRAFT_ROWS = 15          # block_size 16 -> 15 draft positions
QWEN3_4B = dict(layers=36, hq=32, hkv=8, head_dim=128, hidden=2560, intermediate=9728, vocab=V_QWEN3)


def cfg1_logits(seed: int = 0, rows: int = DRAFT_ROWS, vocab: int = V_QWEN3, peak: float = 8.0) -> torch.Tensor:
    g = torch.Generator().manual_seed(seed)
    logits = torch.randn(rows, vocab, generator=g)
    peaks = torch.randint(0, vocab, (rows,), generator=g)
    logits[torch.arange(rows), peaks] += peak
    return logits


def deep_logits(seed: int = 1, peak: float = 16.0, rows: int = DRAFT_ROWS, vocab: int = V_QWEN3) -> torch.Tensor:
    """Same as ``cfg1_logits`` with a larger peak, which makes the top-1 chain
    dominate and the trees deep (exercises depths up to 15)."""
    return cfg1_logits(seed=seed, rows=rows, vocab=vocab, peak=peak)


def posterior_for_tree(node_token_ids: np.ndarray, node_depths: np.ndarray, top_ids: np.ndarray, vocab: int,
                       seed: int = 0, p_top1: float = 0.7) -> np.ndarray:
    """Greedy target token for each verify row (root + nodes).

    Row i sits at depth d_i (root: 0).  With probability ``p_top1`` its target
    token is the draft top-1 token of row d_i (the next depth), otherwise a
    uniform random token.
    """
    rs = np.random.RandomState(seed)
    depths = np.concatenate([[0], np.asarray(node_depths, np.int64)])
    L = top_ids.shape[0]
    out = np.empty(len(depths), np.int64)
    for i, d in enumerate(depths):
        if d < L and rs.rand() < p_top1:
            out[i] = int(top_ids[d, 0])
        else:
            out[i] = int(rs.randint(0, vocab))
    return out


def verify_logits_for_posterior(posterior: np.ndarray, vocab: int, seed: int = 0, peak: float = 20.0,
                                dtype=torch.bfloat16) -> torch.Tensor:
    """[N, V] target logits whose row-wise argmax is ``posterior``."""
    g = torch.Generator().manual_seed(seed)
    n = len(posterior)
    x = torch.randn(n, vocab, generator=g)
    x[torch.arange(n), torch.as_tensor(posterior)] = peak
    return x.to(dtype)


def random_tree(n_nodes: int, max_depth: int = 16, seed: int = 0):
    """Tree of 1 + n_nodes rows: each node's parent is uniform over the earlier
    rows, resampled until its depth is <= max_depth.  Returns (parents [N]
    with parents[0] = -1, depths [N], visibility bool [N, N])."""
    rs = np.random.RandomState(seed)
    N = n_nodes + 1
    parents = np.full(N, -1, np.int64)
    depths = np.zeros(N, np.int64)
    for i in range(1, N):
        while True:
            p = int(rs.randint(0, i))
            if depths[p] + 1 <= max_depth:
                break
        parents[i] = p
        depths[i] = depths[p] + 1
    vis = np.zeros((N, N), bool)
    vis[0, 0] = True
    for i in range(1, N):
        vis[i, :i] = vis[parents[i], :i]
        vis[i, i] = True
    return parents, depths, vis


def tree_attention_inputs(seed: int, past: int, n: int, hq: int, hkv: int, d: int, max_depth: int = 16):
    """float32 numpy inputs for one layer of tree-verify attention:
    q [n, hq, d]; k, v [hkv, past + n, d] (keys scaled by 1/sqrt(d)); the
    ancestor visibility of a random tree of n rows; the softmax scale."""
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(n, hq, d, generator=g)
    k = torch.randn(hkv, past + n, d, generator=g) / np.sqrt(d)
    v = torch.randn(hkv, past + n, d, generator=g)
    _, _, vis = random_tree(n - 1, max_depth=max_depth, seed=seed)
    return (q.numpy(), k.numpy(), v.numpy(), vis, float(d) ** -0.5)


# ----------------------------------------------------------------------------
# random-init models of the end-to-end decode configurations
# ----------------------------------------------------------------------------
TARGET_SHAPES = {
    # Qwen3-4B: 36 layers, hidden 2560, intermediate 9728, 32 q / 8 kv heads
    "qwen3-4b": dict(hidden_size=2560, intermediate_size=9728, num_hidden_layers=36, num_attention_heads=32,
                     num_key_value_heads=8, head_dim=128, vocab_size=V_QWEN3, tie_word_embeddings=True),
    # Qwen3-8B: 36 layers, hidden 4096, intermediate 12288, 32 q / 8 kv heads
    "qwen3-8b": dict(hidden_size=4096, intermediate_size=12288, num_hidden_layers=36, num_attention_heads=32,
                     num_key_value_heads=8, head_dim=128, vocab_size=V_QWEN3, tie_word_embeddings=False),
    # a small model whose every projection takes the decode kernels' fast
    # paths (multiples of 128 rows and 64 columns): for tests
    "qwen3-small": dict(hidden_size=256, intermediate_size=512, num_hidden_layers=4, num_attention_heads=4,
                        num_key_value_heads=2, head_dim=128, vocab_size=1024, tie_word_embeddings=False),
}


def target_config(shape: str = "qwen3-4b"):
    """Qwen3Config of a target shape (rope theta 1e6, 40960 positions)."""
    from transformers import Qwen3Config
    return Qwen3Config(max_position_embeddings=40960, rope_theta=1000000.0, rms_norm_eps=1e-6,
                       **TARGET_SHAPES[shape])


def dflash_config(target_cfg, num_layers: int = 5, block_size: int = 16, mask_token_id: int | None = None):
    """A DFlash block-diffusion draft of the target's width: ``num_layers``
    Qwen3 layers, context features from build_target_layer_ids(target
    layers, num_layers), the given block size and mask token (default the
    last vocabulary id)."""
    from transformers import Qwen3Config
    from .model import build_target_layer_ids
    t = target_cfg
    rope = dict(getattr(t, "rope_parameters", None) or {"rope_type": "default", "rope_theta": 1000000.0})
    cfg = Qwen3Config(hidden_size=t.hidden_size, intermediate_size=t.intermediate_size, num_hidden_layers=num_layers,
                      num_attention_heads=t.num_attention_heads, num_key_value_heads=t.num_key_value_heads,
                      head_dim=t.head_dim, vocab_size=t.vocab_size, max_position_embeddings=t.max_position_embeddings,
                      rope_parameters=rope, rms_norm_eps=t.rms_norm_eps)
    cfg.block_size = block_size
    cfg.num_target_layers = t.num_hidden_layers
    cfg.dflash_config = {
        "target_layer_ids": build_target_layer_ids(t.num_hidden_layers, num_layers),
        "mask_token_id": t.vocab_size - 1 if mask_token_id is None else mask_token_id,
    }
    return cfg


def build_decode_models(shape: str, device, dtype=torch.bfloat16, seed: int = 0, draft_layers: int = 5,
                        block_size: int = 16):
    """Random-init (HF initialisation, seeded) target and DFlash draft,
    created directly on ``device`` in ``dtype``."""
    from transformers import Qwen3ForCausalLM
    from .model import DFlashDraftModel
    tcfg = target_config(shape)
    dcfg = dflash_config(tcfg, draft_layers, block_size)
    old = torch.get_default_dtype()
    torch.manual_seed(seed)
    try:
        torch.set_default_dtype(dtype)
        with torch.device(device):
            target = Qwen3ForCausalLM(tcfg).eval()
            draft = DFlashDraftModel(dcfg).eval()
    finally:
        torch.set_default_dtype(old)
    return target.to(dtype), draft.to(dtype)


def random_prompt(length: int, vocab: int = V_QWEN3, seed: int = 0, exclude: int | None = None) -> torch.Tensor:
    """[1, length] uniform random token ids (never ``exclude``)."""
    g = torch.Generator().manual_seed(seed)
    hi = vocab if exclude is None else vocab - 1
    ids = torch.randint(0, hi, (1, length), generator=g)
    if exclude is not None:
        ids[ids >= exclude] += 1
    return ids
