"""Drop-in replacements for the EAGLE3 verify/accept step of the reference's
``eagle3.py`` (kimwin2/ddtree_eagle3_patch):

  compile_eagle3_attention_mask   eagle3.py:28-43
  evaluate_eagle3_posterior       eagle3.py:46-79

The EAGLE3 tree path reuses the verify-attention kernel (through the masks
built here, which carry their packed ancestor bits) and the acceptance
kernel (argmax + path evaluation in one launch).
"""
from __future__ import annotations

import torch

from . import kernels
from .ddtree import _attach_bits


def compile_eagle3_attention_mask(tree_mask: torch.Tensor, past_length: int, dtype: torch.dtype,
                                  device: torch.device) -> torch.Tensor:
    """[1, 1, T, past+T] additive mask: past visible, tree block from the
    [.., T, T] tree mask (eagle3.py:28-43)."""
    tm = tree_mask.to(device=device, dtype=torch.bool)
    T = tm.shape[-1]
    mask = torch.zeros((1, 1, T, past_length + T), dtype=dtype, device=device)
    tm2 = tm.reshape(-1, T, T)[-1]
    bits = kernels.mask_to_bits(tm2, 0, T)
    kernels.tree_mask_fill(mask[0, 0], past_length, T, bits, 0, 0)
    _attach_bits(mask, bits, past_length)
    return mask


def evaluate_eagle3_posterior(logits: torch.Tensor, draft_tokens: torch.Tensor, retrieve_indices: torch.Tensor,
                              temperature: float):
    """Longest accepted path over ``retrieve_indices`` (eagle3.py:46-79).

    Returns ``(best_candidate, accept_length, sample_token, candidates,
    accepted_indices)`` with the reference's types: ints, a [1, 1] token
    tensor on the logits' device, the [leaves, width] candidate tokens and a
    list of tree indices."""
    device = logits.device
    retrieve_indices = retrieve_indices.to(device=device)
    padded = torch.cat([draft_tokens.to(device=device),
                        torch.full((1, 1), -1, dtype=draft_tokens.dtype, device=device)], dim=1)
    candidates = padded[0, retrieve_indices]
    if temperature < 1e-5:
        info, accepted, _ = kernels.eagle3_accept(logits, draft_tokens, retrieve_indices)
        info_h = info.cpu()
        best, accept_length, tok = int(info_h[0]), int(info_h[1]), int(info_h[2])
        accepted_indices = accepted[: accept_length + 1].cpu().tolist()
        sample_token = torch.full((1, 1), tok, dtype=torch.long, device=device)
        return best, accept_length, sample_token, candidates, accepted_indices
    # temperature > 0 keeps the reference's sampling semantics (model/utils.py:31-35)
    bsz, seq_len, vocab = logits.shape
    probs = torch.softmax(logits.view(-1, vocab) / temperature, dim=-1)
    node_posterior = torch.multinomial(probs, num_samples=1).view(bsz, seq_len)[0]
    gather = retrieve_indices.clamp(min=0)
    paths = node_posterior[gather[:, :-1]]
    valid = retrieve_indices[:, 1:] >= 0
    ok = (candidates[:, 1:] == paths) & valid
    lengths = ok.int().cumprod(dim=1).sum(dim=1)
    accept_length = int(lengths.max().item())
    best = 0 if accept_length == 0 else int(torch.argmax(lengths).item())
    accepted_indices = [int(i) for i in retrieve_indices[best, : accept_length + 1].tolist()]
    last = accepted_indices[-1]
    p_last = torch.softmax(logits[:, last, :] / temperature, dim=-1)
    sample_token = torch.multinomial(p_last, num_samples=1).view(1, 1)
    return best, accept_length, sample_token, candidates, accepted_indices
