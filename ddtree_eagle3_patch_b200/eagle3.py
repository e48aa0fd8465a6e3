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
    # temperature > 0: the reference draws every row once from
    # softmax(logits / T) (sample, model/utils.py:31-35), then the bonus
    # token once more from the last accepted row; both draws run on the
    # sampling kernel (Gumbel-max, seeded from torch's generator)
    node_posterior = kernels.sample(logits, temperature)[0]
    gather = retrieve_indices.clamp(min=0)
    paths = node_posterior[gather[:, :-1]]
    valid = retrieve_indices[:, 1:] >= 0
    ok = (candidates[:, 1:] == paths) & valid
    lengths = ok.int().cumprod(dim=1).sum(dim=1)
    accept_length = int(lengths.max().item())
    best = 0 if accept_length == 0 else int(torch.argmax(lengths).item())
    accepted_indices = [int(i) for i in retrieve_indices[best, : accept_length + 1].tolist()]
    last = accepted_indices[-1]
    sample_token = kernels.sample(logits[:, last: last + 1, :], temperature).view(1, 1)
    return best, accept_length, sample_token, candidates, accepted_indices


# ----------------------------------------------------------------------------
# The EAGLE3 decode loop
# ----------------------------------------------------------------------------
EAGLE3_STAGE_ORDER = ("draft", "verify", "commit")


def eagle3_target_layer_ids(target_config, draft_model) -> list[int]:
    """The draft's aux layer ids, else [2, L // 2, L - 3] (eagle3.py:14-18)."""
    if getattr(draft_model, "target_layer_ids", None) is not None:
        return list(draft_model.target_layer_ids)
    n = getattr(target_config, "num_hidden_layers")
    return [2, n // 2, n - 3]


def extract_eagle3_context_feature(hidden_states, target_layer_ids) -> torch.Tensor:
    """Concatenate the target hidden states at the given indices of HF's
    ``hidden_states`` (no +1 offset, unlike DFlash; eagle3.py:21-25)."""
    return torch.cat([hidden_states[i] for i in target_layer_ids], dim=-1)


@torch.inference_mode()
def eagle3_generate(model, target, input_ids: torch.Tensor, max_new_tokens: int, stop_token_ids,
                    temperature: float = 0.0):
    """EAGLE3 speculative decoding (eagle3.py:156-281), same arguments and
    ``SimpleNamespace`` result.

    ``model`` is the EAGLE3 draft (its ``topk_generate`` builds each round's
    depth x top-k tree and stays as it is); the target verifies the tree
    through the tree-attention kernel with the tree mask given as packed
    bits, with its KV cache preallocated, appended at a device-side offset
    and compacted in one launch; at temperature 0 the accept kernel takes
    every verify row's argmax and picks the longest accepted path of
    ``retrieve_indices`` (evaluate_eagle3_posterior).  From the third round
    the verify forward is replayed from a CUDA graph (DDTREE_EAGER=1 runs
    it eagerly).  One host read per round returns the accepted path."""
    import os
    from contextlib import nullcontext
    from types import SimpleNamespace

    from .cache import TreeAppendCache
    from .fused_layers import fused_decoder_layers
    from .runtime import EventClock, Readback, TreeMask, empty_stage_times, tree_attention_for

    device = target.device
    P = input_ids.shape[1]
    max_length = P + max_new_tokens
    T = model.total_tokens + 1
    position_ids = torch.arange(max_length + model.total_tokens + 8, device=device).unsqueeze(0)
    stop_ids = None if stop_token_ids is None else set(int(t) for t in stop_token_ids)
    layer_ids = eagle3_target_layer_ids(target.config, model)
    use_graph = os.environ.get("DDTREE_EAGER", "0") != "1"
    fuse = os.environ.get("DDTREE_FUSED", "1") != "0"
    cache = TreeAppendCache(max_length + T + 9, config=target.config)
    clock = EventClock(device)
    stage_times = empty_stage_times(EAGLE3_STAGE_ORDER)
    readback = Readback(8 + 2 * T, device)
    rs_host = torch.zeros((4,), dtype=torch.int32, pin_memory=True)
    rs = torch.zeros((4,), dtype=torch.int32, device=device)
    ids_buf = torch.empty((1, T), dtype=torch.int64, device=device)
    pos_buf = torch.empty((1, T), dtype=torch.int64, device=device)
    bits_buf = torch.zeros((T, (T + 31) // 32), dtype=torch.int32, device=device)
    retrieve_buf = None
    model.reset_kv()
    graph = None
    graph_kernels = replays = 0

    with tree_attention_for(target), (fused_decoder_layers(target) if fuse else nullcontext()), \
            kernels.pdl(fuse and os.environ.get("DDTREE_PDL", "1") != "0"):
        ev_prefill = clock.mark()
        output = target(input_ids, position_ids=position_ids[:, :P], past_key_values=cache, use_cache=True,
                        logits_to_keep=1, output_hidden_states=True)
        next_root = kernels.sample(output.logits, temperature).to(device)
        target_hidden = extract_eagle3_context_feature(output.hidden_states, layer_ids).to(model.device)
        ev_first = clock.mark()
        # static mode: appends at rs[0], attention prefix from rs[0]
        past_max = cache.capacity - T
        t_cfg = target.config
        ws = kernels.attention_workspace(T, t_cfg.num_attention_heads, t_cfg.num_key_value_heads, past_max, device)
        cache.set_static(rs[0:1])
        mask = TreeMask(target.dtype, device).static(bits_buf, rs[0:1], past_max, T, ws)

        def verify():
            out = target(ids_buf, position_ids=pos_buf, attention_mask=mask, past_key_values=cache, use_cache=True,
                         output_hidden_states=True)
            return out.logits, extract_eagle3_context_feature(out.hidden_states, layer_ids)

        ev0 = clock.mark()
        draft_tokens, retrieve_indices, tree_mask, tree_position_ids = model.topk_generate(
            target_hidden, torch.cat((input_ids, next_root), dim=1).to(model.device))
        ev1 = clock.mark()
        clock.span("draft", ev0, ev1)
        committed = [int(t) for t in input_ids[0].tolist()]
        committed_dev = input_ids.clone()
        ev_decode = clock.mark()
        ev_round_clock = ev_decode
        acceptance, round_ends = [], []
        rnd = 0
        while len(committed) < max_length:
            past = len(committed)
            rs_host[0] = past
            rs.copy_(rs_host, non_blocking=True)
            ids_buf.copy_(draft_tokens.to(device).reshape(1, T))
            torch.add(tree_position_ids.to(device).reshape(1, T), past, out=pos_buf)
            tm = tree_mask.to(device=device).reshape(-1, T, T)[-1].to(torch.bool)
            kernels.mask_to_bits(tm, 0, T, out=bits_buf)
            ev2 = clock.mark()
            if graph is not None:
                graph[0].replay()
                replays += 1
                logits, features = graph[1], graph[2]
            else:
                logits, features = verify()
            ev3 = clock.mark()
            clock.span("verify", ev2, ev3)
            r_dev = retrieve_indices.to(device=device, dtype=torch.int64)
            if temperature < 1e-5:
                info, accepted, _ = kernels.eagle3_accept(logits, draft_tokens.to(device), r_dev)
                got = readback.fetch([(info, 3), (accepted, r_dev.shape[1])])
                best, acc_len, sample_tok = got[0]
                acc_idx = got[1][: acc_len + 1]
            else:
                best, acc_len, sample_token, _, acc_idx = evaluate_eagle3_posterior(
                    logits, draft_tokens.to(device), r_dev, temperature)
                sample_tok = int(sample_token.reshape(-1)[0])
            remaining = max_length - len(committed)
            acc_idx = acc_idx[:remaining]
            n_acc = len(acc_idx)
            keep = torch.tensor(acc_idx, dtype=torch.int64, device=device)
            draft_row = draft_tokens.to(device).reshape(-1)
            accepted_tokens = draft_row.index_select(0, keep)
            committed_dev = torch.cat([committed_dev, accepted_tokens.view(1, -1)], dim=1)
            count = torch.full((1,), n_acc, dtype=torch.int64, device=device)
            from .runtime import compact_on_device
            compact_on_device(cache, past, T, keep, count, n_acc, {})
            accepted_hidden = features.index_select(1, keep).to(model.device)
            new_tokens = [int(t) for t in draft_row.index_select(0, keep).tolist()]
            committed += new_tokens
            acceptance.append(n_acc)
            ev4 = clock.mark()
            clock.span("commit", ev3, ev4)
            round_ends.append(ev4)
            rnd += 1
            if n_acc == remaining or (stop_ids is not None and any(t in stop_ids for t in new_tokens)):
                break
            if use_graph and graph is None and rnd == 2:
                from ._lib import load
                lib = load()
                n0 = lib.ddt_launch_count()
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g):
                    g_logits, g_features = verify()
                graph_kernels = lib.ddt_launch_count() - n0
                graph = (g, g_logits, g_features)
            ev5 = clock.mark()
            sample_dev = torch.full((1, 1), sample_tok, dtype=torch.int64, device=model.device)
            draft_tokens, retrieve_indices, tree_mask, tree_position_ids = model.topk_generate(
                accepted_hidden, torch.cat((committed_dev.to(model.device), sample_dev), dim=1))
            ev6 = clock.mark()
            clock.span("draft", ev5, ev6)
        ev_end = clock.mark()
        graph = None

    output_ids = committed_dev[:, :max_length]
    if stop_ids is not None:
        for i, t in enumerate(output_ids[0, P:].tolist()):
            if t in stop_ids:
                output_ids = output_ids[:, : P + i + 1]
                break
    num_output_tokens = output_ids.shape[1] - P
    clock.resolve(stage_times)
    total = clock.seconds(ev_decode, ev_end)
    return SimpleNamespace(
        output_ids=output_ids.cpu(),
        num_input_tokens=P,
        num_output_tokens=num_output_tokens,
        time_to_first_token=clock.seconds(ev_prefill, ev_first),
        time_per_output_token=total / max(num_output_tokens, 1),
        acceptance_lengths=acceptance,
        decode_rounds=len(acceptance),
        stage_times=stage_times,
        round_timestamps=[clock.seconds(ev_round_clock, e) for e in round_ends],
        graph_rounds=replays,
        graph_kernels=graph_kernels,
    )
