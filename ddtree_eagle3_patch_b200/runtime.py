"""Host-side plumbing shared by the decode loops (``ddtree_generate``,
``eagle3_generate``): stage timing on CUDA events, routing a target's
attention to the tree kernel, the verify-mask stand-in that carries the
packed tree bits, and the per-round host read-back.

The reference times every stage with ``cuda_time()``, a device synchronize
plus ``perf_counter`` (dflash.py:146-148), about a dozen host syncs per
round.  Here each stage boundary records a CUDA event instead; the events
are resolved once, after the loop, so a round has exactly one host wait:
the read-back of the accepted count that the host needs to size the next
round.
"""
from __future__ import annotations

from contextlib import contextmanager

import torch

from . import kernels


def empty_stage_times(stage_names) -> dict:
    """{stage: 0.0} for every stage name (dflash.py:151-152)."""
    return {name: 0.0 for name in stage_names}


class EventClock:
    """Stage and round timing on CUDA events of the current stream.

    ``mark()`` records an event and returns it; ``span(stage, a, b)`` books
    the time between two marks to a stage; ``resolve()`` synchronizes once
    and returns the per-stage sums in seconds.  Events are pooled."""

    def __init__(self, device: torch.device):
        self.device = device
        self._pool: list = []
        self._used = 0
        self._spans: list = []

    def mark(self) -> torch.cuda.Event:
        if self._used == len(self._pool):
            self._pool.append(torch.cuda.Event(enable_timing=True))
        ev = self._pool[self._used]
        self._used += 1
        ev.record(torch.cuda.current_stream(self.device))
        return ev

    def span(self, stage: str, a: torch.cuda.Event, b: torch.cuda.Event) -> None:
        self._spans.append((stage, a, b))

    def resolve(self, stage_times: dict) -> dict:
        if self._used:
            self._pool[self._used - 1].synchronize()
        for stage, a, b in self._spans:
            stage_times[stage] = stage_times.get(stage, 0.0) + a.elapsed_time(b) / 1000.0
        return stage_times

    @staticmethod
    def seconds(a: torch.cuda.Event, b: torch.cuda.Event) -> float:
        b.synchronize()
        return a.elapsed_time(b) / 1000.0


def _text_configs(model):
    cfg = getattr(model, "config", None)
    out = []
    if cfg is not None:
        out.append(cfg)
        for name in ("text_config", "decoder"):
            sub = getattr(cfg, name, None)
            if sub is not None and sub is not cfg and hasattr(sub, "_attn_implementation"):
                out.append(sub)
    return out


@contextmanager
def tree_attention_for(target):
    """Route ``target``'s attention layers to the tree-verify kernel for the
    duration of a decode call, then restore the implementation it had.  The
    reference requires the target to be loaded with SDPA so that its 4-D
    tree mask is honoured (benchmark.py:102-105); the tree kernel honours the
    same mask, given as packed bits."""
    from .attention import ATTN_NAME, register
    register()
    configs = _text_configs(target)
    saved = [c._attn_implementation for c in configs]
    try:
        for c in configs:
            c._attn_implementation = ATTN_NAME
        yield
    finally:
        for c, s in zip(configs, saved):
            c._attn_implementation = s


class TreeMask:
    """Builds the ``attention_mask`` argument of a verify forward without a
    dense mask: a zero-stride [1, 1, N, past + N] view that carries the
    packed ancestor bits (``ddtree_bits``) and the prefix length
    (``ddtree_past``), which the registered attention function reads.  HF
    passes a 4-D mask through to the attention layers untouched."""

    def __init__(self, dtype: torch.dtype, device: torch.device):
        self._zero = torch.zeros((1, 1, 1, 1), dtype=dtype, device=device)

    def __call__(self, bits: torch.Tensor, past: int, n: int, key_lo: torch.Tensor | None = None) -> torch.Tensor:
        m = self._zero.expand(1, 1, n, past + n)
        m.ddtree_bits = bits
        m.ddtree_past = int(past)
        if key_lo is not None:
            m.ddtree_key_lo = key_lo
        return m

    def static(self, bits: torch.Tensor, past_dev: torch.Tensor, past_max: int, n: int,
               workspace: torch.Tensor) -> torch.Tensor:
        """The stand-in for a captured verify forward: the prefix length is
        the int32 device scalar ``past_dev`` (at most ``past_max``), read by
        the attention kernel at run time, and the attention uses the
        caller's ``workspace`` (which the graph keeps alive)."""
        m = self._zero.expand(1, 1, n, past_max + n)
        m.ddtree_bits = bits
        m.ddtree_past_dev = past_dev
        m.ddtree_past_max = int(past_max)
        m.ddtree_workspace = workspace
        return m


class Readback:
    """One pinned host buffer per decode call and one event: the round's
    only host wait reads the accept info and the newly written tokens."""

    def __init__(self, n: int, device: torch.device):
        self.host = torch.empty((n,), dtype=torch.int64, pin_memory=True)
        self.event = torch.cuda.Event()
        self.device = device

    def fetch(self, pieces) -> list:
        """Copy each (device tensor, count) piece into the pinned buffer
        (int64), wait once, return host lists."""
        off = 0
        spans = []
        for t, n in pieces:
            if n > 0:
                self.host[off: off + n].copy_(t.reshape(-1)[:n], non_blocking=True)
            spans.append((off, n))
            off += n
        self.event.record(torch.cuda.current_stream(self.device))
        self.event.synchronize()
        flat = self.host[:off].tolist()
        return [flat[o: o + n] for o, n in spans]


def device_sample_seed(generator: torch.Generator | None = None) -> int:
    """Seed of the device sampler drawn from torch's CPU generator, so that
    ``torch.manual_seed`` makes sampled runs repeat (as it does for the
    reference's ``torch.multinomial``)."""
    return int(torch.randint(0, 2 ** 62, (1,), generator=generator).item())


def cache_tensors_for_compaction(cache):
    """K and V tensors of every initialised layer of a TreeAppendCache or
    DynamicCache, de-aliased (ddtree.py:335-367)."""
    from .ddtree import _cache_tensors
    tensors, ok = _cache_tensors(cache)
    if not ok:
        raise RuntimeError("Unsupported DynamicCache layout for DDTree cache compaction.")
    return tensors


def compact_on_device(cache, past_length: int, cur_len: int, keep: torch.Tensor, keep_count: torch.Tensor,
                      max_keep: int, tables: dict) -> None:
    """Keep rows ``past + keep[k]`` (k < keep_count, both on the device) of
    every cache tensor's appended window at ``past + k``: the in-place half
    of compact_dynamic_cache (ddtree.py:323-369) with the count left on the
    device.  Tensors sharing a layout go in one launch."""
    groups: dict = {}
    for t in cache_tensors_for_compaction(cache):
        groups.setdefault((t.device, t.dtype, tuple(t.shape), t.stride()), []).append(t)
    for key, group in groups.items():
        if key[2][-2] - past_length <= 0:
            continue
        table = tables.setdefault((key, len(group)), kernels.PointerTable())
        kernels.kv_compact(group, past_length, cur_len, keep, keep_count, max_keep, table=table)
