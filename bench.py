"""Benchmark of DDTree decoding and its per-step draft-tree hot path on B200.

Two workloads (``--workload``):

decode (default): end-to-end DDTree decoding at the Qwen3-4B shape, B=1.
One step = one ``ddtree_generate`` call: a random-init Qwen3-4B target
(36 layers, hidden 2560, intermediate 9728, 32/8 heads, vocab 151936, bf16)
with a random-init 5-layer DFlash draft of the same width, block size 16,
node budget 32, a 512-token uniform random prompt, 1024 new tokens, greedy.
``value`` is whole-job generated tokens/s over the K calls (prefill
included), prompts resident on the device; ``e2e`` passes the prompt from
pinned host memory and returns ids to the host inside the timed region.
With N GPUs every rank decodes its own prompts (the reference shards
prompts by rank) and one NCCL all-gather of a fixed-size counter tensor
collects tokens, rounds and times.

step: one step = the device work of one DDTree decoding round outside the
model GEMMs, at the Qwen3-4B verify shape:
  1. tree build from draft logits [15, 151936] fp32, node budget 64
     (top-k + log-normaliser + best-first expansion + ancestor bitmask);
  2. tree-masked verify attention for 36 layers: 32 query / 8 KV heads,
     head_dim 128, bf16, 4096-token prefix + 65 verify rows (one launch per
     layer: in a real round each layer's queries come from the model);
  3. greedy acceptance on verify logits [65, 151936] bf16 (argmax + walk);
  4. in-place compaction of the accepted rows in 72 cache tensors.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

``value`` is whole-job steps/s with inputs resident in HBM (CUDA-graph
replays, CUDA events, max over ranks); ``e2e`` is the same metric through
the public API with host buffers (pinned host inputs copied in and the
accept result copied out every step).  ``--impl reference`` times the
reference's CPU path (a port making the reference's library calls) on the
host cores.  Multi-GPU: one process per GPU, independent replicas (the
reference shards prompts across GPUs; the hot path has no exchange step),
NCCL only for the timing barrier and the max over ranks.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

import numpy as np
import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

LAYERS, HQ, HKV, HD = 36, 32, 8, 128
ROWS, VOCAB, BUDGET, PAST = 15, 151936, 64, 4096
N_VERIFY = BUDGET + 1
QUERY_CHUNK = 9   # layers of queries per host-to-device copy in the e2e leg
E2E_MIN_STEPS = 300
DEC_SHAPE, DEC_PROMPT, DEC_NEW_TOKENS, DEC_BUDGET, DEC_BLOCK, DEC_DRAFT_LAYERS = "qwen3-4b", 512, 1024, 32, 16, 5
DEC_METRIC = "decode tok/s (Qwen3-4B shape, B=1)"
DEC_UNIT = "tok/s"
METRIC = "tree build+verify steps/s (DDTree hot-path step, Qwen3-4B shape, B=1)"
UNIT = "steps/s"
WORKLOAD = (f"tree build [{ROWS}x{VOCAB}] fp32 budget {BUDGET} + tree-verify attention {LAYERS} layers "
            f"(hq {HQ}, hkv {HKV}, d {HD}, prefix {PAST} + {N_VERIFY} rows, bf16) + greedy accept "
            f"[{N_VERIFY}x{VOCAB}] bf16 + KV compaction of {2 * LAYERS} tensors")


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--workload", choices=["decode", "decode-dp", "step"], default="decode",
                    help="decode: Qwen3-4B, 512-token prompt, 1024 tokens, budget 32 (the headline); decode-dp: "
                         "Qwen3-8B, --prompts prompts of 256-2048 tokens sharded over the GPUs, 512 tokens, "
                         "budget 64; step: the per-round hot path alone")
    ap.add_argument("--prompts", type=int, default=0, help="decode-dp: prompts in the list (default 64)")
    ap.add_argument("--steps", type=int, default=None, help="timed steps (decode: 3 calls; step: 200)")
    ap.add_argument("--warmup", type=int, default=None, help="untimed steps (default 3 / 5)")
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cuda-profiler-range", action="store_true",
                    help="decode: bracket the timed calls with cudaProfilerStart/Stop (for "
                         "ncu --profile-from-start off launch lists of exactly the timed rounds)")
    ap.add_argument("--kernel", choices=["attention", "tree_build", "expand", "accept", "compact", "sample", "gemm"],
                    default=None,
                    help="launch only this kernel of the step (warmup + steps times, eager) and print its "
                         "average CUDA-event time; used for small profiler captures")
    ap.add_argument("--new-tokens", type=int, default=DEC_NEW_TOKENS, help="decode: tokens per call")
    args = ap.parse_args()
    if args.steps is None:
        args.steps = 3 if args.workload == "decode" and not args.kernel else 200
    if args.warmup is None:
        args.warmup = 3 if args.workload == "decode" and not args.kernel else 5
    return args


def dist_env():
    rank = int(os.environ.get("RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", 1))
    local = int(os.environ.get("LOCAL_RANK", 0))
    return rank, world, local


def init_dist(world: int, backend: str):
    import datetime
    import torch.distributed as dist
    if world > 1 and not dist.is_initialized():
        dist.init_process_group(backend=backend, timeout=datetime.timedelta(seconds=120))
    return dist


# ----------------------------------------------------------------------------
# clocks sampled during the timed region
# ----------------------------------------------------------------------------
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.path = Path(f"/tmp/ddt_clocks_{os.getpid()}.csv")

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
            time.sleep(0.3)
        except (OSError, FileNotFoundError):
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        if self.proc is None or not self.path.exists():
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unavailable"]}
        sms, mx, reasons = [], None, set()
        for line in self.path.read_text().splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sms.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for name, val in zip(("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"),
                                 parts[5:9]):
                if val.lower() == "active":
                    reasons.add(name)
        self.path.unlink(missing_ok=True)
        return {"sm_mhz": statistics.median(sms) if sms else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sms)}


# ----------------------------------------------------------------------------
# our implementation
# ----------------------------------------------------------------------------
class Workload:
    """Device-resident inputs of the step (two alternating input sets for the
    logits; 613 MB of KV per step keeps every step's working set above L2)."""

    def __init__(self, device, seed: int):
        from ddtree_eagle3_patch_b200.synthetic import cfg1_logits, posterior_for_tree, verify_logits_for_posterior
        g = torch.Generator().manual_seed(seed)
        self.device = device
        self.draft = [cfg1_logits(seed=seed + i).to(device) for i in range(2)]
        self.kcap = PAST + N_VERIFY
        # one allocation per cache tensor kind, as a static KV cache holds it:
        # every layer's [HKV, kcap, HD] is a view, so the new tree rows of all
        # layers are one strided region (one 2D copy in the e2e path)
        self.k_all = torch.empty((LAYERS, HKV, self.kcap, HD), dtype=torch.bfloat16, device=device)
        self.v_all = torch.empty((LAYERS, HKV, self.kcap, HD), dtype=torch.bfloat16, device=device)
        self.ks = list(self.k_all.unbind(0))
        self.vs = list(self.v_all.unbind(0))
        gd = torch.Generator(device=device).manual_seed(seed)
        for t in self.ks:
            t.normal_(generator=gd).mul_(HD ** -0.5)
        for t in self.vs:
            t.normal_(generator=gd)
        self.qs = [torch.randn((N_VERIFY, HQ, HD), generator=g).to(torch.bfloat16).to(device) for _ in range(LAYERS)]
        self.outs = [torch.empty((N_VERIFY, HQ, HD), dtype=torch.bfloat16, device=device) for _ in range(LAYERS)]
        # verify logits whose argmax follows the configuration-1 posterior rule
        from ddtree_eagle3_patch_b200 import kernels
        tree = kernels.tree_build(self.draft[0], BUDGET)
        n = int(tree.info[0])
        post = posterior_for_tree(tree.node_token_ids[:n].cpu().numpy(), tree.node_depths[:n].cpu().numpy(),
                                  tree.top_ids.cpu().numpy(), VOCAB, seed=seed)
        self.verify = [verify_logits_for_posterior(post, VOCAB, seed=seed + i).to(device) for i in range(2)]
        self.scale = HD ** -0.5


def gpu_step(w: Workload, i: int, tree_out, accept_bufs, table):
    from ddtree_eagle3_patch_b200 import kernels
    tree = kernels.tree_build(w.draft[i % 2], BUDGET, out=tree_out)
    for layer in range(LAYERS):
        kernels.tree_attention(w.qs[layer], w.ks[layer], w.vs[layer], PAST, tree.visibility, w.scale,
                               out=w.outs[layer])
    acc, info, post = kernels.tree_accept(w.verify[i % 2], tree.parents, tree.node_token_ids, tree.info,
                                          max_accept=ROWS + 1, accepted=accept_bufs[0], accept_info=accept_bufs[1],
                                          posterior=accept_bufs[2])
    kernels.kv_compact([t for pair in zip(w.ks, w.vs) for t in pair], PAST, N_VERIFY, acc, info[:1], ROWS + 1,
                       table=table)
    return info


def run_ours(args, rank, world, local):
    from ddtree_eagle3_patch_b200 import kernels
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    dist = init_dist(world, "nccl")
    w = Workload(device, seed=1000 + rank)
    tree_out = kernels.DeviceTree.allocate(ROWS, VOCAB, BUDGET, device)
    accept_bufs = (torch.zeros(ROWS + 1, dtype=torch.int64, device=device),
                   torch.zeros(2, dtype=torch.int64, device=device),
                   torch.empty(N_VERIFY, dtype=torch.int64, device=device))
    table = kernels.PointerTable()
    stream = torch.cuda.Stream(device)
    # warm-up eagerly (allocates workspaces, sets kernel attributes)
    with torch.cuda.stream(stream):
        for i in range(max(args.warmup, 1)):
            gpu_step(w, i, tree_out, accept_bufs, table)
    torch.cuda.synchronize()
    status = kernels.attention_status(device)
    # capture one step per input set
    graphs = []
    for i in range(2):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            gpu_step(w, i, tree_out, accept_bufs, table)
        graphs.append(g)
    for i in range(args.warmup):
        graphs[i % 2].replay()
    torch.cuda.synchronize()
    launches_per_step = 1 + LAYERS * (2 if _attention_splits() > 1 else 1) + 1 + 1

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    # timed region: K graph replays
    with ClockSampler(_physical_index(local)) as clocks:
        barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(stream):
            e0.record(stream)
            for i in range(args.steps):
                graphs[i % 2].replay()
            e1.record(stream)
        barrier()
    elapsed_ms = e0.elapsed_time(e1)
    clock = clocks.summary()
    ms = torch.tensor([elapsed_ms], dtype=torch.float64, device=device)
    if world > 1:
        dist.all_reduce(ms, op=dist.ReduceOp.MAX)
    elapsed_ms = float(ms.item())
    ms_per_step = elapsed_ms / args.steps
    value = world * args.steps / (elapsed_ms / 1e3)

    # dominant kernel: the per-layer attention op, timed alone (graph of 36 layers)
    ga = torch.cuda.CUDAGraph()
    with torch.cuda.graph(ga, stream=stream):
        for layer in range(LAYERS):
            kernels.tree_attention(w.qs[layer], w.ks[layer], w.vs[layer], PAST, tree_out.visibility, w.scale,
                                   out=w.outs[layer])
    for _ in range(3):
        ga.replay()
    torch.cuda.synchronize()
    reps = max(5, args.steps // 2)
    a0, a1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        a0.record(stream)
        for _ in range(reps):
            ga.replay()
        a1.record(stream)
    torch.cuda.synchronize()
    attn_us = a0.elapsed_time(a1) * 1e3 / (reps * LAYERS)
    kv_bytes = 2 * HKV * (PAST + N_VERIFY) * HD * 2
    qo_bytes = 2 * N_VERIFY * HQ * HD * 2
    alg_bytes = kv_bytes + qo_bytes
    peaks = _peaks()
    achieved = alg_bytes / (attn_us * 1e-6) / 1e9
    roofline = {"bound": "hbm", "kernel": "tree_attn_split_kernel + combine_kernel (one layer)",
                "achieved": round(achieved, 1), "peak": peaks["hbm_gbs"], "peak_source": peaks["source"],
                "unit": "GB/s", "frac": round(achieved / peaks["hbm_gbs"], 4),
                "traffic": _profiled_traffic(), "algorithmic_bytes": alg_bytes, "us_per_launch": round(attn_us, 3)}

    # end to end through the public API with host buffers
    e2e = run_e2e(args, w, device, stream, tree_out, table, world, dist)

    status |= kernels.attention_status(device)
    out = None
    if rank == 0:
        out = {
            "metric": METRIC, "value": round(value, 2), "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms_per_step, 5), "us_per_step": round(ms_per_step * 1e3, 2),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded; random-init inputs of the Qwen3-4B verify shape)",
            "config": {"workload": WORKLOAD, "parallelism": f"replicas x{world} (prompt-sharded data parallel)",
                       "l2": "inputs larger than L2 (613 MB of KV per step)", "cuda_graph": True},
            "roofline": roofline, "e2e": e2e, "gpu_launches": launches_per_step * args.steps,
            "clocks": clock, "attention_status": status,
        }
        if world == 1 and not args.no_cpu_baseline:
            out["cpu_baseline"] = cpu_baseline(sample_steps=2, attn_layers=4)
    if world > 1:
        dist.barrier()
    del graphs, ga
    return out


def run_e2e(args, w: Workload, device, stream, tree_out, table, world, dist):
    """Per step: pinned host draft logits, per-layer queries and new tree K/V
    rows, and verify logits are copied in; the accept result is copied out.
    The copies run on a copy stream in the order the step needs them: draft
    logits, the new K and V rows of every layer and head in one contiguous
    copy to a staging buffer (the compute stream scatters them into the
    cache rows), the queries in chunks of QUERY_CHUNK layers, then the
    verify logits.  The compute stream waits on an event just before each
    use, so the host-to-device traffic overlaps the kernels (a step still
    contains all of its own copies: the next step starts after this one's
    result is back on the host).  Few, large copies keep the copy engine at
    its bandwidth: a 2D copy of the 288 strided (layer, head) rows cost
    ~1.5 us per row and 36 per-layer query copies ~5 us each on B200."""
    from ddtree_eagle3_patch_b200 import kernels
    h_draft = [t.cpu().pin_memory() for t in w.draft]
    h_verify = [t.cpu().pin_memory() for t in w.verify]
    h_q = torch.stack([q.cpu() for q in w.qs]).pin_memory()
    # [2, layers, heads, tree rows, dim]: new K rows, then new V rows
    h_kvt = torch.stack([torch.stack([t[:, PAST:].cpu() for t in w.ks]),
                         torch.stack([t[:, PAST:].cpu() for t in w.vs])]).pin_memory()
    d_kvt = torch.empty(h_kvt.shape, dtype=torch.bfloat16, device=device)
    d_draft = torch.empty_like(w.draft[0])
    d_verify = torch.empty_like(w.verify[0])
    d_q = torch.empty((LAYERS, N_VERIFY, HQ, HD), dtype=torch.bfloat16, device=device)
    h_result = torch.empty(ROWS + 3, dtype=torch.int64).pin_memory()
    acc_bufs = (torch.zeros(ROWS + 1, dtype=torch.int64, device=device),
                torch.zeros(2, dtype=torch.int64, device=device),
                torch.empty(N_VERIFY, dtype=torch.int64, device=device))
    h2d = h_draft[0].numel() * 4 + h_verify[0].numel() * 2 + h_q.numel() * 2 + h_kvt.numel() * 2
    d2h = h_result.numel() * 8
    copy_stream = torch.cuda.Stream(device)
    ev_draft, ev_kv, ev_verify = torch.cuda.Event(), torch.cuda.Event(), torch.cuda.Event()
    chunks = [(c, min(c + QUERY_CHUNK, LAYERS)) for c in range(0, LAYERS, QUERY_CHUNK)]
    ev_chunk = [torch.cuda.Event() for _ in chunks]

    def step(i):
        with torch.cuda.stream(copy_stream):
            d_draft.copy_(h_draft[i % 2], non_blocking=True)
            ev_draft.record(copy_stream)
            d_kvt.copy_(h_kvt, non_blocking=True)
            ev_kv.record(copy_stream)
            for (c0, c1), ev in zip(chunks, ev_chunk):
                d_q[c0:c1].copy_(h_q[c0:c1], non_blocking=True)
                ev.record(copy_stream)
            d_verify.copy_(h_verify[i % 2], non_blocking=True)
            ev_verify.record(copy_stream)
        with torch.cuda.stream(stream):
            stream.wait_event(ev_draft)
            tree = kernels.tree_build(d_draft, BUDGET, out=tree_out)
            stream.wait_event(ev_kv)
            w.k_all[:, :, PAST:PAST + N_VERIFY].copy_(d_kvt[0])
            w.v_all[:, :, PAST:PAST + N_VERIFY].copy_(d_kvt[1])
            for layer in range(LAYERS):
                if layer % QUERY_CHUNK == 0:
                    stream.wait_event(ev_chunk[layer // QUERY_CHUNK])
                kernels.tree_attention(d_q[layer], w.ks[layer], w.vs[layer], PAST, tree.visibility, w.scale,
                                       out=w.outs[layer])
            stream.wait_event(ev_verify)
            acc, info, _ = kernels.tree_accept(d_verify, tree.parents, tree.node_token_ids, tree.info,
                                               max_accept=ROWS + 1, accepted=acc_bufs[0], accept_info=acc_bufs[1],
                                               posterior=acc_bufs[2])
            kernels.kv_compact([t for pair in zip(w.ks, w.vs) for t in pair], PAST, N_VERIFY, acc, info[:1],
                               ROWS + 1, table=table)
            h_result[: ROWS + 1].copy_(acc, non_blocking=True)
            h_result[ROWS + 1:].copy_(info, non_blocking=True)
        stream.synchronize()
        return int(h_result[ROWS + 1])

    for i in range(max(args.warmup, 1)):
        step(i)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    # at least E2E_MIN_STEPS steps (~0.35 s): each step waits on the host, so
    # a short run is dominated by host scheduling noise
    n_steps = max(args.steps, E2E_MIN_STEPS)
    e0.record(stream)
    for i in range(n_steps):
        step(i)
    e1.record(stream)
    torch.cuda.synchronize()
    ms = torch.tensor([e0.elapsed_time(e1)], dtype=torch.float64, device=device)
    if world > 1:
        dist.all_reduce(ms, op=dist.ReduceOp.MAX)
    el = float(ms.item())
    return {"value": round(world * n_steps / (el / 1e3), 2), "unit": UNIT, "h2d_bytes_per_step": int(h2d),
            "d2h_bytes_per_step": int(d2h), "ms_per_step": round(el / n_steps, 4), "steps": n_steps,
            "api": "ddtree_eagle3_patch_b200.kernels (C-ABI via ctypes), eager launches, copies on a copy stream",
            "copies_per_step": 4 + len(chunks)}


def _attention_splits() -> int:
    from ddtree_eagle3_patch_b200 import _lib
    sms = _lib.load().ddt_sm_count(torch.cuda.current_device())
    mtiles = -(-N_VERIFY // (128 // (HQ // HKV)))
    n_kt = -(-(PAST + N_VERIFY) // 128)
    return max(1, min(n_kt, sms // (HKV * mtiles)))


def _physical_index(local: int) -> int:
    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    if vis:
        parts = vis.split(",")
        if local < len(parts) and parts[local].strip().isdigit():
            return int(parts[local])
    return local


def _peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": float(d["hbm_gbs"]), "bf16_tflops": float(d["bf16_tflops"]), "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "source": "fallback"}


def _profile_traffic(f: Path, field: str = "traffic_bytes_per_launch:"):
    """DRAM bytes per launch (ncu dram__bytes_read.sum + dram__bytes_write.sum)
    from a committed profile summary's ``field`` line, or None."""
    if not f.exists():
        return None
    for line in f.read_text().splitlines():
        if line.startswith(field):
            try:
                return int(line.split(":", 1)[1].strip().split()[0])
            except ValueError:
                return None
    return None


def _profiled_traffic():
    """DRAM bytes per attention launch from the committed ncu summary, or None."""
    return _profile_traffic(ROOT / "profiles" / "tree_attn_split_kernel_qwen3_4b_verify.md",
                            "traffic_bytes_per_layer:")


# ----------------------------------------------------------------------------
# the reference's CPU path
# ----------------------------------------------------------------------------
def _cpu_step_inputs(layers_alloc: int, attn_layers: int):
    from ddtree_eagle3_patch_b200.synthetic import cfg1_logits, posterior_for_tree, verify_logits_for_posterior
    from oracle import cpu_reference as C
    draft = cfg1_logits(seed=0)
    toks, deps, parents, cm, vis = C.build_tree(draft, BUDGET)
    top = torch.topk(draft, 1, dim=-1).indices.numpy()
    post = posterior_for_tree(toks, deps, np.repeat(top, 1, axis=1), VOCAB, seed=0)
    verify = verify_logits_for_posterior(post, VOCAB, seed=0)[None]
    g = torch.Generator().manual_seed(5)
    base_k = (torch.randn(1, HKV, PAST + N_VERIFY, HD, generator=g) * HD ** -0.5).to(torch.bfloat16)
    base_v = torch.randn(1, HKV, PAST + N_VERIFY, HD, generator=g).to(torch.bfloat16)
    ks = [base_k.clone() for _ in range(layers_alloc)]
    vs = [base_v.clone() for _ in range(layers_alloc)]
    qs = [torch.randn(1, HQ, N_VERIFY, HD, generator=g).to(torch.bfloat16) for _ in range(attn_layers)]
    return C.CpuStep(draft, verify, qs, ks, vs, PAST, BUDGET, HD ** -0.5, LAYERS)


def cpu_step_seconds(step, attn_layers: int):
    r = step.run(attn_layers)
    return r["build"] + r["accept_compact"] + r["attention"] * LAYERS / attn_layers, r


def cpu_baseline(sample_steps: int, attn_layers: int):
    torch.set_num_threads(os.cpu_count() or 1)
    step = _cpu_step_inputs(LAYERS, attn_layers)
    cpu_step_seconds(step, attn_layers)  # warm
    secs = [cpu_step_seconds(step, attn_layers)[0] for _ in range(sample_steps)]
    s = statistics.median(secs)
    return {"value": round(1.0 / s, 4), "unit": UNIT, "cores": torch.get_num_threads(), "kind": "port",
            "sample": (f"{sample_steps} steps; per step the full tree build, accept and 72-tensor compaction "
                       f"plus {attn_layers} of {LAYERS} attention layers, attention time scaled x{LAYERS // attn_layers}"),
            "s_per_step": round(s, 4)}


def run_reference(args, rank, world, local):
    if world > 1:
        init_dist(world, "gloo")
        import torch.distributed as dist
        dist.barrier()
        if rank != 0:
            return None
    torch.set_num_threads(os.cpu_count() or 1)
    attn_layers = 2
    step = _cpu_step_inputs(LAYERS, attn_layers)
    for _ in range(args.warmup):
        cpu_step_seconds(step, attn_layers)
    t0 = time.perf_counter()
    secs = [cpu_step_seconds(step, attn_layers)[0] for _ in range(args.steps)]
    wall = time.perf_counter() - t0
    s = sum(secs) / len(secs)
    value = 1.0 / s
    sample = (f"each step: full tree build, accept and 72-tensor compaction plus {attn_layers} of {LAYERS} "
              f"attention layers (bf16 SDPA with repeat_kv and the dense mask), attention scaled x{LAYERS // attn_layers}")
    return {"metric": METRIC, "value": round(value, 4), "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(s * 1e3, 3), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic", "impl": "reference",
            "config": {"workload": WORKLOAD, "parallelism": "host CPU, rank 0"},
            "cpu_baseline": {"value": round(value, 4), "unit": UNIT, "cores": torch.get_num_threads(),
                             "kind": "port", "sample": sample},
            "e2e": {"value": round(value, 4), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "wall_s": round(wall, 2)}


def run_kernel_only(args, local):
    """One kernel of the step on the bench workload, eager launches."""
    from ddtree_eagle3_patch_b200 import kernels
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    w = Workload(device, seed=1000)
    tree = kernels.tree_build(w.draft[0], BUDGET)
    lp, ids = tree.top_lp.clone(), tree.top_ids.clone()
    exp_tree = kernels.DeviceTree.allocate(ROWS, lp.shape[1], BUDGET, device)   # outputs reused every launch
    acc, info, post = kernels.tree_accept(w.verify[0], tree.parents, tree.node_token_ids, tree.info,
                                          max_accept=ROWS + 1)
    tensors = [t for pair in zip(w.ks, w.vs) for t in pair]
    acc_bufs_sample = torch.empty(N_VERIFY, dtype=torch.int64, device=device)
    if args.kernel == "gemm":
        # the decode round's gate/up GEMM: 33 verify rows x [2 * 9728, 2560]
        # bf16, 36 different weights in turn (3.6 GB: every launch from HBM)
        gg = torch.Generator(device=device).manual_seed(21)
        gws = [(torch.randn((2 * 9728, 2560), generator=gg, device=device) * 0.02).to(torch.bfloat16)
               for _ in range(LAYERS)]
        gxs = [torch.randn((33, 2560), generator=gg, device=device).to(torch.bfloat16) for _ in range(LAYERS)]
        gys = [torch.empty((33, 9728), dtype=torch.bfloat16, device=device) for _ in range(LAYERS)]

    def once(i):
        if args.kernel == "gemm":
            kernels.wgemm_gate_up(gxs[i % LAYERS], gws[i % LAYERS], out=gys[i % LAYERS])
        elif args.kernel == "attention":
            layer = i % LAYERS
            kernels.tree_attention(w.qs[layer], w.ks[layer], w.vs[layer], PAST, tree.visibility, w.scale,
                                   out=w.outs[layer])
        elif args.kernel == "tree_build":
            kernels.tree_build(w.draft[i % 2], BUDGET, out=tree)
        elif args.kernel == "sample":
            # temperature 1 draw of every verify row (the accept path at temperature > 0)
            kernels.sample_rows(w.verify[i % 2], 1.0, seed=1234, offset=i, out=acc_bufs_sample)
        elif args.kernel == "expand":
            kernels.tree_from_log_probs(lp, ids, BUDGET, out=exp_tree)
        elif args.kernel == "accept":
            # the step's own preallocated outputs: no allocation or fill per launch
            kernels.tree_accept(w.verify[i % 2], tree.parents, tree.node_token_ids, tree.info, max_accept=ROWS + 1,
                                accepted=acc, accept_info=info, posterior=post)
        else:
            kernels.kv_compact(tensors, PAST, N_VERIFY, acc, info[:1], ROWS + 1)

    for i in range(args.warmup):
        once(i)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for i in range(args.steps):
        once(i)
    e1.record()
    torch.cuda.synchronize()
    eager_us = e0.elapsed_time(e1) * 1e3 / args.steps
    # the same launches captured once in a CUDA graph: device time without launch gaps
    per_graph = LAYERS
    stream = torch.cuda.Stream(device)
    stream.wait_stream(torch.cuda.current_stream(device))
    g = torch.cuda.CUDAGraph()
    with torch.cuda.stream(stream):
        once(0)
        torch.cuda.synchronize()
        with torch.cuda.graph(g, stream=stream):
            for i in range(per_graph):
                once(i)
    torch.cuda.synchronize()
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize()
    reps = max(1, args.steps // per_graph)
    with torch.cuda.stream(stream):
        e0.record(stream)
        for _ in range(reps):
            g.replay()
        e1.record(stream)
    torch.cuda.synchronize()
    graph_us = e0.elapsed_time(e1) * 1e3 / (reps * per_graph)
    del g
    print(json.dumps({"kernel": args.kernel, "launches": args.steps,
                      "us_per_launch_eager": round(eager_us, 3), "us_per_launch_graph": round(graph_us, 3),
                      "attention_status": kernels.attention_status(device)}))


# ----------------------------------------------------------------------------
# decode workload (end-to-end ddtree_generate)
# ----------------------------------------------------------------------------
def _decode_workload(new_tokens: int) -> str:
    return (f"DDTree decode, random-init {DEC_SHAPE} target (36 layers, hidden 2560, intermediate 9728, 32/8 heads, "
            f"vocab 151936) + {DEC_DRAFT_LAYERS}-layer DFlash draft, block {DEC_BLOCK}, budget {DEC_BUDGET}, "
            f"prompt {DEC_PROMPT} random ids, {new_tokens} new tokens, greedy, batch 1")


def _decode_prompts(rank: int, count: int, mask_id: int):
    from ddtree_eagle3_patch_b200.synthetic import random_prompt
    # rank r decodes prompts r, r + world, ... of one seeded list (benchmark.py:175)
    return [random_prompt(DEC_PROMPT, seed=7000 + 64 * i + rank, exclude=mask_id) for i in range(count)]


def _attention_roofline_at(device, past: int, n: int, reps: int = 20):
    """The tree-attention op at one verify shape, 36 layers per graph replay
    (inputs larger than L2 across the 36 layers of K/V at long prefixes)."""
    from ddtree_eagle3_patch_b200 import kernels
    from ddtree_eagle3_patch_b200.synthetic import random_tree
    g = torch.Generator(device=device).manual_seed(3)
    ks = [torch.randn((HKV, past + n, HD), generator=g, device=device).mul_(HD ** -0.5).to(torch.bfloat16)
          for _ in range(LAYERS)]
    vs = [torch.randn((HKV, past + n, HD), generator=g, device=device).to(torch.bfloat16) for _ in range(LAYERS)]
    qs = [torch.randn((n, HQ, HD), generator=g, device=device).to(torch.bfloat16) for _ in range(LAYERS)]
    outs = [torch.empty((n, HQ, HD), dtype=torch.bfloat16, device=device) for _ in range(LAYERS)]
    _, _, vis = random_tree(n - 1, max_depth=16, seed=5)
    bits = kernels.mask_to_bits(torch.from_numpy(np.ascontiguousarray(vis)).to(device), 0, n)
    stream = torch.cuda.Stream(device)
    stream.wait_stream(torch.cuda.current_stream(device))
    with torch.cuda.stream(stream):
        for layer in range(LAYERS):
            kernels.tree_attention(qs[layer], ks[layer], vs[layer], past, bits, HD ** -0.5, out=outs[layer])
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            for layer in range(LAYERS):
                kernels.tree_attention(qs[layer], ks[layer], vs[layer], past, bits, HD ** -0.5, out=outs[layer])
        for _ in range(3):
            graph.replay()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(reps):
            graph.replay()
        e1.record(stream)
    torch.cuda.synchronize()
    us = e0.elapsed_time(e1) * 1e3 / (reps * LAYERS)
    alg = 2 * HKV * (past + n) * HD * 2 + 2 * n * HQ * HD * 2
    peaks = _peaks()
    achieved = alg / (us * 1e-6) / 1e9
    del graph
    return {"bound": "hbm", "kernel": f"tree attention op (split kernel + combine), prefix {past} + {n} rows",
            "achieved": round(achieved, 1), "peak": peaks["hbm_gbs"], "peak_source": peaks["source"],
            "unit": "GB/s", "frac": round(achieved / peaks["hbm_gbs"], 4), "algorithmic_bytes": alg,
            "us_per_launch": round(us, 3)}


def _gemm_roofline(target, device, rows: int, reps: int = 20):
    """The decode round's dominant kernel: the weight-streaming gate/up GEMM
    with the SiLU product in its epilogue (ddt_wgemm_gate_up), at the verify
    rows, over the 36 layers' own packed weights in turn (3.6 GB per graph
    replay, so every launch streams its 100 MB from HBM).  Algorithmic
    bytes per launch: the weight, the activations in and the product out."""
    from ddtree_eagle3_patch_b200 import kernels
    from ddtree_eagle3_patch_b200.fused_layers import packed_weights
    layers = list(target.model.layers)
    wps = [packed_weights(layer)[1] for layer in layers]
    H = wps[0].shape[1]
    inter = wps[0].shape[0] // 2
    g = torch.Generator(device=device).manual_seed(11)
    xs = [torch.randn((rows, H), generator=g, device=device).to(torch.bfloat16) for _ in layers]
    outs = [torch.empty((rows, inter), dtype=torch.bfloat16, device=device) for _ in layers]
    stream = torch.cuda.Stream(device)
    stream.wait_stream(torch.cuda.current_stream(device))
    with torch.cuda.stream(stream), kernels.pdl(False):
        for x, w, o in zip(xs, wps, outs):
            kernels.wgemm_gate_up(x, w, out=o)
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            for x, w, o in zip(xs, wps, outs):
                kernels.wgemm_gate_up(x, w, out=o)
        for _ in range(3):
            graph.replay()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(reps):
            graph.replay()
        e1.record(stream)
    torch.cuda.synchronize()
    us = e0.elapsed_time(e1) * 1e3 / (reps * len(layers))
    alg = wps[0].numel() * 2 + rows * H * 2 + rows * inter * 2
    peaks = _peaks()
    achieved = alg / (us * 1e-6) / 1e9
    del graph
    prof = ROOT / "profiles" / "wgemm_gate_up_qwen3_4b_verify.md"
    traffic = _profile_traffic(prof)
    return {"bound": "hbm", "kernel": f"wgemm_kernel gate/up + SiLU (ddt_wgemm_gate_up), {rows} rows x "
                                      f"[{2 * inter} x {H}] bf16 weight",
            "achieved": round(achieved, 1), "peak": peaks["hbm_gbs"], "peak_source": peaks["source"],
            "unit": "GB/s", "frac": round(achieved / peaks["hbm_gbs"], 4), "algorithmic_bytes": alg,
            "us_per_launch": round(us, 3), "timing": "CUDA events over 36-launch graph replays, serial launches",
            "traffic": traffic, "traffic_source": (f"profiles/{prof.name} (ncu, not this run)" if traffic else None)}


def _round_bytes(target, draft, context: int) -> int:
    """Algorithmic bytes of one decode round: every projection weight the
    verify and draft forwards stream (the draft reuses the target's lm_head,
    read again), and the K/V rows the attention reads at ``context``."""
    lin = lambda m: sum(x.weight.numel() * x.weight.element_size() for x in m.modules()
                        if isinstance(x, torch.nn.Linear))
    cfg = target.config
    kv = 2 * cfg.num_hidden_layers * cfg.num_key_value_heads * cfg.head_dim * 2 * context
    dkv = 2 * len(draft.layers) * cfg.num_key_value_heads * cfg.head_dim * 2 * context
    return lin(target) + lin(draft) + target.lm_head.weight.numel() * 2 + kv + dkv


def run_decode(args, rank, world, local):
    from ddtree_eagle3_patch_b200 import _lib, kernels
    from ddtree_eagle3_patch_b200 import distributed as D
    from ddtree_eagle3_patch_b200.ddtree import ddtree_generate
    from ddtree_eagle3_patch_b200.synthetic import build_decode_models
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    dist = init_dist(world, "nccl")
    t_build = time.perf_counter()
    target, draft = build_decode_models(DEC_SHAPE, device, torch.bfloat16, seed=0, draft_layers=DEC_DRAFT_LAYERS,
                                        block_size=DEC_BLOCK)
    t_build = time.perf_counter() - t_build
    mask_id = draft.mask_token_id
    n_prompts = args.warmup + 2 * args.steps
    host_prompts = [p.pin_memory() for p in _decode_prompts(rank, n_prompts, mask_id)]
    dev_prompts = [p.to(device) for p in host_prompts]
    lib = _lib.load()

    def gen(ids):
        return ddtree_generate(draft, target, ids, mask_token_id=mask_id, max_new_tokens=args.new_tokens,
                               block_size=DEC_BLOCK, stop_token_ids=None, temperature=0.0, tree_budget=DEC_BUDGET)

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    for i in range(args.warmup):
        gen(dev_prompts[i])
    barrier()
    # timed region: K calls, prompts resident on the device
    with ClockSampler(_physical_index(local)) as clocks:
        barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        if args.cuda_profiler_range:
            torch.cuda.profiler.start()
        e0.record()
        results = [gen(dev_prompts[args.warmup + i]) for i in range(args.steps)]
        e1.record()
        barrier()
        if args.cuda_profiler_range:
            torch.cuda.profiler.stop()
    # this library's kernels run in the timed calls: eager launches plus every
    # replay of the ones captured in the per-call graphs
    launches = sum(r.native_launches for r in results)
    clock = clocks.summary()
    elapsed_s = e0.elapsed_time(e1) / 1e3
    tokens = sum(r.num_output_tokens for r in results)
    rounds = sum(r.decode_rounds for r in results)
    decode_s = sum(r.time_per_output_token * r.num_output_tokens for r in results)
    stage = {k: sum(r.stage_times[k] for r in results) for k in ("draft", "tree_build", "tree_compile", "verify",
                                                                  "commit")}
    # the round's counters, one NCCL all-gather of a fixed-size vector
    counters = D.gather_counters([elapsed_s, tokens, rounds, decode_s, sum(r.time_to_first_token for r in results)],
                                 device=device)
    wall = float(counters[:, 0].max())
    total_tokens = float(counters[:, 1].sum())
    value = total_tokens / wall

    # e2e: prompt from pinned host memory, ids back on the host, inside the timed region
    barrier()
    h0, h1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    h0.record()
    e2e_tokens = 0
    for i in range(args.steps):
        ids = host_prompts[args.warmup + args.steps + i].to(device, non_blocking=True)
        r = gen(ids)
        e2e_tokens += r.num_output_tokens
    h1.record()
    barrier()
    e2e_c = D.gather_counters([h0.elapsed_time(h1) / 1e3, e2e_tokens], device=device)
    e2e_value = float(e2e_c[:, 1].sum()) / float(e2e_c[:, 0].max())

    # roofline of the round's dominant kernel (the weight-streaming GEMMs hold
    # about half of a round; the gate/up one is the largest), the tree
    # attention at the verify shape of mid-generation (prefix 512 + 512, 33
    # rows) beside it, and the round as a whole: algorithmic bytes per round
    # over the measured decode time per round
    roof = _gemm_roofline(target, device, DEC_BUDGET + 1)
    roof_attn = _attention_roofline_at(device, DEC_PROMPT + args.new_tokens // 2, DEC_BUDGET + 1)
    peaks = _peaks()
    round_s = decode_s / max(rounds, 1)
    round_bytes = _round_bytes(target, draft, DEC_PROMPT + args.new_tokens // 2)
    roof_round = {"bound": "hbm", "algorithmic_bytes_per_round": round_bytes, "ms_per_round": round(round_s * 1e3, 4),
                  "achieved": round(round_bytes / round_s / 1e9, 1), "peak": peaks["hbm_gbs"], "unit": "GB/s",
                  "frac": round(round_bytes / round_s / 1e9 / peaks["hbm_gbs"], 4),
                  "bytes": "verify + draft projection weights (lm_head read twice) + K/V at the mean context"}
    status = kernels.attention_status(device)
    out = None
    if rank == 0:
        acc = [a for r in results for a in r.acceptance_lengths]
        per_round_ms = {k: round(v / max(rounds, 1) * 1e3, 4) for k, v in stage.items()}
        out = {
            "metric": DEC_METRIC, "value": round(value, 2), "unit": DEC_UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(wall / args.steps * 1e3, 2),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (random-init weights, seeded uniform random prompt ids)",
            "config": {"workload": _decode_workload(args.new_tokens), "global_batch": world, "seq_len": DEC_PROMPT,
                       "parallelism": f"data parallel x{world} (prompts sharded by rank, one stream per GPU)",
                       "l2": "weights (8.1 GB per verify) larger than L2"},
            "decode_tok_s_excluding_prefill": round(float(counters[:, 1].sum()) / float(counters[:, 3].max()), 2),
            "time_to_first_token_ms": round(float(counters[:, 4].max()) / args.steps * 1e3, 2),
            "tokens_per_round": round(tokens / max(rounds, 1), 4),
            "acceptance_histogram": {str(k): acc.count(k) for k in sorted(set(acc))},
            "stage_ms_per_round": per_round_ms,
            "roofline": roof, "roofline_attention": roof_attn, "roofline_round": roof_round,
            "e2e": {"value": round(e2e_value, 2), "unit": DEC_UNIT, "h2d_bytes_per_step": DEC_PROMPT * 8,
                    "d2h_bytes_per_step": (DEC_PROMPT + args.new_tokens) * 8,
                    "api": "ddtree_eagle3_patch_b200.ddtree.ddtree_generate (host prompt in, host ids out)"},
            "gpu_launches": int(launches), "clocks": clock, "attention_status": status,
            "model_build_s": round(t_build, 1),
            "graph_capture_ms_per_call": round(1e3 * sum(r.graph_capture_s for r in results) / len(results), 2),
            "graph_rounds": sum(r.graph_rounds for r in results),
        }
        if world == 1 and not args.no_cpu_baseline:
            out["cpu_baseline"] = cpu_decode_baseline(rounds=2)
    if world > 1:
        dist.barrier()
    return out


DP_SHAPE, DP_PROMPTS, DP_NEW_TOKENS, DP_BUDGET, DP_LEN = "qwen3-8b", 64, 512, 64, (256, 2048)


def run_decode_dp(args, rank, world, local):
    """Data-parallel decoding over prompts at the Qwen3-8B shape: a seeded
    list of ``--prompts`` (default 64) uniform random prompts with lengths
    uniform in [256, 2048], 512 new tokens each, node budget 64, block 16;
    rank r decodes prompts r, r + N, ... (the reference shards its prompt
    list the same way, benchmark.py:175) and one NCCL all-gather of a fixed
    counter vector collects tokens and times.  ``value`` = every rank's
    generated tokens / the slowest rank's time."""
    from ddtree_eagle3_patch_b200 import distributed as D
    from ddtree_eagle3_patch_b200.ddtree import ddtree_generate
    from ddtree_eagle3_patch_b200.synthetic import build_decode_models, random_prompt
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    dist = init_dist(world, "nccl")
    target, draft = build_decode_models(DP_SHAPE, device, torch.bfloat16, seed=0, draft_layers=DEC_DRAFT_LAYERS,
                                        block_size=DEC_BLOCK)
    mask_id = draft.mask_token_id
    n_prompts = args.prompts or DP_PROMPTS
    lens = np.random.RandomState(8000).randint(DP_LEN[0], DP_LEN[1] + 1, size=n_prompts)
    mine = [random_prompt(int(lens[i]), seed=9000 + i, exclude=mask_id).to(device)
            for i in range(rank, n_prompts, world)]

    def gen(ids):
        return ddtree_generate(draft, target, ids, mask_token_id=mask_id, max_new_tokens=DP_NEW_TOKENS,
                               block_size=DEC_BLOCK, stop_token_ids=None, temperature=0.0, tree_budget=DP_BUDGET)

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    gen(random_prompt(DP_LEN[1], seed=1, exclude=mask_id).to(device))   # capture at the longest prompt
    barrier()
    with ClockSampler(_physical_index(local)) as clocks:
        barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        results = [gen(p) for p in mine]
        e1.record()
        barrier()
    elapsed = e0.elapsed_time(e1) / 1e3
    tokens = sum(r.num_output_tokens for r in results)
    rounds = sum(r.decode_rounds for r in results)
    c = D.gather_counters([elapsed, tokens, rounds, len(results)], device=device)
    wall = float(c[:, 0].max())
    out = None
    if rank == 0:
        out = {"metric": "decode tok/s (Qwen3-8B shape, prompts sharded over GPUs)",
               "value": round(float(c[:, 1].sum()) / wall, 2), "unit": DEC_UNIT, "n_gpus": world,
               "steps": int(c[:, 3].sum()), "warmup": 1, "ms_per_step": round(wall / max(len(results), 1) * 1e3, 2),
               "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
               "data": "synthetic (random-init weights, seeded uniform random prompt ids)",
               "config": {"workload": (f"DDTree decode, random-init {DP_SHAPE} target + {DEC_DRAFT_LAYERS}-layer "
                                       f"DFlash draft, block {DEC_BLOCK}, budget {DP_BUDGET}, {n_prompts} prompts of "
                                       f"U[{DP_LEN[0]}, {DP_LEN[1]}] random ids, {DP_NEW_TOKENS} new tokens each, "
                                       f"greedy, batch 1 per GPU"),
                          "global_batch": world, "parallelism": f"data parallel x{world} over prompts"},
               "per_rank_tokens": [int(x) for x in c[:, 1].tolist()],
               "per_rank_s": [round(float(x), 3) for x in c[:, 0].tolist()],
               "tokens_per_round": round(float(c[:, 1].sum()) / max(float(c[:, 2].sum()), 1.0), 4),
               "clocks": clocks.summary()}
    if world > 1:
        dist.barrier()
    return out


def _cpu_decode_models():
    from ddtree_eagle3_patch_b200.synthetic import dflash_config, target_config
    from oracle.cpu_decode import build_cpu_models
    tcfg = target_config(DEC_SHAPE)
    dcfg = dflash_config(tcfg, DEC_DRAFT_LAYERS, DEC_BLOCK)
    return build_cpu_models(tcfg, dcfg, torch.bfloat16, seed=0)


def _cpu_decode_estimate(prefill_s: float, rounds: list, new_tokens: int):
    per_round = sum(r["total"] for r in rounds) / len(rounds)
    tokens_per_round = sum(r["accepted"] for r in rounds) / len(rounds)
    call_s = prefill_s + new_tokens / tokens_per_round * per_round
    return new_tokens / call_s, per_round, tokens_per_round


def cpu_decode_baseline(rounds: int):
    """The reference's decode loop on the host (oracle/cpu_decode.py): one
    prefill of the 512-token prompt, then ``rounds`` decode rounds; the
    whole-call rate of the 1024-token workload is estimated from them."""
    from oracle.cpu_decode import CpuDecode
    torch.set_num_threads(os.cpu_count() or 1)
    target, draft = _cpu_decode_models()
    prompt = _decode_prompts(0, 1, draft.mask_token_id)[0]
    run = CpuDecode(draft, target, prompt, DEC_NEW_TOKENS, DEC_BLOCK, DEC_BUDGET)
    prefill_s = run.prefill()
    rec = [run.round() for _ in range(rounds)]
    value, per_round, tpr = _cpu_decode_estimate(prefill_s, rec, DEC_NEW_TOKENS)
    return {"value": round(value, 4), "unit": DEC_UNIT, "cores": torch.get_num_threads(), "kind": "port",
            "sample": (f"prefill of the {DEC_PROMPT}-token prompt plus {rounds} decode rounds of the reference loop; "
                       f"whole-call rate = {DEC_NEW_TOKENS} / (prefill + {DEC_NEW_TOKENS} / tokens-per-round x "
                       f"round time)"),
            "prefill_s": round(prefill_s, 3), "round_s": round(per_round, 3), "tokens_per_round": round(tpr, 3)}


def run_decode_reference(args, rank, world, local):
    """The reference arm of the decode workload: the reference's loop on the
    host cores (rank 0 only).  A step is one decode round after one shared
    prefill; ``value`` is the whole-call rate of the configured workload
    estimated from the measured prefill and the K timed rounds."""
    if world > 1:
        init_dist(world, "gloo")
        import torch.distributed as tdist
        tdist.barrier()
        if rank != 0:
            return None
    from oracle.cpu_decode import CpuDecode
    torch.set_num_threads(os.cpu_count() or 1)
    target, draft = _cpu_decode_models()
    prompt = _decode_prompts(0, 1, draft.mask_token_id)[0]
    run = CpuDecode(draft, target, prompt, DEC_NEW_TOKENS, DEC_BLOCK, DEC_BUDGET)
    prefill_s = run.prefill()
    for _ in range(args.warmup):
        run.round()
    t0 = time.perf_counter()
    rec = [run.round() for _ in range(args.steps)]
    wall = time.perf_counter() - t0
    value, per_round, tpr = _cpu_decode_estimate(prefill_s, rec, args.new_tokens)
    sample = (f"one prefill of the {DEC_PROMPT}-token prompt ({prefill_s:.2f} s), {args.warmup} untimed and "
              f"{args.steps} timed decode rounds ({per_round:.3f} s each, {tpr:.2f} tokens per round); value = "
              f"{args.new_tokens} / (prefill + {args.new_tokens} / tokens-per-round x round time)")
    return {"metric": DEC_METRIC, "value": round(value, 4), "unit": DEC_UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(per_round * 1e3, 2), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (random-init weights, seeded uniform random prompt ids)", "impl": "reference",
            "config": {"workload": _decode_workload(args.new_tokens), "parallelism": "host CPU, rank 0"},
            "cpu_baseline": {"value": round(value, 4), "unit": DEC_UNIT, "cores": torch.get_num_threads(),
                             "kind": "port", "sample": sample},
            "e2e": {"value": round(value, 4), "unit": DEC_UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "stage_s_per_round": {k: round(sum(r[k] for r in rec) / len(rec), 4)
                                  for k in ("draft", "tree_build", "tree_compile", "verify", "commit")},
            "wall_s": round(wall, 2)}


def main():
    args = parse()
    rank, world, local = dist_env()
    if args.kernel:
        run_kernel_only(args, local)
        return
    if args.workload == "decode-dp":
        out = {"impl": "reference", "unavailable": "the Qwen3-8B data-parallel workload has no CPU arm (hours of "
                                                   "CPU time per prompt); its reference arm is the decode workload's"} \
            if args.impl == "reference" else run_decode_dp(args, rank, world, local)
    elif args.workload == "decode":
        out = run_decode_reference(args, rank, world, local) if args.impl == "reference" else \
            run_decode(args, rank, world, local)
    elif args.impl == "reference":
        out = run_reference(args, rank, world, local)
    else:
        out = run_ours(args, rank, world, local)
    if rank == 0 and out is not None:
        print(json.dumps(out), flush=True)
    try:
        import torch.distributed as dist
        if dist.is_initialized():
            dist.destroy_process_group()
    except Exception:
        pass


if __name__ == "__main__":
    main()
