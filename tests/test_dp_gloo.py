"""Data-parallel plumbing on two CPU processes (gloo): prompt sharding,
gather / all_gather conventions and counter merging, as the reference's
harness uses them (benchmark.py:175, 237-241; distributed.py:55-72)."""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

WORLD = 2


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank: int, world: int, port: int, n_prompts: int, out, ready):
    os.environ.update({"RANK": str(rank), "WORLD_SIZE": str(world), "LOCAL_RANK": str(rank),
                       "LOCAL_WORLD_SIZE": str(world), "MASTER_ADDR": "127.0.0.1", "MASTER_PORT": str(port)})
    from datetime import timedelta
    from ddtree_eagle3_patch_b200 import distributed as dist
    ready.wait(timeout=300)   # both ranks imported: the rendezvous does not wait on a cold import
    dist.init(backend="gloo", timeout=timedelta(seconds=300))
    try:
        mine = list(dist.shard_indices(n_prompts))
        # per-prompt "results": accepted lengths derived from the prompt index
        responses = [{"idx": i, "accepted": (i % 5) + 1} for i in mine]
        counters = {"prompts": len(mine), "accepted": sum(r["accepted"] for r in responses), "steps": len(mine) * 3}
        gathered = dist.gather(responses, dst=0)
        everyone = dist.all_gather(counters)
        dist.barrier()
        out.put((rank, mine, gathered, everyone, dist.is_main()))
    finally:
        torch.distributed.destroy_process_group()


@pytest.mark.parametrize("n_prompts", [0, 1, 7, 80])
def test_sharding_gather_and_counters(n_prompts):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ready = ctx.Barrier(WORLD)
    procs = [ctx.Process(target=_worker, args=(r, WORLD, port, n_prompts, q, ready)) for r in range(WORLD)]
    for p in procs:
        p.start()
    results = {}
    for _ in range(WORLD):
        rank, mine, gathered, everyone, main = q.get(timeout=300)
        results[rank] = (mine, gathered, everyone, main)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    # every prompt is decoded by exactly one rank, rank r taking r, r + W, ...
    shards = [results[r][0] for r in range(WORLD)]
    assert sorted(i for s in shards for i in s) == list(range(n_prompts))
    for r in range(WORLD):
        assert shards[r] == list(range(r, n_prompts, WORLD))
    # gather: rank-ordered lists on rank 0, None elsewhere
    assert results[0][3] and not results[1][3]
    assert results[1][1] is None
    gathered = results[0][1]
    assert [[x["idx"] for x in part] for part in gathered] == shards
    # all_gather: the same rank-ordered counters everywhere, merged to totals
    from ddtree_eagle3_patch_b200.distributed import merge_counters
    assert results[0][2] == results[1][2]
    total = merge_counters(results[0][2])
    assert total["prompts"] == n_prompts
    assert total["accepted"] == sum((i % 5) + 1 for i in range(n_prompts))
    assert total["steps"] == 3 * n_prompts


def test_single_process_fallbacks(monkeypatch):
    """Without RANK the reference warns and runs alone: gather returns [obj]."""
    from ddtree_eagle3_patch_b200 import distributed as dist
    monkeypatch.delenv("RANK", raising=False)
    monkeypatch.delenv("WORLD_SIZE", raising=False)
    with pytest.warns(UserWarning):
        dist.init(backend="gloo")
    assert not dist.is_initialized()
    assert dist.size() == 1 and dist.rank() == 0 and dist.is_main()
    assert dist.gather({"a": 1}) == [{"a": 1}]
    assert dist.all_gather(3) == [3]
    dist.barrier()
    assert list(dist.shard_indices(5)) == [0, 1, 2, 3, 4]
    with pytest.raises(ValueError):
        dist.shard_indices(5, rank_=2, size_=2)


def _counter_worker(rank: int, world: int, port: int, out, ready):
    os.environ.update({"RANK": str(rank), "WORLD_SIZE": str(world), "LOCAL_RANK": str(rank),
                       "MASTER_ADDR": "127.0.0.1", "MASTER_PORT": str(port)})
    from datetime import timedelta
    from ddtree_eagle3_patch_b200 import distributed as dist
    ready.wait(timeout=300)   # both ranks imported: the rendezvous does not wait on a cold import
    dist.init(backend="gloo", timeout=timedelta(seconds=300))
    try:
        # tokens, rounds, seconds: one fixed-size vector per rank
        m = dist.gather_counters([100.0 * (rank + 1), 10.0 + rank, 0.5 * (rank + 1)])
        out.put((rank, m.tolist()))
    finally:
        torch.distributed.destroy_process_group()


def test_gather_counters_one_collective():
    """The end-of-run counter exchange: one all-gather of a fixed-size
    float64 vector per rank, the same [world, n] matrix on every rank."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ready = ctx.Barrier(WORLD)
    procs = [ctx.Process(target=_counter_worker, args=(r, WORLD, port, q, ready)) for r in range(WORLD)]
    for p in procs:
        p.start()
    got = dict(q.get(timeout=300) for _ in range(WORLD))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    expect = [[100.0, 10.0, 0.5], [200.0, 11.0, 1.0]]
    assert got[0] == expect and got[1] == expect


def _failing_worker(rank: int, world: int, port: int, mode: str, out, ready):
    """Rank 1 fails between steps (exits, raises, or stalls); rank 0 goes on
    to the next step's collective and must get an error within the process
    group's timeout instead of waiting for ever."""
    import time
    os.environ.update({"RANK": str(rank), "WORLD_SIZE": str(world), "LOCAL_RANK": str(rank),
                       "MASTER_ADDR": "127.0.0.1", "MASTER_PORT": str(port)})
    from datetime import timedelta
    from ddtree_eagle3_patch_b200 import distributed as dist
    # both ranks have imported everything before the rendezvous starts, so
    # the short timeout below measures the failure, not a slow import
    ready.wait(timeout=300)
    try:
        dist.init(backend="gloo", timeout=timedelta(seconds=3))
    except Exception:                            # noqa: BLE001 - a loaded host missed the short rendezvous
        if rank == 0:
            out.put(("set-up failed", 0.0))
        os._exit(0)
    t0 = time.perf_counter()
    try:
        dist.gather_counters([1.0, 2.0])        # step 1 on both ranks
        if rank == 1:
            time.sleep(0.5)                      # let rank 0 finish receiving step 1
            if mode == "exit":
                os._exit(0)
            if mode == "raise":
                raise RuntimeError("rank 1 failed between steps")
            time.sleep(60)                       # stall: never joins step 2
            os._exit(0)
        t0 = time.perf_counter()
        dist.gather_counters([3.0, 4.0])        # step 2: the peer is gone
        out.put(("no error", time.perf_counter() - t0))
    except Exception as exc:                    # noqa: BLE001 - any error type is a detected failure
        if rank == 0:
            out.put((type(exc).__name__, time.perf_counter() - t0))
    os._exit(0)


@pytest.mark.parametrize("mode", ["exit", "raise", "stall"])
def test_failed_rank_is_detected_by_the_next_collective(mode):
    ctx = mp.get_context("spawn")
    # the group's short timeout also bounds its set-up: on a loaded host a
    # missed rendezvous is reported as such and the scenario starts over
    for _attempt in range(3):
        q = ctx.Queue()
        port = _free_port()
        ready = ctx.Barrier(WORLD)
        procs = [ctx.Process(target=_failing_worker, args=(r, WORLD, port, mode, q, ready)) for r in range(WORLD)]
        for p in procs:
            p.start()
        kind, waited = q.get(timeout=360)   # cold imports in a fresh container take minutes
        for p in procs:
            p.join(timeout=5)
            if p.is_alive():
                p.kill()
                p.join(timeout=5)
        if kind != "set-up failed":
            break
    assert kind not in ("no error", "set-up failed")
    assert waited < 30.0, waited
